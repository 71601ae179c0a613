"""A paged decode step captured once as a CUDA graph and replayed every step.

The reference's step loop (core/model_runner.py:28-159) rebuilds its metadata
in Python, writes each new K/V row with a dozen launches and two host
synchronisations per token (transformer/model.py:85-122), converts the block
table dict to a tensor with ``.item()`` calls (:126-152) and only then runs
the kernel.  ``DecodeStepGraph`` replaces all of that for the decode rows of a
step with one graph replay:

  1. one host-to-device copy of the step's per-sequence values (pool slot and
     length) from a fixed pinned staging buffer;
  2. ``block_pool_step``: padded block table, block counts and each new
     token's position and row, from the device-resident block pool;
  3. ``write_kv``: the new K/V rows into the paged cache (quantise-on-write for
     INT8 pools);
  4. paged attention of every sequence's new query over its whole cache.

Decode positions follow the sequence: a sequence holding ``n`` tokens after
this step's append writes its new token at position ``n - 1`` and attends to
``n`` keys (the reference runner puts it at ``n``, one past, with ``n + 1``
keys, core/model_runner.py:96-97).

The graph has fixed shapes: ``max_seqs`` rows.  A step with fewer sequences
fills the remaining rows with a reserved one-block sequence that writes and
reads only its own block, so padding never touches real cache rows.  Block
allocation stays with the caller's scheduler (``pool.allocate``) or is done by
``step`` itself for sequences that cross a block boundary; the queued pool
operations are applied (one launch) before the replay.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

from . import ops
from .block_pool import AllocStatus, DeviceBlockManager


class DecodeStepGraph:
    """Decode rows of one attention layer as a captured CUDA graph (see the module docstring)."""

    PAD_SEQ = -1  # the reserved padding sequence's id in the pool

    def __init__(self, pool: DeviceBlockManager, k_cache: torch.Tensor, v_cache: torch.Tensor,
                 k_scale: Optional[torch.Tensor], v_scale: Optional[torch.Tensor], num_q_heads: int, max_seqs: int,
                 q_dtype: torch.dtype = torch.float16):
        self.pool = pool
        self.K, self.V, self.ks, self.vs = k_cache, v_cache, k_scale, v_scale
        self.dev = k_cache.device
        NB, BS, Hkv, D = k_cache.shape
        self.BS, self.Hkv, self.D, self.Hq = BS, Hkv, D, int(num_q_heads)
        self.S = int(max_seqs)
        self.cols = pool.max_blocks_per_seq
        if pool.ledger.allocate(self.PAD_SEQ, 1)[0] is not AllocStatus.SUCCESS:
            raise RuntimeError("the pool has no free block for the padding sequence")
        pool.flush()
        i32 = dict(dtype=torch.int32, device=self.dev)
        S = self.S
        # inputs the caller's step fills (device) and the per-step host values (pinned)
        self.q = torch.zeros(S, self.Hq, 1, D, dtype=q_dtype, device=self.dev)
        self.k_new = torch.zeros(S, Hkv, D, dtype=q_dtype, device=self.dev)
        self.v_new = torch.zeros(S, Hkv, D, dtype=q_dtype, device=self.dev)
        # two pinned staging buffers and two graphs, used by alternate steps: a
        # step fills the buffer the replay two steps back read, after that
        # replay's event, so the host never waits for the step just enqueued
        self.staging = [torch.zeros(2 * S, dtype=torch.int32).pin_memory() for _ in range(2)]
        self.events: list = [None, None]
        self.meta = torch.zeros(2 * S, **i32)               # [slots | kv_len]
        self.q_len = torch.ones(S, **i32)
        self.cu = torch.arange(S + 1, **i32)
        self.block_table = torch.zeros(S, self.cols, **i32)
        self.num_blocks = torch.zeros(S, **i32)
        self.positions = torch.zeros(S, **i32)
        self.token_seq = torch.zeros(S, **i32)
        self.out = torch.zeros(S, self.Hq, 1, D, dtype=torch.float16, device=self.dev)
        self.lse = torch.zeros(S, self.Hq, 1, dtype=torch.float16, device=self.dev)
        self.status = torch.zeros(1, **i32)
        self.graphs: Optional[list] = None
        self.n_steps = 0
        for k in range(2):
            self._fill(k, [], [])

    # ---- the captured work -------------------------------------------------
    def _body(self, k: int) -> None:
        S = self.S
        self.meta.copy_(self.staging[k], non_blocking=True)
        slots, kv_len = self.meta[:S], self.meta[S:]
        self.pool.step_rows(slots, self.q_len, kv_len, self.cu, S, self.block_table, self.num_blocks, self.positions,
                            self.token_seq, self.status)
        ops.write_kv(self.k_new, self.v_new, self.block_table, self.token_seq, self.positions, self.K, self.V, self.ks,
                     self.vs, status=self.status)
        ops.paged_attention(self.q, self.K, self.V, self.q_len, self.block_table, self.num_blocks, self.BS, kv_len,
                            self.ks, self.vs, out=self.out, lse=self.lse, mode="decode", status=self.status)

    def capture(self) -> None:
        """Run the step body once eagerly (workspaces, library state), then capture it twice."""
        stream = torch.cuda.Stream(self.dev)
        stream.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(stream):
            self._body(0)
        torch.cuda.current_stream(self.dev).wait_stream(stream)
        torch.cuda.synchronize(self.dev)
        self.graphs = []
        for k in range(2):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._body(k)
            self.graphs.append(g)

    # ---- one step ----------------------------------------------------------
    def _fill(self, k: int, seq_ids: Sequence[int], seq_lens: Sequence[int]) -> None:
        S, n = self.S, len(seq_ids)
        st = self.staging[k].numpy()  # the pinned buffer itself
        st[:n] = [self.pool.slot_of(int(x)) for x in seq_ids]
        st[n:S] = self.pool.slot_of(self.PAD_SEQ)
        st[S:S + n] = [int(x) for x in seq_lens]
        st[S + n:] = 1

    def step(self, seq_ids: Sequence[int], seq_lens: Sequence[int], q: torch.Tensor, k_new: torch.Tensor,
             v_new: torch.Tensor) -> torch.Tensor:
        """Append one token to each of ``seq_ids`` and attend.

        ``seq_lens[i]``: tokens of sequence i including this step's;
        ``q`` [n, Hq, D], ``k_new`` / ``v_new`` [n, Hkv, D] on the device.
        Returns O [n, Hq, D] (float16), a view of the graph's output buffer:
        consume it before the next ``step``.
        """
        n = len(seq_ids)
        if n > self.S:
            raise ValueError(f"{n} sequences, the graph holds {self.S}")
        if self.graphs is None:
            self.capture()
        for sid, ln in zip(seq_ids, seq_lens):
            need = -(-int(ln) // self.BS) - self.pool.blocks_of(int(sid))
            if need > 0 and self.pool.allocate(int(sid), need).status is not AllocStatus.SUCCESS:
                raise RuntimeError(f"no free block for sequence {sid}")
        self.pool.flush()
        k = self.n_steps & 1
        if self.events[k] is not None:
            self.events[k].synchronize()  # the replay two steps back has copied staging[k]
        self._fill(k, seq_ids, seq_lens)
        self.q[:n, :, 0].copy_(q)
        self.k_new[:n].copy_(k_new)
        self.v_new[:n].copy_(v_new)
        self.graphs[k].replay()
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.dev))
        self.events[k] = ev
        self.n_steps += 1
        return self.out[:n, :, 0]

    def check(self) -> None:
        """Raise if a replay reported a device status bit (reads the device)."""
        ops._raise_status("decode step", self.status)
