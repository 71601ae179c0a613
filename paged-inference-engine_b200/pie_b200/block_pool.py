"""Device-resident block pool with the reference BlockManager's interface.

The reference keeps the free list and every sequence's block list in Python
(core/block_manager.py:19-68) and rebuilds a padded int32 block table from
that dict on every step with host loops and ``.item()`` calls
(transformer/model.py:126-152), next to host-built step metadata
(core/model_runner.py:66-107).  Here the free list, the per-sequence lists and
the padded table live in device memory:

* ``DeviceBlockManager.allocate`` / ``release_blocks`` / ``num_free_blocks`` /
  ``can_allocate`` keep the reference's names, arguments and statuses.  The
  statuses are decided on the host, which tracks how many blocks are free and
  which sequences hold blocks (the decisions the reference makes,
  core/block_manager.py:32-33,49-50); the block ids themselves exist only on
  the device.  Calls are queued and applied in order by one launch at
  ``flush()`` (``block_pool_apply``), so a scheduler step costs one launch and
  one small host-to-device copy, whatever the number of calls.
* ``step_inputs(...)`` builds a step's attention inputs on the device
  (``block_pool_step``): the zero-padded block table and ``num_blocks_per_seq``
  of the scheduled sequences, and each query token's position and row.

``AllocResult.block_ids`` is a device tensor (the ids the call appended, valid
once the queued operations have been flushed) rather than a host list.
"""
from __future__ import annotations

import ctypes
import enum
from dataclasses import dataclass
from typing import Optional, Sequence

import torch

from . import _lib


class AllocStatus(enum.Enum):
    """core/block_manager.py:9-12."""

    SUCCESS = 0
    INSUFFICIENT_SPACE = 1
    FAILURE = 2


@dataclass
class AllocResult:
    status: AllocStatus
    block_ids: Optional[torch.Tensor]


class PaBlockPool(ctypes.Structure):
    """Mirror of pa_block_pool_t."""

    _fields_ = [("free_stack", ctypes.c_void_p), ("free_top", ctypes.c_void_p), ("table", ctypes.c_void_p),
                ("count", ctypes.c_void_p), ("table_stride", ctypes.c_int64), ("num_blocks", ctypes.c_int32),
                ("max_seqs", ctypes.c_int32), ("max_blocks_per_seq", ctypes.c_int32), ("_reserved", ctypes.c_int32)]


POOL_ALLOCATE, POOL_RELEASE = 0, 1


class BlockLedger:
    """Host half of the pool: the decisions the reference's BlockManager makes, without the ids.

    Tracks how many blocks are free, how many each sequence holds and which
    table row (slot) it uses, decides every call's status exactly as
    core/block_manager.py:29-57 does, and queues the (kind, slot, n)
    operations the device applies in the same order.
    """

    def __init__(self, num_blocks: int, max_seqs: int, max_blocks_per_seq: int):
        self.num_blocks = int(num_blocks)
        self.max_seqs = int(max_seqs)
        self.max_blocks_per_seq = int(max_blocks_per_seq)
        self.free = self.num_blocks
        self.blocks: dict[int, int] = {}      # seq_id -> blocks held
        self.slot: dict[int, int] = {}        # seq_id -> table row
        self.free_slots = list(range(self.max_seqs - 1, -1, -1))
        self.ops: list[tuple[int, int, int]] = []

    def allocate(self, seq_id: int, num_blocks: int) -> tuple[AllocStatus, int, int]:
        """Returns (status, slot, first new column); queues the operation on success."""
        num_blocks = int(num_blocks)
        if num_blocks < 0:
            raise ValueError("num_blocks must be >= 0")
        if self.free < num_blocks:
            return AllocStatus.INSUFFICIENT_SPACE, -1, 0
        held = self.blocks.get(seq_id)
        base = held or 0
        if base + num_blocks > self.max_blocks_per_seq:
            raise ValueError(f"sequence {seq_id} would hold {base + num_blocks} blocks, more than "
                             f"max_blocks_per_seq={self.max_blocks_per_seq}")
        if held is None:
            if not self.free_slots:
                raise RuntimeError(f"more than max_seqs={self.max_seqs} sequences hold blocks")
            self.slot[seq_id] = self.free_slots.pop()
        slot = self.slot[seq_id]
        self.ops.append((POOL_ALLOCATE, slot, num_blocks))
        self.blocks[seq_id] = base + num_blocks
        self.free -= num_blocks
        return AllocStatus.SUCCESS, slot, base

    def release(self, seq_id: int) -> AllocStatus:
        if seq_id not in self.blocks:
            return AllocStatus.FAILURE
        slot = self.slot.pop(seq_id)
        self.ops.append((POOL_RELEASE, slot, 0))
        self.free += self.blocks.pop(seq_id)
        self.free_slots.append(slot)
        return AllocStatus.SUCCESS

    def take_ops(self) -> list[tuple[int, int, int]]:
        ops, self.ops = self.ops, []
        return ops


class DeviceBlockManager:
    """The paged pool's bookkeeping in device memory (see the module docstring).

    ``max_seqs`` sequences may hold blocks at once, each at most
    ``max_blocks_per_seq``; both size the device table
    ``[max_seqs, max_blocks_per_seq]`` (int32).
    """

    def __init__(self, num_blocks: int, block_size: int, max_seqs: int, max_blocks_per_seq: int,
                 device: torch.device | str = "cuda"):
        self.num_blocks = int(num_blocks)
        self.block_size = int(block_size)
        self.max_seqs = int(max_seqs)
        self.max_blocks_per_seq = int(max_blocks_per_seq)
        self.device = torch.device(device)
        i32 = dict(dtype=torch.int32, device=self.device)
        self.free_stack = torch.empty(max(1, self.num_blocks), **i32)
        self.free_top = torch.empty(1, **i32)
        self.table = torch.empty(max(1, self.max_seqs), max(1, self.max_blocks_per_seq), **i32)
        self.count = torch.empty(max(1, self.max_seqs), **i32)
        self.status = torch.zeros(1, **i32)
        self._desc = PaBlockPool(self.free_stack.data_ptr(), self.free_top.data_ptr(), self.table.data_ptr(),
                                 self.count.data_ptr(), self.table.stride(0), self.num_blocks, self.max_seqs,
                                 self.max_blocks_per_seq, 0)
        self.ledger = BlockLedger(self.num_blocks, self.max_seqs, self.max_blocks_per_seq)
        self._results: Optional[torch.Tensor] = None
        lib = _lib.load()
        with torch.cuda.device(self.device):
            _lib.check("block_pool_init", lib.block_pool_init(ctypes.byref(self._desc), self._stream()))

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    # ---- the reference interface (core/block_manager.py) --------------------
    def allocate(self, seq_id: int, num_blocks: int) -> AllocResult:
        """core/block_manager.py:29-44: take ``num_blocks`` ids off the free list for ``seq_id``."""
        st, slot, base = self.ledger.allocate(seq_id, num_blocks)
        if st is not AllocStatus.SUCCESS:
            return AllocResult(st, None)
        return AllocResult(st, self.table[slot, base:base + int(num_blocks)])

    def release_blocks(self, seq_id: int) -> AllocStatus:
        """core/block_manager.py:47-57: return ``seq_id``'s blocks to the free list."""
        return self.ledger.release(seq_id)

    def num_free_blocks(self) -> int:
        return self.ledger.free

    def can_allocate(self, num_blocks: int) -> bool:
        return self.ledger.free >= num_blocks

    # ---- device side --------------------------------------------------------
    def flush(self, keep_results: bool = False) -> None:
        """Apply the queued allocate / release calls on the device, in order, in one launch.

        ``keep_results``: keep the per-call device statuses (``last_results``)
        for checking against the host's decisions.
        """
        ops_list = self.ledger.take_ops()
        if not ops_list:
            return
        n = len(ops_list)
        host = torch.tensor(ops_list, dtype=torch.int32).pin_memory()
        ops = host.to(self.device, non_blocking=True)
        res = torch.empty(n, dtype=torch.int32, device=self.device) if keep_results else None
        lib = _lib.load()
        with torch.cuda.device(self.device):
            _lib.check("block_pool_apply", lib.block_pool_apply(ctypes.byref(self._desc), ops.data_ptr(), n,
                                                                None if res is None else res.data_ptr(),
                                                                self._stream()))
        self._results = res

    @property
    def last_results(self) -> Optional[torch.Tensor]:
        """Device statuses of the last ``flush(keep_results=True)``, one per queued call."""
        return self._results

    def slot_of(self, seq_id: int) -> int:
        return self.ledger.slot[seq_id]

    def blocks_of(self, seq_id: int) -> int:
        return self.ledger.blocks.get(seq_id, 0)

    def step_inputs(self, sequence_ids: Sequence[int], q_lens: Sequence[int], kv_lens: Sequence[int],
                    bt_cols: Optional[int] = None) -> dict:
        """A step's attention inputs for ``sequence_ids`` (in the step's order), built on the device.

        Returns device int32 tensors: ``block_table`` [S, bt_cols] (zero
        padded; bt_cols defaults to the most blocks any of them holds, as
        transformer/model.py:145 sizes it), ``num_blocks_per_seq`` [S],
        ``q_len`` / ``kv_len`` [S], ``cu_seqlens`` [S + 1], and per query token
        ``positions`` [T] (``kv_len - q_len + i``) and ``token_seq`` [T] (its
        row of ``block_table``).  Queued allocate / release calls are flushed
        first.  One pinned host-to-device copy of the per-sequence values and
        one launch; no host synchronisation.
        """
        self.flush()
        S = len(sequence_ids)
        slots = [self.ledger.slot[int(s)] for s in sequence_ids]
        if bt_cols is None:
            bt_cols = max((self.ledger.blocks[int(s)] for s in sequence_ids), default=0)
        cu = [0]
        for q in q_lens:
            cu.append(cu[-1] + int(q))
        T = cu[-1]
        host = torch.tensor(slots + [int(q) for q in q_lens] + [int(k) for k in kv_lens] + cu,
                            dtype=torch.int32).pin_memory()
        dev = host.to(self.device, non_blocking=True)
        seq_slot, ql, kl, cus = dev[:S], dev[S:2 * S], dev[2 * S:3 * S], dev[3 * S:]
        i32 = dict(dtype=torch.int32, device=self.device)
        bt = torch.empty(S, bt_cols, **i32)
        nb = torch.empty(S, **i32)
        pos = torch.empty(T, **i32)
        tseq = torch.empty(T, **i32)
        lib = _lib.load()
        with torch.cuda.device(self.device):
            _lib.check("block_pool_step", lib.block_pool_step(
                ctypes.byref(self._desc), seq_slot.data_ptr(), ql.data_ptr(), kl.data_ptr(), cus.data_ptr(), S,
                bt.data_ptr() if bt.numel() else None, max(bt_cols, 1), bt_cols, nb.data_ptr(),
                pos.data_ptr() if T else None, tseq.data_ptr() if T else None, T, self.status.data_ptr(),
                self._stream()))
        return dict(block_table=bt, num_blocks_per_seq=nb, q_len=ql, kv_len=kl, cu_seqlens=cus, positions=pos,
                    token_seq=tseq)

    def step_rows(self, seq_slot: torch.Tensor, q_len: torch.Tensor, kv_len: torch.Tensor, cu_seqlens: torch.Tensor,
                  total_tokens: int, block_table: torch.Tensor, num_blocks: torch.Tensor, positions: torch.Tensor,
                  token_seq: torch.Tensor, status: Optional[torch.Tensor] = None) -> None:
        """``block_pool_step`` on caller-owned device tensors (no host copy, no allocation: capturable).

        ``seq_slot`` / ``q_len`` / ``kv_len`` int32 [S], ``cu_seqlens`` [S + 1]; writes ``block_table``
        [S, bt_cols] (row stride honoured), ``num_blocks`` [S], ``positions`` / ``token_seq`` [total_tokens].
        """
        S = seq_slot.numel()
        lib = _lib.load()
        with torch.cuda.device(self.device):
            _lib.check("block_pool_step", lib.block_pool_step(
                ctypes.byref(self._desc), seq_slot.data_ptr(), q_len.data_ptr(), kv_len.data_ptr(),
                cu_seqlens.data_ptr(), S, block_table.data_ptr(), block_table.stride(0), block_table.shape[1],
                num_blocks.data_ptr(), positions.data_ptr(), token_seq.data_ptr(), int(total_tokens),
                None if status is None else status.data_ptr(), self._stream()))

    @property
    def block_table(self) -> dict:
        """The per-sequence block lists as a host dict (reads the device: synchronises; for checks)."""
        self.flush()
        tab = self.table.cpu()
        return {sid: tab[slot, :self.ledger.blocks[sid]].tolist() for sid, slot in self.ledger.slot.items()}

    def free_list(self) -> list[int]:
        """The free list bottom to top, as the reference's ``st`` (reads the device: synchronises)."""
        self.flush()
        top = int(self.free_top.item())
        return self.free_stack[:top].tolist()
