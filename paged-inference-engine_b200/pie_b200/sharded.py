"""KV-head sharded paged attention (decode and prefill) across the GPUs of one node.

Attention has no cross-head dependency, so rank r of a world of G ranks owns
KV heads [r*Hkv/G, (r+1)*Hkv/G) -- its own block pool [NB_r, BS, Hkv/G, D]
(and scales) -- and the Hq/G query heads that read them.  Each rank runs the
attention kernels on its local heads (split-K decode for short query blocks,
the tcgen05 prefill kernel for long ones: any query length); one NCCL
``all_gather_into_tensor`` over NVLink then assembles O for all heads in head
order, which is only needed where the consumer wants every head (e.g. the
output projection).  Sharding by sequence needs no collective at all: every
rank runs its own sequences with all heads (the replicas of bench.py's
per-rank batches).

The reference has no multi-GPU path; this module is the B200 scaling layer for
the paged-attention hot path (kernels/flash_attention.py:139-172 per rank).
"""
from __future__ import annotations

import ctypes
import math
from typing import Callable, Optional

import torch
import torch.distributed as dist


def head_range(num_heads: int, world: int, rank: int) -> tuple[int, int]:
    if num_heads % world:
        raise ValueError(f"{num_heads} heads do not split over {world} ranks")
    n = num_heads // world
    return rank * n, (rank + 1) * n


class _DeviceBuffer:
    """A raw device allocation presented to torch through __cuda_array_interface__."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerOutputExchange:
    """Output buffers of every rank mapped into every rank (plain CUDA IPC peer mappings).

    Two fp16 output buffers (steps alternate between them, so a rank never
    overwrites rows a peer may still be reading) and one int32 flag array per
    rank.  Set-up is collective: every rank calls ``ensure`` with the same shape.
    """

    def __init__(self, group, world: int, rank: int, device: torch.device):
        self.group, self.world, self.rank, self.device = group, world, rank, device
        self.shape = None
        self.epoch = 0
        # Device status word shared by the decode kernels and the barrier of every
        # step; after each step it is copied into a pinned host slot of that step's
        # buffer parity, and read back two steps later (when the buffer comes round
        # again), so a peer that missed the barrier raises without a per-step sync.
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self._host_status = torch.zeros(2, dtype=torch.int32, pin_memory=True)
        self._events: list = [None, None]

    def ensure(self, shape: tuple[int, ...]) -> None:
        if self.shape == tuple(shape):
            return
        if self.shape is not None:
            raise RuntimeError("the peer output buffers were set up for another shape")
        from . import _lib

        lib = _lib.load()
        nbytes = math.prod(shape) * 2
        local, handles = [], []
        with torch.cuda.device(self.device):
            for size in (nbytes, nbytes, 256):
                ptr, h = ctypes.c_void_p(), (ctypes.c_char * 64)()
                _lib.check("paged_attn_peer_alloc", lib.paged_attn_peer_alloc(size, ctypes.byref(ptr), h))
                local.append(ptr.value)
                handles.append(bytes(h))
            all_h: list = [None] * self.world
            dist.all_gather_object(all_h, handles, group=self.group)
            peers = [[0] * self.world for _ in range(3)]
            for r in range(self.world):
                for k in range(3):
                    if r == self.rank:
                        peers[k][r] = local[k]
                        continue
                    ptr = ctypes.c_void_p()
                    _lib.check("paged_attn_peer_open", lib.paged_attn_peer_open(all_h[r][k], ctypes.byref(ptr)))
                    peers[k][r] = ptr.value
        self.local, self.peers = local, peers
        self.views = [torch.as_tensor(_DeviceBuffer(local[k], shape, "<f2"), device=self.device) for k in range(2)]
        self.flags = (ctypes.c_void_p * self.world)(*peers[2])
        self.shape = tuple(shape)
        dist.barrier(group=self.group)  # every rank has mapped every buffer before the first exchange

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective: no exchange may be in flight)."""
        if self.shape is None:
            return
        from . import _lib

        lib = _lib.load()
        torch.cuda.synchronize(self.device)
        pending = [int(self._host_status[k]) for k in (0, 1) if self._events[k] is not None]
        self._events = [None, None]
        dist.barrier(group=self.group)  # no peer still writes into this rank's buffers
        with torch.cuda.device(self.device):
            for k in range(3):
                for r in range(self.world):
                    if r != self.rank:
                        _lib.check("paged_attn_peer_close", lib.paged_attn_peer_close(self.peers[k][r]))
            dist.barrier(group=self.group)  # every peer has unmapped before the memory is freed
            for k in range(3):
                _lib.check("paged_attn_peer_free", lib.paged_attn_peer_free(self.local[k]))
        self.shape, self.views = None, None
        bad = [v for v in pending if v]
        if bad:
            from . import ops

            ops._raise_status_value("peer output exchange", bad[0])

    def check(self, parity: Optional[int] = None) -> None:
        """Raise if a finished step (both parities, or one) reported a device error.

        Waits for that step's status copy; a step still in flight is waited for.
        """
        from . import ops

        for k in ((0, 1) if parity is None else (parity,)):
            ev = self._events[k]
            if ev is None:
                continue
            ev.synchronize()
            self._events[k] = None
            v = int(self._host_status[k])
            if v:
                self.status.zero_()
                self._host_status.zero_()
                ops._raise_status_value("peer output exchange", v)

    def exchange(self, run_decode: Callable[[torch.Tensor, list[int], torch.Tensor], None], head_lo: int,
                 head_hi: int) -> torch.Tensor:
        """run_decode(out_view, peer_ptrs, status) writes heads [head_lo, head_hi) into every rank.

        Returns the buffer holding all heads.  Raises IndexError (naming the
        status bits) when the step that last used the same buffer reported a
        device error: a peer that never reached the barrier (its heads are then
        missing) or bad paging metadata.
        """
        from . import _lib

        lib = _lib.load()
        k = self.epoch & 1
        self.check(k)  # the step two back used this buffer: its status must be clean
        self.epoch += 1
        full = self.views[k]
        view = full[:, head_lo:head_hi]
        off = view.data_ptr() - full.data_ptr()
        run_decode(view, [p + off for p in self.peers[k]], self.status)
        stream = torch.cuda.current_stream(self.device)
        _lib.check("paged_attn_peer_barrier",
                   lib.paged_attn_peer_barrier(self.local[2], self.flags, self.world, self.rank, self.epoch,
                                               self.status.data_ptr(), stream.cuda_stream))
        self._host_status[k:k + 1].copy_(self.status, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(stream)
        self._events[k] = ev
        return full


class KVHeadShardedDecoder:
    """Per-rank attention over the local KV heads + all-gather of head outputs.

    Works for any query length (decode, prefill, chunked prefill): the local
    call dispatches like ``flash_attention_forward``.

    ``attention_fn(Q_local, K, V, q_len, block_table, num_blocks, block_size,
    kv_len, k_scale, v_scale) -> (O, L)`` computes the local heads; it defaults
    to the CUDA ``flash_attention_forward``.  The gather uses the default
    process group (NCCL on GPUs; any backend works for the host logic).

    ``exchange="peer"`` (GPUs of one box) replaces the all-gather by the
    fused exchange for decode shapes (max_q_len * Hq / Hkv <= 16; longer
    query blocks use the all-gather): the decode kernels store every finished
    output row into every rank's mapped output buffer and a cross-GPU flag
    barrier ends the step.  The returned tensor is then one of two buffers the
    steps alternate between: consume it on the current stream before the
    next-but-one ``forward``.  Each step's device status (a peer that never
    reached the barrier, bad paging metadata) is read back two steps later,
    when its buffer comes round again, and raised there; ``check()`` reads the
    outstanding ones.
    """

    def __init__(self, num_q_heads: int, num_kv_heads: int, head_dim: int, group=None,
                 attention_fn: Optional[Callable] = None, exchange: str = "nccl"):
        if exchange not in ("nccl", "peer"):
            raise ValueError(f"exchange must be 'nccl' or 'peer', not {exchange!r}")
        self.exchange = exchange
        self._peer: Optional[PeerOutputExchange] = None
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if num_kv_heads % self.world:
            raise ValueError(f"{num_kv_heads} KV heads do not split over {self.world} ranks")
        self.Hq, self.Hkv, self.D = num_q_heads, num_kv_heads, head_dim
        self.kv_lo, self.kv_hi = head_range(num_kv_heads, self.world, self.rank)
        self.q_lo, self.q_hi = head_range(num_q_heads, self.world, self.rank)
        if attention_fn is None:
            from kernels.flash_attention import flash_attention_forward
            attention_fn = flash_attention_forward
        self.attention_fn = attention_fn
        self._gather_buf = None

    def check(self) -> None:
        """Wait for the outstanding peer-exchange steps and raise if one reported a device error.

        ``forward`` checks each step two steps later on its own; call this after
        the last step whose output is used.
        """
        if self._peer is not None:
            self._peer.check()

    def close(self) -> None:
        """Release the peer-exchange buffers (collective; a no-op for the NCCL exchange)."""
        if self._peer is not None:
            self._peer.close()
            self._peer = None

    def local_q(self, Q_full: torch.Tensor) -> torch.Tensor:
        """This rank's query heads of a full [B, Hq, q, D] tensor."""
        return Q_full[:, self.q_lo:self.q_hi]

    def forward(self, Q_local, K, V, q_len, block_table, num_blocks, block_size, kv_len, k_scale=None,
                v_scale=None, gather: bool = True):
        """Returns O for all heads [B, Hq, q, D] (gather=True) or the local heads [B, Hq/G, q, D]."""
        decode_shape = Q_local.shape[2] * (self.Hq // self.Hkv) <= 16
        if gather and self.world > 1 and self.exchange == "peer" and decode_shape:
            return self._forward_peer(Q_local, K, V, q_len, block_table, num_blocks, block_size, kv_len, k_scale,
                                      v_scale)
        O_loc, _ = self.attention_fn(Q_local, K, V, q_len, block_table, num_blocks, block_size, kv_len, k_scale,
                                     v_scale)
        if not gather or self.world == 1:
            return O_loc
        return self.gather(O_loc)

    def _forward_peer(self, Q_local, K, V, q_len, block_table, num_blocks, block_size, kv_len, k_scale, v_scale):
        from . import ops

        B, hl, q, D = Q_local.shape
        if self._peer is None:
            self._peer = PeerOutputExchange(self.group, self.world, self.rank, Q_local.device)
        self._peer.ensure((B, self.Hq, q, D))

        def run(view, ptrs, status):
            ops.paged_attention_peers(Q_local, K, V, q_len, block_table, num_blocks, int(block_size), kv_len,
                                      k_scale, v_scale, view, ptrs, status=status)

        return self._peer.exchange(run, self.q_lo, self.q_hi)

    def gather(self, O_loc: torch.Tensor) -> torch.Tensor:
        B, hl, q, D = O_loc.shape
        n = O_loc.numel()
        if self._gather_buf is None or self._gather_buf.numel() != n * self.world or \
                self._gather_buf.device != O_loc.device or self._gather_buf.dtype != O_loc.dtype:
            self._gather_buf = torch.empty(n * self.world, dtype=O_loc.dtype, device=O_loc.device)
        dist.all_gather_into_tensor(self._gather_buf, O_loc.contiguous().view(-1), group=self.group)
        return self._gather_buf.view(self.world, B, hl, q, D).permute(1, 0, 2, 3, 4).reshape(B, self.world * hl, q, D)


KVHeadShardedAttention = KVHeadShardedDecoder  # the same layer, named for any query length


# ----------------------------------------------------------------------------
# long-context benchmark (strong scaling over KV heads)
# ----------------------------------------------------------------------------
def build_rank_pool(ctx: list[int], Hkv_local: int, D: int, BS: int, seed: int, device, outliers: float = 0.01):
    """Seeded INT8 pool (per-token fp16 scales, head-major) for this rank's KV heads, built on the device."""
    from .workloads import block_tables, empty_head_major_scales, quantize_rows_torch

    gen = torch.Generator().manual_seed(seed)
    bt, nblk, NB = block_tables(gen, ctx, BS)
    K = torch.empty(NB, BS, Hkv_local, D, dtype=torch.int8, device=device)
    V = torch.empty_like(K)
    ks = empty_head_major_scales(NB, BS, Hkv_local, device=device)
    vs = empty_head_major_scales(NB, BS, Hkv_local, device=device)
    dg = torch.Generator(device=device).manual_seed(seed)
    step = 16384
    for lo in range(0, NB, step):
        hi = min(NB, lo + step)
        for pool, sc in ((K, ks), (V, vs)):
            x = torch.randn(hi - lo, BS, Hkv_local, D, generator=dg, device=device)
            if outliers:
                x = x * torch.where(torch.rand(x.shape, generator=dg, device=device) < outliers, 8.0, 1.0)
            q, s = quantize_rows_torch(x.half())
            pool[lo:hi] = q
            sc[lo:hi] = s
    return K, V, ks, vs, bt.to(device), nblk.to(device), NB
