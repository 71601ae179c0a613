"""KV-head sharded paged decode across the GPUs of one node.

Attention has no cross-head dependency, so rank r of a world of G ranks owns
KV heads [r*Hkv/G, (r+1)*Hkv/G) -- its own block pool [NB_r, BS, Hkv/G, D]
(and scales) -- and the Hq/G query heads that read them.  Each rank runs the
split-K decode kernel on its local heads; one NCCL ``all_gather_into_tensor``
over NVLink then assembles O for all heads in head order, which is only needed
where the consumer wants every head (e.g. the output projection).

The reference has no multi-GPU path; this module is the B200 scaling layer for
the paged-attention hot path (kernels/flash_attention.py:139-172 per rank).
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


def head_range(num_heads: int, world: int, rank: int) -> tuple[int, int]:
    if num_heads % world:
        raise ValueError(f"{num_heads} heads do not split over {world} ranks")
    n = num_heads // world
    return rank * n, (rank + 1) * n


class KVHeadShardedDecoder:
    """Per-rank decode over the local KV heads + all-gather of head outputs.

    ``attention_fn(Q_local, K, V, q_len, block_table, num_blocks, block_size,
    kv_len, k_scale, v_scale) -> (O, L)`` computes the local heads; it defaults
    to the CUDA ``flash_attention_forward``.  The gather uses the default
    process group (NCCL on GPUs; any backend works for the host logic).
    """

    def __init__(self, num_q_heads: int, num_kv_heads: int, head_dim: int, group=None,
                 attention_fn: Optional[Callable] = None):
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

    def local_q(self, Q_full: torch.Tensor) -> torch.Tensor:
        """This rank's query heads of a full [B, Hq, q, D] tensor."""
        return Q_full[:, self.q_lo:self.q_hi]

    def forward(self, Q_local, K, V, q_len, block_table, num_blocks, block_size, kv_len, k_scale=None,
                v_scale=None, gather: bool = True):
        """Returns O for all heads [B, Hq, q, D] (gather=True) or the local heads."""
        O_loc, _ = self.attention_fn(Q_local, K, V, q_len, block_table, num_blocks, block_size, kv_len, k_scale,
                                     v_scale)
        if not gather or self.world == 1:
            return O_loc
        return self.gather(O_loc)

    def gather(self, O_loc: torch.Tensor) -> torch.Tensor:
        B, hl, q, D = O_loc.shape
        n = O_loc.numel()
        if self._gather_buf is None or self._gather_buf.numel() != n * self.world or \
                self._gather_buf.device != O_loc.device or self._gather_buf.dtype != O_loc.dtype:
            self._gather_buf = torch.empty(n * self.world, dtype=O_loc.dtype, device=O_loc.device)
        dist.all_gather_into_tensor(self._gather_buf, O_loc.contiguous().view(-1), group=self.group)
        return self._gather_buf.view(self.world, B, hl, q, D).permute(1, 0, 2, 3, 4).reshape(B, self.world * hl, q, D)


# ----------------------------------------------------------------------------
# long-context benchmark (strong scaling over KV heads)
# ----------------------------------------------------------------------------
def build_rank_pool(ctx: list[int], Hkv_local: int, D: int, BS: int, seed: int, device, outliers: float = 0.01):
    """Seeded INT8 pool (per-token fp16 scales) for this rank's KV heads, built on the device."""
    from .workloads import block_tables, quantize_rows_torch

    gen = torch.Generator().manual_seed(seed)
    bt, nblk, NB = block_tables(gen, ctx, BS)
    K = torch.empty(NB, BS, Hkv_local, D, dtype=torch.int8, device=device)
    V = torch.empty_like(K)
    ks = torch.empty(NB, BS, Hkv_local, dtype=torch.float16, device=device)
    vs = torch.empty_like(ks)
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
