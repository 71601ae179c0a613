"""Seeded synthetic paged-attention workloads with the shapes of the reference's
benchmark configurations (no public dataset is involved in this path).

Every tensor is drawn on the CPU from a ``torch.Generator`` seeded by the
caller, so the CUDA kernels and the CPU oracle see identical bytes.

Configurations (sizes as in the reference's measurement plan):
  cpu_decode     B=4, ctx [17,64,100,128], H=8, D=64, BS=16, 64-block pool
  decode_fp16    B=64, Hq=32, Hkv=8, D=128, BS=16, ctx ~ U[512, 4096]
  decode_int8    decode_fp16 shape + quantise-on-write of 64 new tokens/seq,
                 K/V ~ N(0,1) with 1% outliers x8, int8 + fp16 per-token scales
  prefill_bf16   B=8, L ~ U[1024, 4096], Hq=32, Hkv=8, D=128, BS=16
  long_ctx_int8  B=256, Hq=64, Hkv=8, D=128, BS=16, ctx ~ U[8192, 32768], int8
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import torch

CONFIGS = {
    "cpu_decode": dict(B=4, Hq=8, Hkv=8, D=64, BS=16, ctx=[17, 64, 100, 128], pool_blocks=64),
    "decode_fp16": dict(B=64, Hq=32, Hkv=8, D=128, BS=16, ctx_range=(512, 4096)),
    "decode_int8": dict(B=64, Hq=32, Hkv=8, D=128, BS=16, ctx_range=(512, 4096), new_tokens=64),
    "prefill_bf16": dict(B=8, Hq=32, Hkv=8, D=128, BS=16, ctx_range=(1024, 4096)),
    "long_ctx_int8": dict(B=256, Hq=64, Hkv=8, D=128, BS=16, ctx_range=(8192, 32768)),
}


@dataclass
class PagedBatch:
    """One step's inputs: Q, the paged pool and the paging metadata (CPU tensors)."""

    Q: torch.Tensor            # [B, Hq, q_max, D]
    K: torch.Tensor            # [NB, BS, Hkv, D]
    V: torch.Tensor
    k_scale: Optional[torch.Tensor]
    v_scale: Optional[torch.Tensor]
    block_table: torch.Tensor  # [B, max_blocks] int32
    num_blocks: torch.Tensor   # [B] int32
    q_len: torch.Tensor        # [B] int32
    kv_len: torch.Tensor       # [B] int32
    block_size: int
    extras: dict = field(default_factory=dict)

    def to(self, device) -> "PagedBatch":
        mv = lambda t: None if t is None else t.to(device)  # noqa: E731
        return PagedBatch(mv(self.Q), mv(self.K), mv(self.V), mv(self.k_scale), mv(self.v_scale),
                          mv(self.block_table), mv(self.num_blocks), mv(self.q_len), mv(self.kv_len),
                          self.block_size, {k: mv(v) if torch.is_tensor(v) else v for k, v in self.extras.items()})

    @property
    def kv_bytes_per_token_head(self) -> int:
        d = self.K.shape[3]
        if self.K.dtype == torch.int8:
            return 2 * d + 2 * (self.k_scale.element_size() if self.k_scale is not None else 0)
        return 2 * d * self.K.element_size()


def draw_context_lengths(gen: torch.Generator, B: int, lo: int, hi: int) -> list[int]:
    return torch.randint(lo, hi + 1, (B,), generator=gen).tolist()


def block_tables(gen: torch.Generator, ctx: list[int], BS: int, slack: float = 0.10,
                 pool_blocks: Optional[int] = None) -> tuple[torch.Tensor, torch.Tensor, int]:
    """Scattered block tables: a seeded permutation of a pool of total+10% blocks."""
    nblk = [max(1, -(-c // BS)) for c in ctx]
    total = sum(nblk)
    NB = pool_blocks if pool_blocks is not None else int(math.ceil(total * (1.0 + slack)))
    assert NB >= total
    perm = torch.randperm(NB, generator=gen).to(torch.int32)
    bt = torch.zeros(len(ctx), max(nblk), dtype=torch.int32)
    cur = 0
    for b, n in enumerate(nblk):
        bt[b, :n] = perm[cur:cur + n]
        cur += n
    return bt, torch.tensor(nblk, dtype=torch.int32), NB


def _normal(gen, shape, dtype, outliers: float = 0.0):
    x = torch.randn(shape, generator=gen)
    if outliers:
        x = x * torch.where(torch.rand(shape, generator=gen) < outliers, 8.0, 1.0)
    return x.to(dtype)


def make_decode_batch(seed: int, B: int, Hq: int, Hkv: int, D: int, BS: int, ctx: list[int], *,
                      kv_dtype=torch.float16, q_dtype=torch.float16, q_len: int = 1, outliers: float = 0.0,
                      scale_dtype=torch.float16, pool_blocks: Optional[int] = None) -> PagedBatch:
    """Decode / short-query batch over an already filled pool.

    INT8 pools are produced from fp16 draws with the per-(token, head) rule of
    the oracle (round-half-even, scale absmax/127) on the CPU.
    """
    gen = torch.Generator().manual_seed(seed)
    bt, nblk, NB = block_tables(gen, ctx, BS, pool_blocks=pool_blocks)
    Q = _normal(gen, (B, Hq, q_len, D), q_dtype)
    if kv_dtype == torch.int8:
        K16 = _normal(gen, (NB, BS, Hkv, D), torch.float16, outliers)
        V16 = _normal(gen, (NB, BS, Hkv, D), torch.float16, outliers)
        K, ks = quantize_rows_torch(K16, scale_dtype)
        V, vs = quantize_rows_torch(V16, scale_dtype)
        ks, vs = head_major(ks), head_major(vs)
    else:
        K = _normal(gen, (NB, BS, Hkv, D), kv_dtype, outliers)
        V = _normal(gen, (NB, BS, Hkv, D), kv_dtype, outliers)
        ks = vs = None
    return PagedBatch(Q, K, V, ks, vs, bt, nblk, torch.full((B,), q_len, dtype=torch.int32),
                      torch.tensor(ctx, dtype=torch.int32), BS)


def head_major(scales: torch.Tensor) -> torch.Tensor:
    """Per-token scales [NB, BS, H] stored head-major ([NB, H, BS] in memory), as the same [NB, BS, H] view.

    The attention kernels read a tile's scales one KV head at a time: in this
    layout the 16 scales of one head and block are one 32-byte sector, where
    the slot-major layout spreads them over 16 * H * 2 bytes.
    """
    return scales.transpose(1, 2).contiguous().transpose(1, 2)


def empty_head_major_scales(NB: int, BS: int, H: int, dtype=torch.float16, device=None) -> torch.Tensor:
    """Uninitialised per-token scales [NB, BS, H] in the head-major layout of ``head_major``."""
    return torch.empty(NB, H, BS, dtype=dtype, device=device).transpose(1, 2)


def quantize_rows_torch(x: torch.Tensor, scale_dtype=torch.float16) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row symmetric INT8 in float32 (round half to even), scales stored as ``scale_dtype``.

    Same rule as the oracle's ``quantize_rows``; used only to fill synthetic
    pools quickly on the CPU.
    """
    x32 = x.float()
    amax = x32.abs().amax(dim=-1)
    s = torch.where(amax == 0, torch.ones_like(amax), amax / 127.0)
    q = torch.round(x32 / s[..., None]).clamp(-127, 127).to(torch.int8)
    return q, s.to(scale_dtype)


def config_batch(name: str, seed: int = 0, **over) -> PagedBatch:
    """The named configuration as a decode batch (ctx drawn from its range)."""
    cfg = dict(CONFIGS[name])
    cfg.update(over)
    gen = torch.Generator().manual_seed(seed)
    ctx = cfg.get("ctx") or draw_context_lengths(gen, cfg["B"], *cfg["ctx_range"])
    kv = torch.int8 if name in ("decode_int8", "long_ctx_int8") else torch.float16
    return make_decode_batch(seed + 1, cfg["B"], cfg["Hq"], cfg["Hkv"], cfg["D"], cfg["BS"], ctx, kv_dtype=kv,
                             outliers=0.01 if kv == torch.int8 else 0.0, pool_blocks=cfg.get("pool_blocks"))
