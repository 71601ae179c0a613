"""CPU oracle for the paged-attention hot path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs
of ``bench.py`` may import it.  The GPU library never calls into it.

It restates, in numpy (integer / quantisation work) and torch-on-CPU float32
(attention), the algorithm of VrajPatel105/paged-inference-engine:

* ``quantize_rows``      -- tests/pre_quantize_test.py:3-12 and
                            transformer/model.py:105-114: symmetric absmax INT8,
                            scale = absmax / 127 (1.0 for an all-zero row),
                            q = clamp(round_half_even(x / scale), -127, 127),
                            applied per (token, kv head) row.
* ``quantize_blocks``    -- the reference cache's per-(block, head) scale
                            granularity (transformer/model.py:66-67,105-110),
                            used to build inputs for the reference-compatible
                            [num_blocks, num_heads] scale layout.
* ``write_kv_cache``     -- the scatter of new K/V rows through the block table
                            (transformer/model.py:85-92,117-122) with the
                            per-token rule above.
* ``paged_attention``    -- flash_attention_kernel
                            (kernels/flash_attention.py:19-136): gather K/V
                            blocks in block-table order (:58-64), dequantise
                            k * scale (:73-84), S = q k^T * softmax_scale
                            (:88-90), padding + causal mask (:96-99), softmax,
                            O = P V / l and L = m + ln(l) (:122-123).  The causal
                            mask is bottom-right aligned by default (query row m
                            sits at kv_len - q_len + m); ``top_left=True`` gives
                            the reference kernel's own mask (row m sees keys
                            0..m, :97).  Keys beyond min(kv_len,
                            num_blocks_per_seq * block_size) are never visited
                            (:58,:67-70).  A row with no visible key returns
                            O = 0 and L = -inf.

Parity status: pinned.  tests/golden/ holds fixtures produced by running the
reference's own Triton kernel (under TRITON_INTERPRET=1) and its own
``quantize`` function; tests/test_oracle_golden.py checks this module against
them.
"""
from __future__ import annotations

import math
from typing import Optional

import numpy as np
import torch

__all__ = [
    "quantize_rows",
    "quantize_tensor",
    "quantize_blocks",
    "write_kv_cache",
    "paged_attention",
    "gather_sequence",
]


def quantize_tensor(x: np.ndarray) -> tuple[np.ndarray, np.float32]:
    """tests/pre_quantize_test.py:3-12 on a whole tensor (fp32 arithmetic)."""
    x32 = np.asarray(x, dtype=np.float32)
    amax = np.float32(np.abs(x32).max()) if x32.size else np.float32(0)
    scale = np.float32(1.0) if amax == 0 else np.float32(amax / np.float32(127.0))
    q = np.clip(np.rint(x32 / scale), -127, 127).astype(np.int8)
    return q, scale


def quantize_rows(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Per-row (last axis) version of ``quantize_tensor``.

    Returns (int8 values, fp32 scales with the leading shape).  The division is
    IEEE float32 and np.rint rounds half to even, matching torch.round.
    """
    x32 = np.asarray(x, dtype=np.float32)
    amax = np.abs(x32).max(axis=-1)
    scale = np.where(amax == 0, np.float32(1.0), amax / np.float32(127.0)).astype(np.float32)
    q = np.clip(np.rint(x32 / scale[..., None]), -127, 127).astype(np.int8)
    return q, scale


def quantize_blocks(pool: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """One scale per (block, head) over [NB, BS, H, D] (reference granularity)."""
    x32 = np.asarray(pool, dtype=np.float32)
    amax = np.abs(x32).max(axis=(1, 3))  # [NB, H]
    scale = np.where(amax == 0, np.float32(1.0), amax / np.float32(127.0)).astype(np.float32)
    q = np.clip(np.rint(x32 / scale[:, None, :, None]), -127, 127).astype(np.int8)
    return q, scale


def write_kv_cache(k_new, v_new, block_table, seq_index, positions, k_cache, v_cache, k_scale=None, v_scale=None,
                   scale_dtype=np.float16):
    """Scatter new rows [T, H, D] into pools [NB, BS, H, D] (numpy, in place).

    INT8 pools (k_cache.dtype == int8) are written with ``quantize_rows`` and
    their per-(token, head) scales [NB, BS, H] are rounded to ``scale_dtype``.
    Other pools receive the values cast to the pool dtype.
    """
    bs = k_cache.shape[1]
    for t in range(len(positions)):
        s = int(seq_index[t])
        p = int(positions[t])
        blk = int(block_table[s][p // bs])
        slot = p % bs
        for src, dst, sc in ((k_new, k_cache, k_scale), (v_new, v_cache, v_scale)):
            row = np.asarray(src[t], dtype=np.float32)
            if dst.dtype == np.int8:
                q, scale = quantize_rows(row)
                dst[blk, slot] = q
                sc[blk, slot] = scale.astype(scale_dtype)
            else:
                dst[blk, slot] = row.astype(dst.dtype)


def _scale_at(scale, blk: np.ndarray, slot: np.ndarray) -> np.ndarray:
    """Scale rows for gathered keys: [NB, H] (per block) or [NB, BS, H] (per token)."""
    s = np.asarray(scale, dtype=np.float32)
    if s.ndim == 2:
        return s[blk]
    return s[blk, slot]


def gather_sequence(pool, scale, block_table_row, n_keys: int) -> np.ndarray:
    """Keys 0..n_keys-1 of one sequence as float32 [n_keys, H, D], dequantised."""
    bs = pool.shape[1]
    keys = np.arange(n_keys)
    blk = np.asarray(block_table_row, dtype=np.int64)[keys // bs]
    slot = keys % bs
    x = np.asarray(pool[blk, slot], dtype=np.float32)
    if scale is not None:
        x = x * _scale_at(scale, blk, slot)[:, :, None]
    return x


def paged_attention(q, k_pool, v_pool, q_len, block_table, num_blocks, block_size: int, kv_len, k_scale=None,
                    v_scale=None, *, top_left: bool = False, softmax_scale: Optional[float] = None,
                    threads: Optional[int] = None) -> tuple[np.ndarray, np.ndarray]:
    """Reference paged attention on the CPU in float32.

    q [B, Hq, maxq, D]; pools [NB, BS, Hkv, D] (any float dtype or int8 with
    scales); metadata int arrays [B].  Returns (O [B, Hq, maxq, D] float32,
    L [B, Hq, maxq] float32); rows >= q_len are zero / -inf.
    """
    q = np.asarray(q)
    B, Hq, maxq, D = q.shape
    Hkv = k_pool.shape[2]
    assert Hq % Hkv == 0
    G = Hq // Hkv
    assert k_pool.shape[1] == block_size
    sm = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    if threads is not None:
        torch.set_num_threads(threads)
    O = np.zeros((B, Hq, maxq, D), dtype=np.float32)
    L = np.full((B, Hq, maxq), -np.inf, dtype=np.float32)
    q_len = np.asarray(q_len)
    kv_len = np.asarray(kv_len)
    num_blocks = np.asarray(num_blocks)
    for b in range(B):
        ql = int(q_len[b])
        if ql <= 0:
            continue
        nb = max(0, min(int(num_blocks[b]), np.asarray(block_table).shape[1]))
        nk = max(0, min(int(kv_len[b]), nb * block_size))
        if top_left:
            nk = min(nk, ql)
        off = 0 if top_left else int(kv_len[b]) - ql
        rows = np.arange(ql)
        lim = np.minimum(nk, off + rows + 1)  # visible keys per row
        if nk == 0:
            continue
        kseq = torch.from_numpy(gather_sequence(k_pool, k_scale, block_table[b], nk))  # [nk, Hkv, D]
        vseq = torch.from_numpy(gather_sequence(v_pool, v_scale, block_table[b], nk))
        qb = torch.from_numpy(np.ascontiguousarray(q[b, :, :ql], dtype=np.float32)).view(Hkv, G * ql, D)
        s = torch.einsum("hmd,khd->hmk", qb, kseq) * sm  # [Hkv, G*ql, nk]
        s = s.view(Hkv, G, ql, nk)
        mask = torch.from_numpy(np.arange(nk)[None, :] < lim[:, None])  # [ql, nk]
        s = s.masked_fill(~mask, float("-inf"))
        lse = torch.logsumexp(s, dim=-1)  # [Hkv, G, ql]
        p = torch.exp(s - torch.where(torch.isfinite(lse), lse, torch.zeros_like(lse))[..., None])
        p = torch.where(torch.isfinite(lse)[..., None], p, torch.zeros_like(p))
        o = torch.einsum("hgmk,khd->hgmd", p, vseq)
        O[b, :, :ql] = o.reshape(Hq, ql, D).numpy()
        L[b, :, :ql] = lse.reshape(Hq, ql).numpy()
    return O, L
