"""Drop-in replacement for ``kernels/flash_attention.py`` of
VrajPatel105/paged-inference-engine, backed by hand-written sm_100a CUDA
kernels (libpaged_attn_b200.so) instead of Triton.

Put ``paged-inference-engine_b200/`` ahead of the reference checkout on
``sys.path`` and ``from kernels.flash_attention import FlashAttentionFunction``
in ``transformer/model.py:8`` picks this module up unchanged.

Public names and signatures follow the reference:

* ``flash_attention_forward(Q, K, V, q_len_per_seq, block_table,
  num_blocks_per_seq, block_size, kv_len_per_seq, k_scale_ptr, v_scale_ptr)
  -> (O, L)``  (reference kernels/flash_attention.py:139-172)
* ``FlashAttentionFunction.apply(<same 10 args>) -> O``  (:175-180)

Argument meaning is the reference's: Q ``[B, H, max_q_len, D]``; K/V pools
addressed as ``[block, slot, head, d]`` (the launcher's stride convention,
:158-159); int32 metadata on the device; ``k_scale_ptr`` / ``v_scale_ptr`` the
dequantisation scales of an INT8 pool; O and L float16.  Differences, all
backward compatible:

* the causal mask is bottom-right aligned (decode query attends to its whole
  prefix); ``causal_top_left=True`` reproduces the reference's mask (:97);
* GQA: ``H_kv = K.shape[2]`` may divide ``H``;
* a pool in the reference model's own layout ``[NB, H, BS, D]``
  (transformer/model.py:64-65, passed unchanged at :156-160) is recognised by
  its dims (dim 1 is not ``block_size``, dim 2 is) and read as such; the
  reference launcher would read it as ``[block, slot, head, d]`` and address
  slots through the head stride;
* float32 pools are rounded to float16 operands in the kernel (the
  precision of the reference's TF32 ``tl.dot``; values must stay below
  65520 in magnitude); float32 ``Q`` is rounded to the pool's 16-bit type;
* scales may be per block ``[NB, H]`` (reference) or per token ``[NB, BS, H]``;
  they are applied for INT8 pools and ignored for float16 / bfloat16 pools
  (pass ``None``);
* outputs are allocated on ``Q.device``; no host synchronisation (the grid is
  sized from ``Q.shape[2]`` instead of ``q_len_per_seq.max().item()``);
* extra keyword arguments ``out=``, ``lse=``, ``softmax_scale=``, ``mode=``.

Errors: a non-CUDA tensor raises ``AssertionError`` as in the reference (:146);
a malformed argument raises ``ValueError``.  There is no CPU path.
"""
from __future__ import annotations

import os
import sys

import torch

_PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if _PKG_ROOT not in sys.path:
    sys.path.insert(0, _PKG_ROOT)

from pie_b200 import ops as _ops  # noqa: E402

__all__ = ["flash_attention_forward", "flash_attention_varlen", "FlashAttentionFunction", "write_kv_cache",
           "project_write_kv_cache"]


def flash_attention_forward(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, q_len_per_seq, block_table,
                            num_blocks_per_seq, block_size, kv_len_per_seq, k_scale_ptr=None, v_scale_ptr=None,
                            *, out=None, lse=None, causal_top_left: bool = False, softmax_scale=None,
                            mode: str = "auto"):
    """Paged causal attention forward; returns (O, L) as float16 tensors.

    O is ``[B, H, max_q_len, D]`` and L ``[B, H, max_q_len]`` (natural-log
    log-sum-exp of the scaled logits).  Rows at or beyond
    ``q_len_per_seq[b]`` are left untouched, as in the reference.
    """
    assert Q.is_cuda and K.is_cuda and V.is_cuda, "Not CUDA Tensors -_-"
    return _ops.paged_attention(Q, K, V, q_len_per_seq, block_table, num_blocks_per_seq, int(block_size),
                                kv_len_per_seq, k_scale_ptr, v_scale_ptr, out=out, lse=lse,
                                causal_top_left=causal_top_left, softmax_scale=softmax_scale, mode=mode)


def flash_attention_varlen(q, cu_seqlens_q, K, V, block_table, num_blocks_per_seq, block_size, kv_len_per_seq,
                           k_scale_ptr=None, v_scale_ptr=None, *, max_q_len=None, out=None, lse=None,
                           causal_top_left: bool = False, softmax_scale=None):
    """flash_attention_forward over packed query rows; returns (O, L) float16.

    ``q`` is ``[T, H, D]`` holding the rows of every sequence back to back,
    sequence b at rows ``cu_seqlens_q[b] : cu_seqlens_q[b + 1]`` (int32 on the
    device), so the caller builds no padded ``[B, H, max_q_len, D]`` copy and
    reads no padded output back (transformer/model.py:133-141,162-167).  O is
    ``[T, H, D]``, L ``[T, H]``.  Pass ``max_q_len`` to avoid the one host read
    of ``cu_seqlens_q``.
    """
    assert q.is_cuda and K.is_cuda and V.is_cuda, "Not CUDA Tensors -_-"
    return _ops.paged_attention_varlen(q, cu_seqlens_q, K, V, block_table, num_blocks_per_seq, int(block_size),
                                       kv_len_per_seq, k_scale_ptr, v_scale_ptr, max_q_len=max_q_len, out=out,
                                       lse=lse, causal_top_left=causal_top_left, softmax_scale=softmax_scale)


class FlashAttentionFunction(torch.autograd.Function):
    """Autograd wrapper (forward only), as kernels/flash_attention.py:175-180."""

    @staticmethod
    def forward(ctx, Q, K, V, q_len_per_seq, block_table, num_blocks_per_seq, block_size, kv_len_per_seq,
                k_scale_ptr, v_scale_ptr):
        O, L = flash_attention_forward(Q, K, V, q_len_per_seq, block_table, num_blocks_per_seq, block_size,
                                       kv_len_per_seq, k_scale_ptr, v_scale_ptr)
        ctx.save_for_backward(Q, K, V, O, L)
        return O

    @staticmethod
    def backward(ctx, *grads):
        raise NotImplementedError("paged attention is inference-only (no backward), as in the reference")


def write_kv_cache(k_new, v_new, block_table, seq_index, positions, k_cache, v_cache, k_scale=None, v_scale=None):
    """Append this step's K/V rows to the paged pool in one launch.

    Replaces the per-token loop of transformer/model.py:85-122.  ``k_new`` /
    ``v_new`` are ``[T, H_kv, D]``; token t goes to row ``seq_index[t]`` of
    ``block_table`` at absolute position ``positions[t]``.  INT8 pools are
    quantised with one symmetric absmax scale per (token, kv head) stored in
    ``k_scale`` / ``v_scale`` ``[NB, BS, H_kv]``; float pools get a rounded copy.
    """
    assert k_new.is_cuda and k_cache.is_cuda, "Not CUDA Tensors -_-"
    _ops.write_kv(k_new, v_new, block_table, seq_index, positions, k_cache, v_cache, k_scale, v_scale)


def project_write_kv_cache(x, w_kv, bias, block_table, seq_index, positions, k_cache, v_cache, k_scale=None,
                           v_scale=None):
    """The K/V projection of transformer/model.py:75-82 with the cache write of :85-122 in its epilogue.

    ``x`` [T, d_model] (float16 / bfloat16), ``w_kv`` = ``torch.cat([W_k.weight, W_v.weight])`` in the same
    dtype, ``bias`` = ``torch.cat([W_k.bias, W_v.bias])`` (float32) or None.  One tensor-core launch computes
    every token's K and V rows and writes them into the paged pool as ``write_kv_cache`` would (quantised
    with one scale per (token, kv head) for INT8 pools); the projected rows never exist unpaged in memory.
    """
    assert x.is_cuda and k_cache.is_cuda, "Not CUDA Tensors -_-"
    _ops.project_write_kv(x, w_kv, bias, block_table, seq_index, positions, k_cache, v_cache, k_scale, v_scale)
