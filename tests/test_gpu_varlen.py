"""Ragged (varlen) query rows: paged_attn_varlen against the padded entry point.

A caller that keeps every sequence's query rows packed ([T, H, D] with
cu_seqlens) must get, row for row, what the padded [B, H, max_q_len, D] call
returns: each row's output depends only on its own query row, so the valid
rows are bit-identical.  Covers the decode kernel (one row and short query
blocks), the tcgen05 prefill kernel, the mma.sync prefill kernel (INT8 pool),
empty sequences, and a start offset past T (rows are clamped to the packed
tensor; guard rows behind it stay untouched).
"""
import numpy as np
import pytest
import torch

from oracle import paged_attention as orc

pytestmark = pytest.mark.gpu


def _pack(Q, q_len):
    """[B, H, maxq, D] + q_len -> packed [T, H, D], cu_seqlens."""
    rows = [Q[b, :, :n].transpose(0, 1) for b, n in enumerate(q_len)]
    cu = np.concatenate([[0], np.cumsum(q_len)]).astype(np.int32)
    return torch.cat(rows, 0).contiguous(), torch.from_numpy(cu)


def _check_rows(Ov, Lv, O, L, q_len, cu):
    for b, n in enumerate(q_len):
        s = int(cu[b])
        assert torch.equal(Ov[s:s + n], O[b, :, :n].transpose(0, 1)), f"seq {b}"
        assert torch.equal(Lv[s:s + n], L[b, :, :n].transpose(0, 1)), f"seq {b} LSE"


def _batch(seed, ctx, q_len, Hq, Hkv, D, kv_dtype, q_dtype=torch.float16):
    from pie_b200.workloads import make_decode_batch

    b = make_decode_batch(seed, len(ctx), Hq, Hkv, D, 16, ctx, kv_dtype=kv_dtype, q_dtype=q_dtype,
                          q_len=max(q_len), outliers=0.01).to("cuda")
    b.q_len = torch.tensor(q_len, dtype=torch.int32, device="cuda")
    return b


@pytest.mark.parametrize("case", ["decode_f16", "decode_i8", "short_q", "prefill_tc", "prefill_tc_bf16",
                                  "prefill_i8"])
def test_varlen_equals_padded(case):
    from kernels.flash_attention import flash_attention_forward, flash_attention_varlen

    if case.startswith("decode"):
        ctx, q_len, Hq, Hkv, D = [1, 40, 300, 1000, 2049, 17], [1] * 6, 32, 8, 128
    elif case == "short_q":
        ctx, q_len, Hq, Hkv, D = [10, 300, 1000, 77], [2, 4, 1, 3], 16, 4, 128
    else:
        ctx, q_len, Hq, Hkv, D = [300, 129, 1000, 1, 640], [300, 129, 1000, 1, 200], 8, 2, 128
    kv_dtype = {"decode_i8": torch.int8, "prefill_i8": torch.int8, "prefill_tc_bf16": torch.bfloat16}.get(case,
                                                                                                       torch.float16)
    q_dtype = torch.bfloat16 if case == "prefill_tc_bf16" else torch.float16
    b = _batch(7, ctx, q_len, Hq, Hkv, D, kv_dtype, q_dtype)
    args = (b.K, b.V, b.q_len, b.block_table, b.num_blocks, 16, b.kv_len, b.k_scale, b.v_scale)
    O, L = flash_attention_forward(b.Q, *args)
    qv, cu = _pack(b.Q, q_len)
    cu = cu.cuda()
    Ov, Lv = flash_attention_varlen(qv, cu, b.K, b.V, b.block_table, b.num_blocks, 16, b.kv_len, b.k_scale,
                                    b.v_scale, max_q_len=max(q_len))
    torch.cuda.synchronize()
    _check_rows(Ov, Lv, O, L, q_len, cu.cpu().numpy())
    # and the oracle, on the packed rows
    O_or, _ = orc.paged_attention(b.Q.float().cpu().numpy(), b.K.cpu().numpy() if kv_dtype == torch.int8 else
                                  b.K.float().cpu().numpy(),
                                  b.V.cpu().numpy() if kv_dtype == torch.int8 else b.V.float().cpu().numpy(),
                                  np.array(q_len), b.block_table.cpu().numpy(), b.num_blocks.cpu().numpy(), 16,
                                  b.kv_len.cpu().numpy(),
                                  None if b.k_scale is None else b.k_scale.cpu().numpy(),
                                  None if b.v_scale is None else b.v_scale.cpu().numpy())
    # max-abs tolerance, or two fp16 ulps of the expected value where that is larger.  With the
    # workload's 8x outliers |O| reaches ~10 on short contexts; the kernels hold P in 16 bits for the
    # P*V product (the reference's TF32 dot keeps the same 10-bit mantissa) and store O in fp16, one
    # rounding of P (relative 2^-12) and half an ulp of O, under two ulps of O.  The bound is the
    # plain tolerance wherever |O| < 2.  bf16 pools hold P and V with 8 significant bits: P's
    # rounding (relative 2^-9) bounds the error by 2^-7 |O| there.
    tol = 2e-2 if kv_dtype == torch.int8 else (1e-2 if kv_dtype == torch.bfloat16 else 2e-3)
    cuh = cu.cpu().numpy()
    for bi, n in enumerate(q_len):
        got = Ov[cuh[bi]:cuh[bi] + n].float().cpu().numpy().transpose(1, 0, 2)
        want = O_or[bi, :, :n]
        if kv_dtype == torch.bfloat16:
            bound = np.maximum(tol, np.abs(want) * 2.0 ** -7)
        else:
            bound = np.maximum(tol, 2 * np.spacing(np.abs(want).astype(np.float16)).astype(np.float32))
        err = np.abs(got - want)
        assert (err <= bound).all(), f"seq {bi}: max err {err.max():.3e}, worst excess {(err - bound).max():.3e}"


def test_varlen_empty_sequences_and_clamped_start():
    from kernels.flash_attention import flash_attention_forward, flash_attention_varlen

    ctx, q_len = [300, 50, 700], [300, 0, 200]
    b = _batch(9, ctx, q_len, 8, 2, 128, torch.float16)
    args = (b.K, b.V, b.q_len, b.block_table, b.num_blocks, 16, b.kv_len, None, None)
    O, L = flash_attention_forward(b.Q, *args)
    qv, cu = _pack(b.Q, q_len)
    cu = cu.cuda()
    T = qv.shape[0]
    guard = 64
    O_big = torch.full((T + guard, 8, 128), float("nan"), dtype=torch.float16, device="cuda")
    L_big = torch.full((T + guard, 8), float("nan"), dtype=torch.float16, device="cuda")
    flash_attention_varlen(qv, cu, b.K, b.V, b.block_table, b.num_blocks, 16, b.kv_len, max_q_len=300,
                           out=O_big[:T], lse=L_big[:T])
    torch.cuda.synchronize()
    _check_rows(O_big[:T], L_big[:T], O, L, q_len, cu.cpu().numpy())
    assert torch.isnan(O_big[T:]).all() and torch.isnan(L_big[T:]).all()

    # a start offset that runs past T: that sequence's rows are clamped to the packed tensor
    bad = torch.tensor([0, 300, 300, T + 5], dtype=torch.int32, device="cuda")
    O_big.fill_(float("nan"))
    L_big.fill_(float("nan"))
    flash_attention_varlen(qv, bad, b.K, b.V, b.block_table, b.num_blocks, 16, b.kv_len, max_q_len=300,
                           out=O_big[:T], lse=L_big[:T])
    torch.cuda.synchronize()
    assert torch.isnan(O_big[T:]).all() and torch.isnan(L_big[T:]).all()
    assert torch.isfinite(O_big[:300]).all()


def test_varlen_zero_rows_is_a_no_op():
    from kernels.flash_attention import flash_attention_varlen

    b = _batch(10, [20, 30], [1, 1], 8, 8, 128, torch.float16)
    qv = torch.empty(0, 8, 128, dtype=torch.float16, device="cuda")
    cu = torch.zeros(3, dtype=torch.int32, device="cuda")
    O, L = flash_attention_varlen(qv, cu, b.K, b.V, b.block_table, b.num_blocks, 16, b.kv_len, max_q_len=0)
    torch.cuda.synchronize()
    assert O.shape == (0, 8, 128) and L.shape == (0, 8)
