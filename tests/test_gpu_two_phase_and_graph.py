"""Decode as two C-ABI calls (split, then reduce) and attention inside CUDA graphs.

paged_attn_decode_split + paged_attn_reduce must reproduce paged_attn_decode
exactly (the same two kernels over the same workspace, nothing in between
depends on timing).  The attention calls carry no host synchronisation and
allocate nothing once the workspace exists, so a decode step and a prefill call
can be captured in a CUDA graph and replayed with new queries; each replay must
equal an eager call on the same inputs.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _io(Q, O, L):
    from pie_b200._lib import PA_DTYPE_BF16, PA_DTYPE_F16, PaAttnIO

    io = PaAttnIO()
    io.q = Q.data_ptr()
    io.q_dtype = PA_DTYPE_BF16 if Q.dtype == torch.bfloat16 else PA_DTYPE_F16
    io.num_q_heads, io.max_q_len = Q.shape[1], Q.shape[2]
    io.q_stride_seq, io.q_stride_head, io.q_stride_row = Q.stride(0), Q.stride(1), Q.stride(2)
    io.o = O.data_ptr()
    io.o_stride_seq, io.o_stride_head, io.o_stride_row = O.stride(0), O.stride(1), O.stride(2)
    io.lse = L.data_ptr()
    io.l_stride_seq, io.l_stride_head, io.l_stride_row = L.stride(0), L.stride(1), L.stride(2)
    return io


@pytest.mark.parametrize("kv_dtype", [torch.float16, torch.int8])
def test_split_then_reduce_equals_decode(kv_dtype):
    from pie_b200 import _lib, ops
    from pie_b200.workloads import make_decode_batch

    lib = _lib.load()
    dev = torch.device("cuda", 0)
    ctx = [1, 40, 300, 1000, 2049, 17, 700, 5000, 64, 129]
    b = make_decode_batch(31, len(ctx), 32, 8, 128, 16, ctx, kv_dtype=kv_dtype, outliers=0.01).to(dev)
    want, want_l = ops.paged_attention(b.Q, b.K, b.V, b.q_len, b.block_table, b.num_blocks, 16, b.kv_len,
                                       b.k_scale, b.v_scale, mode="decode")
    keep: list = []
    kc = ops.kv_cache_desc(b.K, b.V, b.k_scale, b.v_scale)
    pg = ops.paging_desc(b.block_table, b.num_blocks, b.q_len, b.kv_len, keep)
    O = torch.full_like(want, float("nan"))
    L = torch.full_like(want_l, float("nan"))
    io = _io(b.Q, O, L)
    nbytes = ctypes.c_size_t(0)
    assert lib.paged_attn_workspace_size(io, kc, pg, ctypes.byref(nbytes)) == 0
    ws = torch.empty(nbytes.value + 256, dtype=torch.uint8, device=dev)
    wp = (ws.data_ptr() + 255) // 256 * 256
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = lib.paged_attn_decode_split(io, kc, pg, wp, nbytes.value, None, stream)
    assert rc == 0, lib.paged_attn_error_string().decode()
    torch.cuda._sleep(1000)  # unrelated work on the stream between the two calls
    rc = lib.paged_attn_reduce(io, kc, pg, wp, nbytes.value, None, stream)
    assert rc == 0, lib.paged_attn_error_string().decode()
    torch.cuda.synchronize()
    assert torch.equal(O, want), (O.float() - want.float()).abs().max().item()
    assert torch.equal(L, want_l)


def test_reduce_rejects_a_short_workspace():
    from pie_b200 import _lib, ops
    from pie_b200.workloads import make_decode_batch

    lib = _lib.load()
    b = make_decode_batch(32, 3, 8, 8, 128, 16, [50, 60, 70]).to("cuda")
    keep: list = []
    kc = ops.kv_cache_desc(b.K, b.V, b.k_scale, b.v_scale)
    pg = ops.paging_desc(b.block_table, b.num_blocks, b.q_len, b.kv_len, keep)
    O = torch.empty_like(b.Q)
    L = torch.empty(b.Q.shape[:3], dtype=torch.float16, device="cuda")
    io = _io(b.Q, O, L)
    ws = torch.empty(256, dtype=torch.uint8, device="cuda")
    rc = lib.paged_attn_reduce(io, kc, pg, ws.data_ptr(), 256, None, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.PA_ERR_WORKSPACE
    assert b"workspace" in lib.paged_attn_error_string()


@pytest.mark.parametrize("kv_dtype", [torch.float16, torch.int8])
def test_decode_step_replays_in_a_cuda_graph(kv_dtype):
    from kernels.flash_attention import flash_attention_forward
    from pie_b200.workloads import make_decode_batch

    dev = torch.device("cuda", 0)
    ctx = [33, 500, 1200, 4000, 7, 2048]
    b = make_decode_batch(41, len(ctx), 32, 8, 128, 16, ctx, kv_dtype=kv_dtype, outliers=0.01).to(dev)
    args = (b.K, b.V, b.q_len, b.block_table, b.num_blocks, 16, b.kv_len, b.k_scale, b.v_scale)
    q = b.Q.clone()
    flash_attention_forward(q, *args)  # workspace, launch plan and GPU module exist before capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        O_g, L_g = flash_attention_forward(q, *args)
    gen = torch.Generator().manual_seed(5)
    for _ in range(3):
        q.copy_(torch.randn(q.shape, generator=gen).to(q.dtype))
        g.replay()
        O_e, L_e = flash_attention_forward(q, *args)
        torch.cuda.synchronize()
        assert torch.equal(O_g, O_e)
        assert torch.equal(L_g, L_e)


def test_prefill_replays_in_a_cuda_graph():
    from kernels.flash_attention import flash_attention_forward
    from pie_b200.workloads import make_decode_batch

    dev = torch.device("cuda", 0)
    ctx = [300, 129, 1000]
    b = make_decode_batch(43, len(ctx), 8, 2, 128, 16, ctx, q_len=max(ctx)).to(dev)
    q_len = b.kv_len.clone()
    q = torch.randn(len(ctx), 8, max(ctx), 128, generator=torch.Generator().manual_seed(1)).half().to(dev)
    args = (b.K, b.V, q_len, b.block_table, b.num_blocks, 16, b.kv_len, None, None)
    flash_attention_forward(q, *args, mode="prefill")
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        O_g, L_g = flash_attention_forward(q, *args, mode="prefill")
    for seed in (2, 3):
        q.copy_(torch.randn(q.shape, generator=torch.Generator().manual_seed(seed)).half())
        g.replay()
        O_e, L_e = flash_attention_forward(q, *args, mode="prefill")
        torch.cuda.synchronize()
        for bi, n in enumerate(ctx):  # rows past q_len are left untouched
            assert torch.equal(O_g[bi, :, :n], O_e[bi, :, :n])
            assert torch.equal(L_g[bi, :, :n], L_e[bi, :, :n])
