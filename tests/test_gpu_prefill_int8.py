"""GPU: prefill over INT8 pools on the tcgen05 kernel (blocks dequantised once into fp16 scratch).

``paged_attn_forward`` / ``paged_attn_varlen`` with a workspace take this
path for head_dim 128 and block sizes >= 8; ``paged_attn_prefill`` (no
workspace) keeps the mma.sync kernel that converts inside the tile loop.
Both are checked against the oracle (2e-2, the INT8 tolerance) and against
each other; the scratch is laid out by gather (the call's table covers fewer
blocks than the pool) or as a mirror of the pool (the table's capacity is
larger), both exercised.
"""
import numpy as np
import pytest
import torch

from oracle import paged_attention as orc

pytestmark = pytest.mark.gpu

TOL_I8 = 2e-2


def _case(seed, ctx, q_lens, BS, Hq, Hkv, scale_mode, bt_cols=None, spare=5):
    gen = torch.Generator().manual_seed(seed)
    nblk = [-(-c // BS) for c in ctx]
    if spare is None:  # a pool larger than the table's capacity (gather layout)
        spare = len(ctx) * max(nblk)
    NB = sum(nblk) + spare
    perm = torch.randperm(NB, generator=gen).to(torch.int32)
    W = bt_cols or max(nblk)
    bt = torch.zeros(len(ctx), W, dtype=torch.int32)
    cur = 0
    for b, n in enumerate(nblk):
        bt[b, :n] = perm[cur:cur + n]
        cur += n
    K32 = torch.randn(NB, BS, Hkv, 128, generator=gen)
    V32 = torch.randn(NB, BS, Hkv, 128, generator=gen) * torch.where(
        torch.rand(NB, BS, Hkv, 128, generator=gen) < 0.01, 8.0, 1.0)
    if scale_mode == "block":
        kq, ks = orc.quantize_blocks(K32.numpy())
        vq, vs = orc.quantize_blocks(V32.numpy())
    else:
        kq, ks = orc.quantize_rows(K32.numpy())
        vq, vs = orc.quantize_rows(V32.numpy())
        ks, vs = ks.astype(np.float16), vs.astype(np.float16)
    Q = torch.randn(len(ctx), Hq, max(q_lens), 128, generator=gen).half()
    return Q, kq, vq, ks, vs, bt, torch.tensor(nblk, dtype=torch.int32), NB


@pytest.mark.parametrize("scale_mode", ["token16", "block"])
@pytest.mark.parametrize("layout", ["gather", "mirror"])
@pytest.mark.parametrize("BS", [16, 32])
def test_int8_prefill_on_tcgen05(scale_mode, layout, BS):
    from pie_b200 import ops

    ctx = [300, 129, 1000, 64]
    q_lens = [300, 129, 200, 1]
    # mirror: a table wider than the pool (B * bt_cols > NB) makes the scratch mirror the pool
    bt_cols = 200 if layout == "mirror" else None
    Q, kq, vq, ks, vs, bt, nblk, NB = _case(7 + BS, ctx, q_lens, BS, 8, 2, scale_mode, bt_cols,
                                            spare=5 if layout == "mirror" else None)
    assert (len(ctx) * bt.shape[1] > NB) == (layout == "mirror")
    d = dict(device="cuda")
    K, V = torch.from_numpy(kq).to(**d), torch.from_numpy(vq).to(**d)
    k_s, v_s = torch.from_numpy(ks).to(**d), torch.from_numpy(vs).to(**d)
    args = (Q.to(**d), K, V, torch.tensor(q_lens, dtype=torch.int32, **d), bt.to(**d), nblk.to(**d), BS,
            torch.tensor(ctx, dtype=torch.int32, **d), k_s, v_s)
    status = torch.zeros(1, dtype=torch.int32, **d)
    O_tc, L_tc = ops.paged_attention(*args, status=status)
    O_ms, L_ms = ops.paged_attention(*args, mode="prefill")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    O_or, L_or = orc.paged_attention(Q.float().numpy(), kq, vq, q_lens, bt.numpy(), nblk.numpy(), BS, ctx, ks, vs)
    for b, n in enumerate(q_lens):
        e_tc = np.abs(O_tc[b, :, :n].float().cpu().numpy() - O_or[b, :, :n]).max()
        e_ms = np.abs(O_ms[b, :, :n].float().cpu().numpy() - O_or[b, :, :n]).max()
        assert e_tc <= TOL_I8, f"tcgen05 path, sequence {b}: {e_tc:.3e}"
        assert e_ms <= TOL_I8, f"mma.sync path, sequence {b}: {e_ms:.3e}"
        np.testing.assert_allclose(L_tc[b, :, :n].float().cpu().numpy(), L_or[b, :, :n], atol=1e-2, rtol=1e-3)


def test_int8_prefill_workspace_and_bad_block():
    """The workspace covers the dequantised blocks; an out-of-pool block id reads as zeros with a status bit."""
    import ctypes

    from pie_b200 import _lib, ops

    Q, kq, vq, ks, vs, bt, nblk, NB = _case(3, [200, 90], [200, 90], 16, 4, 2, "token16")
    d = dict(device="cuda")
    K, V = torch.from_numpy(kq).to(**d), torch.from_numpy(vq).to(**d)
    k_s, v_s = torch.from_numpy(ks).to(**d), torch.from_numpy(vs).to(**d)
    q_len = torch.tensor([200, 90], dtype=torch.int32, **d)
    kv_len = q_len.clone()
    keep = []
    kc = ops.kv_cache_desc(K, V, k_s, v_s)
    pg = ops.paging_desc(bt.to(**d), nblk.to(**d), q_len, kv_len, keep)
    io = _lib.PaAttnIO()
    Qd = Q.to(**d)
    io.q, io.q_dtype, io.num_q_heads, io.max_q_len = Qd.data_ptr(), _lib.PA_DTYPE_F16, 4, 200
    io.q_stride_seq, io.q_stride_head, io.q_stride_row = Qd.stride(0), Qd.stride(1), Qd.stride(2)
    io.o = Qd.data_ptr()  # sizing only: the layout of an output shaped like Q
    io.o_stride_seq, io.o_stride_head, io.o_stride_row = Qd.stride(0), Qd.stride(1), Qd.stride(2)
    n = ctypes.c_size_t()
    _lib.check("paged_attn_workspace_size", _lib.load().paged_attn_workspace_size(io, kc, pg, ctypes.byref(n)))
    blocks = min(2 * bt.shape[1], NB)  # the table's blocks, or the pool when that is smaller
    assert n.value >= 2 * blocks * 16 * 2 * 128 * 2, "K and V of every block read, in fp16"
    bad = bt.clone()
    bad[1, 2] = NB + 7
    status = torch.zeros(1, dtype=torch.int32, **d)
    O, _ = ops.paged_attention(Qd, K, V, q_len, bad.to(**d), nblk.to(**d), 16, kv_len, k_s, v_s, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & _lib.PA_STATUS_BAD_BLOCK_ID
    assert torch.isfinite(O[1, :, :90].float()).all()
