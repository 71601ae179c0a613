"""GPU: the K/V projection with the cache write in its epilogue (kv_project_write).

Checked against the same projection computed in float32 on the CPU from the
same 16-bit inputs (x @ W^T + b, transformer/model.py:75-82) and written with
the oracle's rule.  The GPU accumulates in float32 in another order, so a
value can differ in its last bits: an INT8 code may differ by one where the
quotient lies within 2e-3 of a rounding boundary (at most 0.1 % of the codes),
an fp16 scale by one unit in its last place, an fp32 scale by 1e-5
relative (the absmax's own accumulation-order error); float16 pools hold
the rounded value (relative 2e-3).
"""
import numpy as np
import pytest
import torch

from oracle import paged_attention as orc

pytestmark = pytest.mark.gpu


def _setup(seed, T_per_seq, d_model, Hkv, BS, dtype):
    gen = torch.Generator().manual_seed(seed)
    D = 128
    nseq = len(T_per_seq)
    start = [int(torch.randint(0, 40, (1,), generator=gen)) for _ in range(nseq)]
    nblk = [-(-(s + t) // BS) for s, t in zip(start, T_per_seq)]
    NB = sum(nblk) + 4
    perm = torch.randperm(NB, generator=gen).to(torch.int32)
    bt = torch.zeros(nseq, max(nblk), dtype=torch.int32)
    cur = 0
    for b, n in enumerate(nblk):
        bt[b, :n] = perm[cur:cur + n]
        cur += n
    seq = torch.cat([torch.full((t,), b, dtype=torch.int32) for b, t in enumerate(T_per_seq)])
    pos = torch.cat([torch.arange(s, s + t, dtype=torch.int32) for s, t in zip(start, T_per_seq)])
    T = int(seq.numel())
    x = (torch.randn(T, d_model, generator=gen) * 0.5).to(dtype)
    w = (torch.randn(2 * Hkv * D, d_model, generator=gen) / d_model ** 0.5).to(dtype)
    bias = torch.randn(2 * Hkv * D, generator=gen) * 0.1
    ref = (x.float() @ w.float().T + bias).view(T, 2, Hkv, D)  # [T, K/V, head, D]
    return x, w, bias, bt, seq, pos, ref, NB


@pytest.mark.parametrize("backend", ["torch", "ctypes"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("pool", ["i8_f16scale", "i8_f32scale", "f16"])
@pytest.mark.parametrize("shape", [(256, 2, 16), (1024, 8, 16), (512, 4, 32)])
def test_projection_write_matches_float32(backend, dtype, pool, shape):
    _check_projection(backend, dtype, pool, shape, [130, 7, 163])


@pytest.mark.parametrize("pool", ["i8_f16scale", "f16"])
def test_projection_write_many_tiles_per_cta(pool):
    """20100 tokens x 8 heads: ~1260 tiles, so every CTA of the persistent grid
    walks several tiles and both TMEM accumulators take turns."""
    _check_projection("torch", torch.bfloat16, pool, (512, 8, 16), [7000, 9000, 4100])


@pytest.mark.parametrize("pool", ["i8_f16scale", "f16"])
@pytest.mark.parametrize("t_per_seq", [[30, 34], [1, 5, 2], [120, 80, 55]])
def test_projection_write_small_batch_cluster_split(pool, t_per_seq):
    """Decode-sized batches: few 128-token tiles, so d_model is split across the
    CTAs of a cluster (eight here: 8 heads, d_model 1024) and the partial tiles
    are summed through distributed shared memory before the epilogue."""
    _check_projection("torch", torch.bfloat16, pool, (1024, 8, 16), t_per_seq)


def _check_projection(backend, dtype, pool, shape, t_per_seq):
    from pie_b200 import ops
    from pie_b200.workloads import empty_head_major_scales

    d_model, Hkv, BS = shape
    x, w, bias, bt, seq, pos, ref, NB = _setup(11, t_per_seq, d_model, Hkv, BS, dtype)
    dev = torch.device("cuda")
    D = 128
    if pool.startswith("i8"):
        sdt = torch.float16 if pool == "i8_f16scale" else torch.float32
        K = torch.zeros(NB, BS, Hkv, D, dtype=torch.int8, device=dev)
        ks = empty_head_major_scales(NB, BS, Hkv, dtype=sdt, device=dev).zero_()
        vs = empty_head_major_scales(NB, BS, Hkv, dtype=sdt, device=dev).zero_()
    else:
        K = torch.zeros(NB, BS, Hkv, D, dtype=torch.float16, device=dev)
        ks = vs = None
    V = torch.zeros_like(K)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    saved = ops.BACKEND
    try:
        ops.BACKEND = backend
        ops.project_write_kv(x.to(dev), w.to(dev), bias.to(dev), bt.to(dev), seq.to(dev), pos.to(dev), K, V, ks, vs,
                             status=status)
        torch.cuda.synchronize()
    finally:
        ops.BACKEND = saved
    assert int(status.item()) == 0
    blk = bt[seq.long(), (pos // BS).long()].numpy()
    slot = (pos % BS).numpy()
    mism = total = 0
    for kv, pool_t, sc_t in ((0, K, ks), (1, V, vs)):
        got = pool_t.cpu().numpy()[blk, slot]  # [T, Hkv, D]
        want = ref[:, kv].numpy()
        if pool_t.dtype == torch.int8:
            q_ref, s_ref = orc.quantize_rows(want)  # fp32 rule of the reference
            s_got = sc_t.float().cpu().numpy()[blk, slot]
            if sc_t.dtype == torch.float16:  # one fp16 ulp
                s_ref_st = s_ref.astype(np.float16)
                tol = np.spacing(np.abs(s_ref_st)).astype(np.float32)
            else:  # the row's absmax carries the accumulation-order error of a d_model-long dot product
                s_ref_st = s_ref
                tol = 1e-5 * np.abs(s_ref)
            assert (np.abs(s_got - s_ref_st.astype(np.float32)) <= tol).all(), "scales"
            d = np.abs(got.astype(np.int32) - q_ref.astype(np.int32))
            assert d.max() <= 1, "INT8 codes differ by more than one"
            y = want / s_ref[..., None]
            near = np.abs(np.abs(y - np.trunc(y)) - 0.5) < 2e-3
            assert not (d.astype(bool) & ~near).any(), "an INT8 code differs away from a rounding boundary"
            mism += int(d.astype(bool).sum())
            total += d.size
        else:
            np.testing.assert_allclose(got.astype(np.float32), want, rtol=2e-3, atol=2e-3)
    assert mism <= 1e-3 * max(total, 1)


def test_drop_in_entry_writes_like_write_kv_cache():
    """kernels.flash_attention.project_write_kv_cache == projection on the host + write_kv_cache."""
    from kernels.flash_attention import project_write_kv_cache, write_kv_cache
    from pie_b200.workloads import empty_head_major_scales

    x, w, bias, bt, seq, pos, ref, NB = _setup(5, [64, 200], 384, 3, 16, torch.bfloat16)
    dev = torch.device("cuda")
    out = []
    for fused in (True, False):
        K = torch.zeros(NB, 16, 3, 128, dtype=torch.int8, device=dev)
        V = torch.zeros_like(K)
        ks = empty_head_major_scales(NB, 16, 3, device=dev).zero_()
        vs = empty_head_major_scales(NB, 16, 3, device=dev).zero_()
        if fused:
            project_write_kv_cache(x.to(dev), w.to(dev), bias.to(dev), bt.to(dev), seq.to(dev), pos.to(dev), K, V,
                                   ks, vs)
        else:
            kv = ref.to(dev)  # float32 rows, the same rule applied by the write kernel
            write_kv_cache(kv[:, 0].contiguous(), kv[:, 1].contiguous(), bt.to(dev), seq.to(dev), pos.to(dev), K, V,
                           ks, vs)
        out.append((K.cpu(), V.cpu(), ks.float().cpu(), vs.float().cpu()))
    torch.cuda.synchronize()
    for a, b in zip(out[0], out[1]):
        d = (a.float() - b.float()).abs()
        assert d.max() <= (1 if a.dtype == torch.int8 else 1e-2 * b.float().abs().max())
        assert (d > 0).float().mean() <= 1e-3


def test_projection_write_bad_sequence_index():
    """A token whose sequence row is outside the block table is skipped and reported."""
    from pie_b200 import _lib, ops
    from pie_b200.workloads import empty_head_major_scales

    x, w, bias, bt, seq, pos, ref, NB = _setup(3, [40, 9], 256, 2, 16, torch.bfloat16)
    seq[5] = 7
    dev = torch.device("cuda")
    K = torch.zeros(NB, 16, 2, 128, dtype=torch.int8, device=dev)
    V = torch.zeros_like(K)
    ks = empty_head_major_scales(NB, 16, 2, device=dev).zero_()
    vs = empty_head_major_scales(NB, 16, 2, device=dev).zero_()
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.project_write_kv(x.to(dev), w.to(dev), None, bt.to(dev), seq.to(dev), pos.to(dev), K, V, ks, vs,
                         status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & _lib.PA_STATUS_BAD_SEQ_INDEX
