"""GPU parity of quantise-on-write / copy-on-write (bit-exact).

The int8 values and scales written by the kernel must equal, bit for bit, the
reference's own ``quantize`` (tests/pre_quantize_test.py:3-12) applied to each
(token, kv head) row in float32 -- the golden fixture -- and the oracle's
restatement of it on random inputs.
"""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import paged_attention as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fa():
    from kernels import flash_attention
    assert torch.cuda.is_available()
    return flash_attention


def _layout(T, BS, extra_blocks, seed, n_seqs=3):
    rng = np.random.default_rng(seed)
    per = -(-T // n_seqs)
    nblk = -(-per // BS)
    NB = n_seqs * nblk + extra_blocks
    perm = rng.permutation(NB).astype(np.int32)
    bt = perm[: n_seqs * nblk].reshape(n_seqs, nblk)
    seq = np.repeat(np.arange(n_seqs, dtype=np.int32), per)[:T]
    pos = np.concatenate([np.arange(per, dtype=np.int32)] * n_seqs)[:T]
    return NB, bt, seq, pos


def test_quant_matches_reference_quantize_golden(fa):
    g = load_golden("quant_reference.npz")
    rows = g["rows"]  # [T, H, D] float32 (fp16-valued), one all-zero row
    T, H, D = rows.shape
    BS = 16
    NB, bt, seq, pos = _layout(T, BS, 2, 0)
    for scale_dtype in (torch.float32, torch.float16):
        kc = torch.zeros(NB, BS, H, D, dtype=torch.int8, device="cuda")
        vc = torch.zeros_like(kc)
        ks = torch.zeros(NB, BS, H, dtype=scale_dtype, device="cuda")
        vs = torch.zeros_like(ks)
        for in_dtype in (torch.float32, torch.float16):
            x = torch.from_numpy(rows).to(in_dtype).cuda()
            fa.write_kv_cache(x, x, torch.from_numpy(bt).cuda(), torch.from_numpy(seq).cuda(),
                              torch.from_numpy(pos).cuda(), kc, vc, ks, vs)
            torch.cuda.synchronize()
            kcn, ksn = kc.cpu().numpy(), ks.float().cpu().numpy()
            for t in range(T):
                blk, slot = bt[seq[t], pos[t] // BS], pos[t] % BS
                assert np.array_equal(kcn[blk, slot], g["rows_q"][t]), (t, in_dtype, scale_dtype)
                want = g["rows_scale"][t].astype(np.float16 if scale_dtype == torch.float16 else np.float32)
                assert np.array_equal(ksn[blk, slot], want.astype(np.float32)), (t, in_dtype, scale_dtype)
            assert torch.equal(kc, vc) and torch.equal(ks, vs)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("in_dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("BS", [16, 32])
def test_quant_bit_exact_vs_oracle(fa, D, in_dtype, BS):
    T, H = 300, 8
    gen = torch.Generator().manual_seed(D + BS)
    k = torch.randn(T, H, D, generator=gen)
    k = k * torch.where(torch.rand(k.shape, generator=gen) < 0.01, 8.0, 1.0)
    v = torch.randn(T, H, D, generator=gen) * 3.0
    k[7, 3] = 0.0
    k, v = k.to(in_dtype), v.to(in_dtype)
    NB, bt, seq, pos = _layout(T, BS, 5, 1)
    kc = torch.zeros(NB, BS, H, D, dtype=torch.int8, device="cuda")
    vc = torch.zeros_like(kc)
    ks = torch.zeros(NB, BS, H, dtype=torch.float16, device="cuda")
    vs = torch.zeros_like(ks)
    fa.write_kv_cache(k.cuda(), v.cuda(), torch.from_numpy(bt).cuda(), torch.from_numpy(seq).cuda(),
                      torch.from_numpy(pos).cuda(), kc, vc, ks, vs)
    torch.cuda.synchronize()
    kcn = np.zeros((NB, BS, H, D), np.int8)
    vcn = np.zeros_like(kcn)
    ksn = np.zeros((NB, BS, H), np.float16)
    vsn = np.zeros_like(ksn)
    orc.write_kv_cache(k.float().numpy(), v.float().numpy(), bt, seq, pos, kcn, vcn, ksn, vsn)
    assert np.array_equal(kc.cpu().numpy(), kcn)
    assert np.array_equal(vc.cpu().numpy(), vcn)
    assert np.array_equal(ks.cpu().numpy().view(np.uint16), ksn.view(np.uint16))
    assert np.array_equal(vs.cpu().numpy().view(np.uint16), vsn.view(np.uint16))


@pytest.mark.parametrize("H", [1, 3, 12])
@pytest.mark.parametrize("D", [64, 128])
def test_quant_near_rounding_boundaries(fa, H, D):
    """Quotients x / scale within a few ulps of k + 0.5, where x * (1 / scale)
    and the correctly rounded quotient can round to different integers, and
    head counts that leave a kv-head group of the write kernel partly empty."""
    T, BS = 64, 16
    rng = np.random.default_rng(10 * H + D)
    amax = rng.uniform(0.5, 4.0, size=(T, H)).astype(np.float32)
    s = (amax / np.float32(127.0)).astype(np.float32)
    k_int = rng.integers(-126, 126, size=(T, H, D))
    x = ((k_int + 0.5).astype(np.float32) * s[..., None]).astype(np.float32)
    x = (x.view(np.int32) + rng.integers(-3, 4, size=x.shape).astype(np.int32)).view(np.float32)
    x[..., 0] = amax  # the row's absmax, so the scale is amax / 127
    k = torch.from_numpy(x)
    v = torch.from_numpy(-x[:, :, ::-1].copy())
    NB, bt, seq, pos = _layout(T, BS, 2, 4)
    kc = torch.zeros(NB, BS, H, D, dtype=torch.int8, device="cuda")
    vc = torch.zeros_like(kc)
    ks = torch.zeros(NB, BS, H, dtype=torch.float32, device="cuda")
    vs = torch.zeros_like(ks)
    fa.write_kv_cache(k.cuda(), v.cuda(), torch.from_numpy(bt).cuda(), torch.from_numpy(seq).cuda(),
                      torch.from_numpy(pos).cuda(), kc, vc, ks, vs)
    torch.cuda.synchronize()
    kcn = np.zeros((NB, BS, H, D), np.int8)
    vcn = np.zeros_like(kcn)
    ksn = np.zeros((NB, BS, H), np.float32)
    vsn = np.zeros_like(ksn)
    orc.write_kv_cache(k.numpy(), v.numpy(), bt, seq, pos, kcn, vcn, ksn, vsn, scale_dtype=np.float32)
    assert np.array_equal(kc.cpu().numpy(), kcn)
    assert np.array_equal(vc.cpu().numpy(), vcn)
    assert np.array_equal(ks.cpu().numpy(), ksn) and np.array_equal(vs.cpu().numpy(), vsn)


@pytest.mark.parametrize("pool_dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("in_dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_copy_write_exact(fa, pool_dtype, in_dtype):
    T, H, D, BS = 100, 4, 128, 16
    k = torch.randn(T, H, D).to(in_dtype)
    v = torch.randn(T, H, D).to(in_dtype)
    NB, bt, seq, pos = _layout(T, BS, 3, 2)
    kc = torch.zeros(NB, BS, H, D, dtype=pool_dtype, device="cuda")
    vc = torch.zeros_like(kc)
    fa.write_kv_cache(k.cuda(), v.cuda(), torch.from_numpy(bt).cuda(), torch.from_numpy(seq).cuda(),
                      torch.from_numpy(pos).cuda(), kc, vc)
    torch.cuda.synchronize()
    want_k = torch.zeros(NB, BS, H, D, dtype=pool_dtype)
    want_v = torch.zeros_like(want_k)
    for t in range(T):
        blk, slot = bt[seq[t], pos[t] // BS], pos[t] % BS
        want_k[blk, slot] = k[t].to(pool_dtype)
        want_v[blk, slot] = v[t].to(pool_dtype)
    assert torch.equal(kc.cpu(), want_k) and torch.equal(vc.cpu(), want_v)


def test_write_then_attend_round_trip(fa):
    """Prefill writes K/V, decode reads them: same result as attending the oracle's pool."""
    T, H, D, BS = 200, 2, 128, 16
    gen = torch.Generator().manual_seed(9)
    k = torch.randn(T, H, D, generator=gen).half()
    v = torch.randn(T, H, D, generator=gen).half()
    NB, bt, seq, pos = _layout(T, BS, 1, 3, n_seqs=1)
    kc = torch.zeros(NB, BS, H, D, dtype=torch.int8, device="cuda")
    vc = torch.zeros_like(kc)
    ks = torch.zeros(NB, BS, H, dtype=torch.float16, device="cuda")
    vs = torch.zeros_like(ks)
    btc = torch.from_numpy(bt).cuda()
    fa.write_kv_cache(k.cuda(), v.cuda(), btc, torch.from_numpy(seq).cuda(), torch.from_numpy(pos).cuda(),
                      kc, vc, ks, vs)
    q = torch.randn(1, 4, 1, D, generator=gen).half()
    one = torch.ones(1, dtype=torch.int32, device="cuda")
    O, _ = fa.flash_attention_forward(q.cuda(), kc, vc, one, btc, torch.tensor([bt.shape[1]], dtype=torch.int32).cuda(),
                                      BS, torch.tensor([T], dtype=torch.int32).cuda(), ks, vs)
    torch.cuda.synchronize()
    O_or, _ = orc.paged_attention(q.float().numpy(), kc.cpu().numpy(), vc.cpu().numpy(), [1], bt, [bt.shape[1]], BS,
                                  [T], ks.cpu().numpy(), vs.cpu().numpy())
    assert np.abs(O.float().cpu().numpy() - O_or).max() < 2e-2


def test_bad_positions_set_status():
    from pie_b200 import ops
    H, D, BS = 2, 64, 16
    kc = torch.zeros(4, BS, H, D, dtype=torch.int8, device="cuda")
    ks = torch.zeros(4, BS, H, dtype=torch.float16, device="cuda")
    bt = torch.tensor([[0, 1], [2, 7]], dtype=torch.int32, device="cuda")
    x = torch.randn(3, H, D, device="cuda").half()
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.write_kv(x, x, bt, torch.tensor([0, 1, 5], dtype=torch.int32, device="cuda"),
                 torch.tensor([40, 20, 0], dtype=torch.int32, device="cuda"), kc, kc.clone(), ks, ks.clone(), status=st)
    torch.cuda.synchronize()
    v = int(st.item())
    assert v & 2 and v & 1 and v & 8, hex(v)  # position past table, block 7 outside pool, seq 5 outside table
