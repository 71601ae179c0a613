"""GPU parity: the sm_100a kernels (through the C ABI) against the CPU oracle
and against the reference kernel's own outputs (golden fixtures).

Tolerances (max-abs on O, the reference's float16 output):
  * float16 / bfloat16 pools: 2e-3 against the float32 oracle;
  * INT8 pools: 2e-2 against the oracle on the same int8 values and scales;
  * against the reference's fp16-rounded outputs add half an fp16 ulp (1e-3).
"""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import paged_attention as orc

pytestmark = pytest.mark.gpu

TOL_F16 = 2e-3
TOL_I8 = 2e-2
TOL_L = 1e-2  # log-sum-exp in float16 (|L| < 16: half-ulp 4e-3 plus math)

GOLDEN_CASES = {
    # name: (top_left, int8)
    "attn_reference_test.npz": (False, False),
    "attn_cfg1_fp32.npz": (False, False),
    "attn_cfg1_int8_block.npz": (False, True),
    "attn_cfg1_int8_token.npz": (False, True),
    "attn_gqa_decode_d128.npz": (False, False),
    "attn_gqa_chunked_d64.npz": (False, False),
    "attn_gqa_int8_token_d128.npz": (False, True),
    "attn_gqa_int8_chunked_bs32.npz": (False, True),
    "attn_top_left.npz": (True, False),
}


@pytest.fixture(scope="module")
def fa():
    from kernels import flash_attention
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return flash_attention


def _cuda(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    return t.to(dtype) if dtype is not None else t


def _pools(g):
    if "K_i8" in g:
        return (_cuda(g["K_i8"]), _cuda(g["V_i8"]), _cuda(g["k_scale"]), _cuda(g["v_scale"]),
                g["K_i8"], g["V_i8"], g["k_scale"], g["v_scale"])
    return _cuda(g["K"]), _cuda(g["V"]), None, None, g["K"], g["V"], None, None


def _compare(O, L, O_exp, L_exp, q_len, tol, what):
    O = O.float().cpu().numpy()
    L = L.float().cpu().numpy()
    worst = 0.0
    for b in range(O.shape[0]):
        ql = int(q_len[b])
        if ql == 0:
            continue
        d = np.abs(O[b, :, :ql] - O_exp[b, :, :ql]).max()
        worst = max(worst, d)
        fin = np.isfinite(L_exp[b, :, :ql])
        assert np.array_equal(np.isfinite(L[b, :, :ql]), fin), f"{what}: seq {b} L finiteness"
        if fin.any():
            np.testing.assert_allclose(L[b, :, :ql][fin], L_exp[b, :, :ql][fin], atol=TOL_L, rtol=1e-3,
                                       err_msg=f"{what}: seq {b} L")
    assert worst <= tol, f"{what}: max |O - expected| = {worst:.3e} > {tol:.1e}"
    return worst


@pytest.mark.parametrize("case", sorted(GOLDEN_CASES))
@pytest.mark.parametrize("mode", ["auto", "prefill", "decode"])
def test_golden_fixture(fa, case, mode):
    top_left, int8 = GOLDEN_CASES[case]
    g = load_golden(case)
    B, Hq, maxq, D = g["Q"].shape
    K, V, ks, vs, Kn, Vn, ksn, vsn = _pools(g)
    G = Hq // K.shape[2]
    if mode == "decode" and maxq * G > 16:
        pytest.skip("decode kernel packs at most 16 (row x head) columns")
    Q = _cuda(g["Q"])
    O, L = fa.flash_attention_forward(Q, K, V, _cuda(g["q_len"]), _cuda(g["block_table"]), _cuda(g["num_blocks"]),
                                      int(g["block_size"]), _cuda(g["kv_len"]), ks, vs, causal_top_left=top_left,
                                      mode=mode)
    torch.cuda.synchronize()
    O_or, L_or = orc.paged_attention(g["Q"], Kn, Vn, g["q_len"], g["block_table"], g["num_blocks"],
                                     int(g["block_size"]), g["kv_len"], ksn, vsn, top_left=top_left)
    tol = TOL_I8 if int8 else TOL_F16
    _compare(O, L, O_or, L_or, g["q_len"], tol, f"{case}/{mode} vs oracle")
    _compare(O, L, g["O_ref"].astype(np.float32), g["L_ref"].astype(np.float32), g["q_len"], tol + 1e-3,
             f"{case}/{mode} vs reference kernel")


def _random_case(seed, B, Hq, Hkv, D, BS, ctx, q_lens, kv_dtype, q_dtype, scale_mode):
    gen = torch.Generator().manual_seed(seed)
    nblk = [max(1, -(-c // BS)) for c in ctx]
    NB = sum(nblk) + 4
    perm = torch.randperm(NB, generator=gen).to(torch.int32)
    bt = torch.zeros(B, max(nblk) + 1, dtype=torch.int32)  # one spare column
    cur = 0
    for b, n in enumerate(nblk):
        bt[b, :n] = perm[cur:cur + n]
        cur += n
    Q = torch.randn(B, Hq, max(q_lens), D, generator=gen)
    K16 = torch.randn(NB, BS, Hkv, D, generator=gen)
    V16 = torch.randn(NB, BS, Hkv, D, generator=gen)
    ks = vs = None
    if kv_dtype == torch.int8:
        if scale_mode == "block":
            kq, ksn = orc.quantize_blocks(K16.numpy())
            vq, vsn = orc.quantize_blocks(V16.numpy())
        else:
            kq, ksn = orc.quantize_rows(K16.numpy())
            vq, vsn = orc.quantize_rows(V16.numpy())
            if scale_mode == "token16":
                ksn, vsn = ksn.astype(np.float16), vsn.astype(np.float16)
        Kn, Vn = kq, vq
        ks, vs = torch.from_numpy(ksn), torch.from_numpy(vsn)
        K, V = torch.from_numpy(kq), torch.from_numpy(vq)
    else:
        K, V = K16.to(kv_dtype), V16.to(kv_dtype)
        Kn, Vn = K.float().numpy(), V.float().numpy()
        ksn = vsn = None
    Q = Q.to(q_dtype)
    meta = dict(q_len=torch.tensor(q_lens, dtype=torch.int32), kv_len=torch.tensor(ctx, dtype=torch.int32),
                num_blocks=torch.tensor(nblk, dtype=torch.int32), block_table=bt)
    return Q, K, V, ks, vs, Kn, Vn, ksn, vsn, meta


RANDOM = [
    # (Hq, Hkv, D, BS, kv_dtype, q_dtype, scale_mode, q_max)
    (32, 8, 128, 16, torch.float16, torch.float16, None, 1),
    (32, 8, 128, 16, torch.bfloat16, torch.bfloat16, None, 1),
    (32, 8, 128, 16, torch.int8, torch.float16, "token16", 1),
    (32, 8, 128, 16, torch.int8, torch.bfloat16, "token16", 1),
    (64, 8, 128, 16, torch.int8, torch.float16, "token16", 1),
    (64, 8, 128, 16, torch.int8, torch.float16, "token16", 2),
    (8, 8, 64, 16, torch.float16, torch.float16, None, 1),
    (8, 8, 64, 64, torch.int8, torch.float16, "block", 1),
    (8, 8, 64, 16, torch.int8, torch.float16, "token32", 3),
    (16, 2, 128, 32, torch.float16, torch.bfloat16, None, 2),
    (4, 4, 128, 8, torch.float16, torch.float16, None, 4),
    (4, 1, 64, 4, torch.bfloat16, torch.bfloat16, None, 4),
    (16, 4, 64, 128, torch.float16, torch.float16, None, 1),
]


@pytest.mark.parametrize("cfg", RANDOM, ids=lambda c: f"{c[0]}x{c[1]}_d{c[2]}_bs{c[3]}_{str(c[4])[6:]}_{str(c[5])[6:]}_{c[6]}_q{c[7]}")
@pytest.mark.parametrize("top_left", [False, True])
@pytest.mark.parametrize("mode", ["auto", "prefill"])
def test_random_vs_oracle(fa, cfg, top_left, mode):
    Hq, Hkv, D, BS, kv_dtype, q_dtype, scale_mode, qmax = cfg
    ctx = [1, 15, 16, 17, 33, 200, 517, 1000]
    q_lens = [min(qmax, c) if i % 3 else 1 for i, c in enumerate(ctx)]
    q_lens[-1] = qmax
    Q, K, V, ks, vs, Kn, Vn, ksn, vsn, meta = _random_case(RANDOM.index(cfg) * 2 + top_left, len(ctx), Hq, Hkv, D, BS,
                                                           ctx, q_lens, kv_dtype, q_dtype, scale_mode)
    O, L = fa.flash_attention_forward(Q.cuda(), K.cuda(), V.cuda(), meta["q_len"].cuda(), meta["block_table"].cuda(),
                                      meta["num_blocks"].cuda(), BS, meta["kv_len"].cuda(),
                                      None if ks is None else ks.cuda(), None if vs is None else vs.cuda(),
                                      causal_top_left=top_left, mode=mode)
    torch.cuda.synchronize()
    O_or, L_or = orc.paged_attention(Q.float().numpy(), Kn, Vn, meta["q_len"].numpy(), meta["block_table"].numpy(),
                                     meta["num_blocks"].numpy(), BS, meta["kv_len"].numpy(), ksn, vsn,
                                     top_left=top_left)
    tol = TOL_I8 if kv_dtype == torch.int8 else TOL_F16
    if q_dtype != kv_dtype and kv_dtype != torch.int8:
        tol = 4e-3  # Q rounded to the pool's 16-bit type before the MMA
    if kv_dtype == torch.bfloat16:
        tol = max(tol, 1e-2)  # bf16 P/V operands: 8-bit significands
    _compare(O, L, O_or, L_or, meta["q_len"].numpy(), tol, f"{cfg}")


@pytest.mark.parametrize("kv", ["f16", "i8"])
@pytest.mark.parametrize("mode", ["decode", "prefill"])
def test_rising_logits_vs_oracle(fa, kv, mode):
    """Key norms that grow ~13x along each sequence: the kernels' reference
    max has to move again and again (their rescale paths), also inside split-K
    pieces, and the softmax ends up dominated by a few late keys."""
    B, Hq, Hkv, D, BS = 3, 8, 2, 128, 16
    ctx = [300, 1000, 2049]
    gen = torch.Generator().manual_seed(77)
    nblk = [-(-c // BS) for c in ctx]
    NB = sum(nblk)
    perm = torch.randperm(NB, generator=gen).to(torch.int32)
    bt = torch.zeros(B, max(nblk), dtype=torch.int32)
    growth = torch.ones(NB, BS)
    cur = 0
    for b, n in enumerate(nblk):
        bt[b, :n] = perm[cur:cur + n]
        cur += n
        pos = torch.arange(n * BS, dtype=torch.float32).view(n, BS)
        growth[bt[b, :n].long()] = 1.0 + pos * (12.0 / ctx[b])
    K16 = torch.randn(NB, BS, Hkv, D, generator=gen) * growth[:, :, None, None]
    V16 = torch.randn(NB, BS, Hkv, D, generator=gen)
    Q = torch.randn(B, Hq, 1, D, generator=gen).half()
    if kv == "i8":
        kq, ksn = orc.quantize_rows(K16.numpy())
        vq, vsn = orc.quantize_rows(V16.numpy())
        ksn, vsn = ksn.astype(np.float16), vsn.astype(np.float16)
        K, V, ks, vs, Kn, Vn = torch.from_numpy(kq), torch.from_numpy(vq), torch.from_numpy(ksn), \
            torch.from_numpy(vsn), kq, vq
    else:
        K, V = K16.half(), V16.half()
        ks = vs = ksn = vsn = None
        Kn, Vn = K.float().numpy(), V.float().numpy()
    q_len = torch.ones(B, dtype=torch.int32)
    kv_len = torch.tensor(ctx, dtype=torch.int32)
    nb = torch.tensor(nblk, dtype=torch.int32)
    O, L = fa.flash_attention_forward(Q.cuda(), K.cuda(), V.cuda(), q_len.cuda(), bt.cuda(), nb.cuda(), BS,
                                      kv_len.cuda(), None if ks is None else ks.cuda(),
                                      None if vs is None else vs.cuda(), mode=mode)
    torch.cuda.synchronize()
    O_or, L_or = orc.paged_attention(Q.float().numpy(), Kn, Vn, q_len.numpy(), bt.numpy(), nb.numpy(), BS,
                                     kv_len.numpy(), ksn, vsn)
    _compare(O, L, O_or, L_or, q_len.numpy(), TOL_I8 if kv == "i8" else TOL_F16, f"rising {kv} {mode}")


@pytest.mark.parametrize("kernel", ["paired", "single"])
def test_extreme_logit_range_prefill(fa, kernel, monkeypatch):
    """Causal prefill where the keys of the first 64 of every 128 are ~140
    log2 units below the others (their probabilities underflow), and keys of
    the second tile sit ~30 log2 units above the first tile's maximum (every
    row's O is rescaled at tile 1).  Run on the paired-head tensor-core kernel
    (even GQA group) and on the single-head one."""
    if kernel == "single":
        monkeypatch.setenv("PIE_B200_TC_SINGLE", "1")
    B, Hq, Hkv, D, BS = 2, 8, 2, 128, 16
    ctx = [300, 260]
    gen = torch.Generator().manual_seed(91)
    nblk = [-(-c // BS) for c in ctx]
    NB = sum(nblk) + 3
    perm = torch.randperm(NB, generator=gen).to(torch.int32)
    bt = torch.zeros(B, max(nblk), dtype=torch.int32)
    K = torch.randn(NB, BS, Hkv, D, generator=gen) * 0.1
    V = torch.randn(NB, BS, Hkv, D, generator=gen)
    cur = 0
    for b, n in enumerate(nblk):
        bt[b, :n] = perm[cur:cur + n]
        cur += n
        for i in range(n):
            pos = i * BS + torch.arange(BS)
            comp = torch.where(pos % 128 < 64, -40.0, 30.0)
            comp = torch.where((pos >= 128) & (pos % 128 >= 64), 45.0, comp)
            K[bt[b, i].long(), :, :, 0] = comp[:, None]
    K = K.half()
    V = V.half()
    maxq = max(ctx)
    Q = torch.randn(B, Hq, maxq, D, generator=gen) * 0.1
    Q[..., 0] = 16.0
    Q = Q.half()
    q_len = torch.tensor(ctx, dtype=torch.int32)
    kv_len = torch.tensor(ctx, dtype=torch.int32)
    nb = torch.tensor(nblk, dtype=torch.int32)
    O, L = fa.flash_attention_forward(Q.cuda(), K.cuda(), V.cuda(), q_len.cuda(), bt.cuda(), nb.cuda(), BS,
                                      kv_len.cuda(), None, None, mode="prefill")
    torch.cuda.synchronize()
    O_or, L_or = orc.paged_attention(Q.float().numpy(), K.float().numpy(), V.float().numpy(), q_len.numpy(),
                                     bt.numpy(), nb.numpy(), BS, kv_len.numpy(), None, None)
    _compare(O, L, O_or, L_or, q_len.numpy(), TOL_F16, f"extreme logits {kernel}")


def test_repeated_decode_calls_share_one_workspace(fa):
    """Alternating batch shapes (different grid chunking) through one
    workspace, three rounds: every call must match the oracle."""
    cases = []
    for seed, ctx in ((21, [700, 1, 3000, 45]), (22, [5000, 130]), (23, [17] * 9 + [2500])):
        Q, K, V, ks, vs, Kn, Vn, ksn, vsn, meta = _random_case(seed, len(ctx), 16, 4, 128, 16, ctx, [1] * len(ctx),
                                                               torch.int8, torch.float16, "token16")
        O_or, L_or = orc.paged_attention(Q.float().numpy(), Kn, Vn, meta["q_len"].numpy(),
                                         meta["block_table"].numpy(), meta["num_blocks"].numpy(), 16,
                                         meta["kv_len"].numpy(), ksn, vsn)
        dev = [Q.cuda(), K.cuda(), V.cuda(), meta["q_len"].cuda(), meta["block_table"].cuda(),
               meta["num_blocks"].cuda(), 16, meta["kv_len"].cuda(), ks.cuda(), vs.cuda()]
        cases.append((dev, O_or, L_or, meta["q_len"].numpy()))
    for rep in range(3):
        for i, (dev, O_or, L_or, ql) in enumerate(cases):
            O, L = fa.flash_attention_forward(*dev, mode="decode")
            torch.cuda.synchronize()
            _compare(O, L, O_or, L_or, ql, TOL_I8, f"call {rep}/{i}")


def test_edge_cases(fa):
    """q_len 0, kv_len 0, num_blocks 0 and keys beyond num_blocks*block_size."""
    BS, D, H = 16, 128, 4
    NB = 6
    g = torch.Generator().manual_seed(5)
    K = torch.randn(NB, BS, H, D, generator=g).half().cuda()
    V = torch.randn(NB, BS, H, D, generator=g).half().cuda()
    bt = torch.tensor([[0, 1, 2], [3, 4, 5], [1, 0, 0], [2, 3, 0]], dtype=torch.int32).cuda()
    q_len = torch.tensor([0, 1, 1, 1], dtype=torch.int32).cuda()
    kv_len = torch.tensor([10, 0, 20, 40], dtype=torch.int32).cuda()
    nblk = torch.tensor([3, 3, 0, 2], dtype=torch.int32).cuda()  # seq 3: 40 keys but 2 blocks -> 32 keys
    Q = torch.randn(4, H, 1, D, generator=g).half().cuda()
    for mode in ("decode", "prefill"):
        O = torch.full((4, H, 1, D), 7.0, dtype=torch.float16, device="cuda")
        O, L = fa.flash_attention_forward(Q, K, V, q_len, bt, nblk, BS, kv_len, None, None, out=O, mode=mode)
        torch.cuda.synchronize()
        assert (O[0] == 7.0).all(), "q_len 0 rows must stay untouched"
        assert (O[1] == 0).all() and torch.isinf(L[1]).all(), "no keys -> O = 0, L = -inf"
        assert (O[2] == 0).all() and torch.isinf(L[2]).all(), "num_blocks 0 -> no keys"
        O_or, _ = orc.paged_attention(Q.float().cpu().numpy(), K.cpu().numpy(), V.cpu().numpy(),
                                      q_len.cpu().numpy(), bt.cpu().numpy(), nblk.cpu().numpy(), BS,
                                      kv_len.cpu().numpy())
        assert np.abs(O[3].float().cpu().numpy() - O_or[3]).max() < TOL_F16


def test_bad_block_id_sets_status(fa):
    """An out-of-pool block id is skipped (zero row) and reported, never dereferenced."""
    from pie_b200 import ops
    BS, D, H = 16, 64, 2
    K = torch.randn(4, BS, H, D, device="cuda").half()
    bt = torch.tensor([[0, 99]], dtype=torch.int32, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    Q = torch.randn(1, H, 1, D, device="cuda").half()
    for mode in ("decode", "prefill"):
        st.zero_()
        ops.paged_attention(Q, K, K, torch.ones(1, dtype=torch.int32, device="cuda"), bt,
                            torch.tensor([2], dtype=torch.int32, device="cuda"), BS,
                            torch.tensor([30], dtype=torch.int32, device="cuda"), mode=mode, status=st)
        torch.cuda.synchronize()
        assert int(st.item()) & 1, mode


def test_outputs_on_q_device_and_no_sync(fa):
    """Outputs are allocated on Q.device (the reference used a module global)."""
    g = load_golden("attn_gqa_decode_d128.npz")
    K, V, *_ = _pools(g)
    O, L = fa.flash_attention_forward(_cuda(g["Q"]), K, V, _cuda(g["q_len"]), _cuda(g["block_table"]),
                                      _cuda(g["num_blocks"]), int(g["block_size"]), _cuda(g["kv_len"]), None, None)
    assert O.device == K.device and O.dtype == torch.float16 and L.dtype == torch.float16
    assert tuple(O.shape) == g["Q"].shape


def test_autograd_wrapper(fa):
    g = load_golden("attn_reference_test.npz")
    args = (_cuda(g["Q"]), _cuda(g["K"]), _cuda(g["V"]), _cuda(g["q_len"]), _cuda(g["block_table"]),
            _cuda(g["num_blocks"]), int(g["block_size"]), _cuda(g["kv_len"]), None, None)
    O = fa.FlashAttentionFunction.apply(*args)
    O2, _ = fa.flash_attention_forward(*args)
    for b, ql in enumerate(g["q_len"]):  # rows >= q_len are left unwritten, as in the reference
        assert torch.equal(O[b, :, :ql], O2[b, :, :ql])
