"""Pin the CPU oracle against fixtures produced by the reference itself.

The fixtures (tests/golden/*.npz, generator tests/golden/make_golden.py) hold
outputs of the reference's ``quantize`` (tests/pre_quantize_test.py:3-12) and
of its Triton kernel (kernels/flash_attention.py:19-136) run by the Triton
interpreter.  CPU only.
"""
import numpy as np
import pytest

from conftest import load_golden
from oracle import paged_attention as orc

ATTN_CASES = [
    "attn_reference_test.npz",
    "attn_cfg1_fp32.npz",
    "attn_cfg1_int8_block.npz",
    "attn_cfg1_int8_token.npz",
    "attn_gqa_decode_d128.npz",
    "attn_gqa_chunked_d64.npz",
    "attn_gqa_int8_token_d128.npz",
    "attn_gqa_int8_chunked_bs32.npz",
    "attn_top_left.npz",
]


def fixture_pools(g):
    """(K, V, k_scale, v_scale) as stored in a fixture."""
    if "K_i8" in g:
        return g["K_i8"], g["V_i8"], g["k_scale"], g["v_scale"]
    return g["K"], g["V"], None, None


def test_quantize_tensor_known_answers():
    g = load_golden("quant_reference.npz")
    for i in (1, 2, 3):
        q, s = orc.quantize_tensor(g[f"x{i}"])
        assert np.array_equal(q, g[f"q{i}"]), f"case {i}"
        assert np.float32(s) == np.float32(g[f"s{i}"]), f"case {i}"
    # values printed at tests/pre_quantize_test.py:51-53
    q1, s1 = orc.quantize_tensor(g["x1"])
    err1 = np.abs(g["x1"] - q1.astype(np.float32) * s1).max()
    assert f"{s1:.6f}" == "0.064590"
    assert f"{err1:.6f}" == "0.032230"
    q3, s3 = orc.quantize_tensor(g["x3"])
    assert f"{s3:.6f}" == "0.393701"
    assert orc.quantize_tensor(g["x2"])[1] == np.float32(1.0)


def test_quantize_rows_matches_reference_per_row():
    g = load_golden("quant_reference.npz")
    q, s = orc.quantize_rows(g["rows"])
    assert np.array_equal(q, g["rows_q"])
    assert np.array_equal(s, g["rows_scale"])
    assert s[5, 2] == 1.0 and not q[5, 2].any()


@pytest.mark.parametrize("case", ATTN_CASES)
def test_oracle_matches_reference_kernel(case):
    g = load_golden(case)
    K, V, ks, vs = fixture_pools(g)
    top_left = case == "attn_top_left.npz"
    O, L = orc.paged_attention(g["Q"], K, V, g["q_len"], g["block_table"], g["num_blocks"], int(g["block_size"]),
                               g["kv_len"], ks, vs, top_left=top_left)
    for b in range(g["Q"].shape[0]):
        ql = int(g["q_len"][b])
        ref_o = g["O_ref"][b, :, :ql].astype(np.float32)
        ref_l = g["L_ref"][b, :, :ql].astype(np.float32)
        # reference O / L are fp16-rounded: half an ulp at |x| < 8 is <= 2e-3
        np.testing.assert_allclose(O[b, :, :ql], ref_o, atol=3e-3, rtol=0)
        np.testing.assert_allclose(L[b, :, :ql], ref_l, atol=1e-2, rtol=1e-3)


def test_oracle_matches_reference_test_sdpa():
    """tests/test_flash_attention.py:85-94: the paged result equals gathered SDPA."""
    g = load_golden("attn_reference_test.npz")
    O, _ = orc.paged_attention(g["Q"], g["K"], g["V"], g["q_len"], g["block_table"], g["num_blocks"],
                               int(g["block_size"]), g["kv_len"])
    for b in range(3):
        ql = int(g["q_len"][b])
        np.testing.assert_allclose(O[b, :, :ql], g["O_sdpa"][b, :, :ql], atol=1e-4, rtol=1e-4)


def test_oracle_write_then_read_round_trip():
    """Quantise-on-write then dequantise.

    The int8 value is round(x / s32) with the fp32 scale s32 (the reference
    rule) while the pool stores s16 = fp16(s32), so the error bound is half a
    step plus 127 * |s32 - s16| <= 127 * 2**-11 * s16: 0.5625 steps.
    """
    rng = np.random.default_rng(0)
    T, H, D, BS, NB = 40, 2, 64, 16, 8
    k = rng.standard_normal((T, H, D)).astype(np.float16)
    v = rng.standard_normal((T, H, D)).astype(np.float16)
    bt = rng.permutation(NB)[None, :].astype(np.int32)
    kc = np.zeros((NB, BS, H, D), np.int8)
    vc = np.zeros_like(kc)
    ksc = np.zeros((NB, BS, H), np.float16)
    vsc = np.zeros_like(ksc)
    orc.write_kv_cache(k, v, bt, np.zeros(T, np.int32), np.arange(T), kc, vc, ksc, vsc)
    back = orc.gather_sequence(kc, ksc, bt[0], T)
    step = orc.gather_sequence(np.ones_like(kc), ksc, bt[0], T)
    assert np.all(np.abs(back - k.astype(np.float32)) <= (0.5 + 127 * 2.0 ** -11) * step * 1.001)


def test_oracle_edge_cases():
    """Empty query rows, zero keys and rows without visible keys."""
    rng = np.random.default_rng(1)
    Q = rng.standard_normal((3, 2, 4, 64)).astype(np.float16)
    K = rng.standard_normal((4, 16, 2, 64)).astype(np.float16)
    bt = np.array([[0, 1], [2, 0], [3, 0]], np.int32)
    O, L = orc.paged_attention(Q, K, K, np.array([0, 2, 4]), bt, np.array([2, 1, 0]), 16,
                               np.array([20, 10, 5]))
    assert not O[0].any() and np.isneginf(L[0]).all()      # q_len 0
    assert not O[2].any() and np.isneginf(L[2, :, :4]).all()  # num_blocks 0 -> no keys
    assert np.isfinite(L[1, :, :2]).all()


def test_model_layer_fixture_is_consistent():
    """model_layer_steps.npz: the captured calls answer to the oracle and the recorded layer outputs.

    The fixture holds the reference layer's own arguments (float32 Q, INT8
    pools in the model's [NB, H, BS, D] layout, float32 per-block scales); the
    oracle on the model layout reproduces O, and W_o over the unpadded float16
    O reproduces the layer output the reference computed.
    """
    g = load_golden("model_layer_steps.npz")
    for s in range(int(g["steps"])):
        a = {k[len(f"s{s}_"):]: v for k, v in g.items() if k.startswith(f"s{s}_")}
        assert a["Q"].dtype == np.float32 and a["K"].dtype == np.int8 and a["k_scale"].dtype == np.float32
        NB, H, BS, D = a["K"].shape
        assert BS == int(a["block_size"]) and H != BS
        O, _ = orc.paged_attention(a["Q"], a["K"].transpose(0, 2, 1, 3), a["V"].transpose(0, 2, 1, 3), a["q_len"],
                                   a["block_table"], a["num_blocks"], BS, a["kv_len"], a["k_scale"], a["v_scale"])
        np.testing.assert_array_equal(O, a["O_ref"])
        T = int(a["length"].sum())
        O16 = O.astype(np.float16).astype(np.float32)
        flat = np.zeros((T, H, D), np.float32)
        for k in range(O.shape[0]):
            st, n = int(a["offset"][k]), int(a["length"][k])
            flat[st:st + n] = O16[k, :, :n].transpose(1, 0, 2)
        y = flat.reshape(T, -1) @ g["W_o"].T + g["b_o"]
        np.testing.assert_allclose(y, a["y"], atol=1e-4)
