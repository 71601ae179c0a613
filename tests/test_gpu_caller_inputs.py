"""GPU parity for the inputs the reference's own caller sends.

The reference's attention layer (transformer/model.py:69-173) calls the
kernel with:
  * a float32 Q holding arbitrary values (the layer computes in float32,
    transformer/model.py:75, :135, :156-160);
  * INT8 pools in the model's own [num_blocks, heads, block_size, d_k] layout
    (transformer/model.py:64-65) with float32 per-(block, head) scales
    (:66-67);
and the reference kernel itself accepts float32 pools
(kernels/flash_attention.py:79-84).  Every case here is checked against the
CPU oracle evaluated on the same float32 inputs.

Tolerances (max-abs on O, float16 output):
  * float16 / float32 pools: 2e-3 (Q and float32 K/V are rounded to float16
    operands, the 11-bit significand of the reference's TF32 dot);
  * bfloat16 pools: 1e-2 (float32 Q is rounded to bfloat16);
  * INT8 pools: 2e-2.
"""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import paged_attention as orc

pytestmark = pytest.mark.gpu

TOL_F16 = 2e-3
TOL_BF16 = 1e-2
TOL_I8 = 2e-2


@pytest.fixture(scope="module")
def fa():
    from kernels import flash_attention
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return flash_attention


def _max_err(O, O_exp, q_len):
    O = O.float().cpu().numpy()
    worst = 0.0
    for b in range(O.shape[0]):
        ql = int(q_len[b])
        if ql:
            worst = max(worst, float(np.abs(O[b, :, :ql] - O_exp[b, :, :ql]).max()))
    return worst


def _tables(gen, ctx, BS, spare=3):
    nblk = [max(1, -(-c // BS)) for c in ctx]
    NB = sum(nblk) + spare
    perm = torch.randperm(NB, generator=gen).to(torch.int32)
    bt = torch.zeros(len(ctx), max(nblk), dtype=torch.int32)
    cur = 0
    for b, n in enumerate(nblk):
        bt[b, :n] = perm[cur:cur + n]
        cur += n
    return bt, torch.tensor(nblk, dtype=torch.int32), NB


CASES = [
    # (B, Hq, Hkv, D, BS, ctx, q_lens)
    (5, 8, 2, 128, 16, [37, 128, 300, 16, 1], [1, 1, 1, 1, 1]),     # GQA decode
    (3, 4, 4, 64, 16, [40, 90, 16], [1, 1, 1]),                      # MHA decode, D=64
    (3, 8, 2, 128, 16, [200, 70, 129], [200, 33, 1]),               # prefill / chunked
    (2, 4, 2, 64, 32, [65, 90], [65, 7]),                            # BS=32, D=64
]


@pytest.mark.parametrize("case", range(len(CASES)))
@pytest.mark.parametrize("pool", ["f16", "bf16", "f32", "i8_token", "i8_block"])
def test_float32_q_with_arbitrary_values(fa, case, pool):
    """float32 Q drawn in float32 (not float16-representable) against the oracle on that Q."""
    B, Hq, Hkv, D, BS, ctx, q_lens = CASES[case]
    gen = torch.Generator().manual_seed(100 + case)
    bt, nblk, NB = _tables(gen, ctx, BS)
    Q = torch.randn(B, Hq, max(q_lens), D, generator=gen, dtype=torch.float32)
    K32 = torch.randn(NB, BS, Hkv, D, generator=gen)
    V32 = torch.randn(NB, BS, Hkv, D, generator=gen)
    ks = vs = ksn = vsn = None
    if pool.startswith("i8"):
        quant = orc.quantize_blocks if pool == "i8_block" else orc.quantize_rows
        kq, ksn = quant(K32.numpy())
        vq, vsn = quant(V32.numpy())
        Kn, Vn = kq, vq
        K, V = torch.from_numpy(kq), torch.from_numpy(vq)
        ks, vs = torch.from_numpy(ksn).cuda(), torch.from_numpy(vsn).cuda()
        tol = TOL_I8
    else:
        dt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[pool]
        K, V = K32.to(dt), V32.to(dt)
        Kn, Vn = K.float().numpy(), V.float().numpy()
        tol = TOL_BF16 if pool == "bf16" else TOL_F16
    assert not torch.equal(Q, Q.half().float()), "Q must hold values float16 cannot represent"
    q_len = torch.tensor(q_lens, dtype=torch.int32)
    kv_len = torch.tensor(ctx, dtype=torch.int32)
    O, L = fa.flash_attention_forward(Q.cuda(), K.cuda(), V.cuda(), q_len.cuda(), bt.cuda(), nblk.cuda(), BS,
                                      kv_len.cuda(), ks, vs)
    torch.cuda.synchronize()
    O_or, L_or = orc.paged_attention(Q.numpy(), Kn, Vn, q_lens, bt.numpy(), nblk.numpy(), BS, ctx, ksn, vsn)
    err = _max_err(O, O_or, q_lens)
    assert err <= tol, f"{pool} case {case}: max |O - oracle| = {err:.3e} > {tol:.0e}"
    Lc = L.float().cpu().numpy()
    for b in range(B):
        np.testing.assert_allclose(Lc[b, :, :q_lens[b]], L_or[b, :, :q_lens[b]], atol=1e-2, rtol=1e-3)


@pytest.mark.parametrize("case", range(len(CASES)))
def test_model_cache_layout_with_per_block_scales(fa, case):
    """INT8 caches allocated as the model does, [NB, H, BS, D] with float32 [NB, H] scales.

    Passed unchanged (as transformer/model.py:156-160 does) and as the
    transposed [NB, BS, H, D] view: the two calls agree bit for bit and match
    the oracle on the model's layout.
    """
    B, Hq, Hkv, D, BS, ctx, q_lens = CASES[case]
    if Hkv == BS:
        pytest.skip("layouts are indistinguishable when heads == block_size")
    gen = torch.Generator().manual_seed(200 + case)
    bt, nblk, NB = _tables(gen, ctx, BS)
    Q = torch.randn(B, Hq, max(q_lens), D, generator=gen)
    Kmodel = torch.randn(NB, Hkv, BS, D, generator=gen)
    Vmodel = torch.randn(NB, Hkv, BS, D, generator=gen)
    # per-(block, head) quantisation in the model's layout (transformer/model.py:105-114)
    kq, ksn = orc.quantize_blocks(Kmodel.numpy().transpose(0, 2, 1, 3))
    vq, vsn = orc.quantize_blocks(Vmodel.numpy().transpose(0, 2, 1, 3))
    kc = torch.from_numpy(np.ascontiguousarray(kq.transpose(0, 2, 1, 3))).cuda()  # [NB, H, BS, D]
    vc = torch.from_numpy(np.ascontiguousarray(vq.transpose(0, 2, 1, 3))).cuda()
    assert kc.shape == (NB, Hkv, BS, D)
    ks, vs = torch.from_numpy(ksn).cuda(), torch.from_numpy(vsn).cuda()
    meta = [torch.tensor(q_lens, dtype=torch.int32).cuda(), bt.cuda(), nblk.cuda(), BS,
            torch.tensor(ctx, dtype=torch.int32).cuda()]
    O1, L1 = fa.flash_attention_forward(Q.cuda(), kc, vc, *meta, ks, vs)
    O2, L2 = fa.flash_attention_forward(Q.cuda(), kc.transpose(1, 2), vc.transpose(1, 2), *meta, ks, vs)
    torch.cuda.synchronize()
    for b in range(B):
        ql = q_lens[b]
        assert torch.equal(O1[b, :, :ql], O2[b, :, :ql]) and torch.equal(L1[b, :, :ql], L2[b, :, :ql])
    O_or, _ = orc.paged_attention(Q.numpy(), kq, vq, q_lens, bt.numpy(), nblk.numpy(), BS, ctx, ksn, vsn)
    err = _max_err(O1, O_or, q_lens)
    assert err <= TOL_I8, f"model layout case {case}: max |O - oracle| = {err:.3e}"


@pytest.mark.parametrize("via", ["forward", "autograd"])
def test_reference_layer_calls(fa, via):
    """The exact arguments the reference's MultiHeadAttention.forward passed over three scheduler steps.

    Fixture ``model_layer_steps.npz`` (tests/golden/make_golden.py) captured
    them from the reference layer driven by its own Scheduler and
    BlockManager: a prefill step, a decode step and a mixed step.  O is
    checked against the oracle and the layer output (W_o applied to the
    unpadded O, transformer/model.py:162-171) against the recorded one.
    """
    g = load_golden("model_layer_steps.npz")
    for s in range(int(g["steps"])):
        a = {k[len(f"s{s}_"):]: v for k, v in g.items() if k.startswith(f"s{s}_")}
        args = (torch.from_numpy(a["Q"]).cuda(), torch.from_numpy(a["K"]).cuda(), torch.from_numpy(a["V"]).cuda(),
                torch.from_numpy(a["q_len"]).cuda(), torch.from_numpy(a["block_table"]).cuda(),
                torch.from_numpy(a["num_blocks"]).cuda(), int(a["block_size"]), torch.from_numpy(a["kv_len"]).cuda(),
                torch.from_numpy(a["k_scale"]).cuda(), torch.from_numpy(a["v_scale"]).cuda())
        assert args[0].dtype == torch.float32 and args[1].dtype == torch.int8 and args[8].dtype == torch.float32
        if via == "forward":
            O, _ = fa.flash_attention_forward(*args)
        else:
            O = fa.FlashAttentionFunction.apply(*args)
        torch.cuda.synchronize()
        err = _max_err(O, a["O_ref"], a["q_len"])
        assert err <= TOL_I8, f"step {s}: max |O - oracle| = {err:.3e}"
        # the layer's tail: unpad, float32, W_o
        T = int(a["length"].sum())
        O_flat = torch.zeros(T, O.shape[1], O.shape[3], dtype=O.dtype, device=O.device)
        for k in range(O.shape[0]):
            st, n = int(a["offset"][k]), int(a["length"][k])
            O_flat[st:st + n] = O[k, :, :n].transpose(0, 1)
        y = torch.nn.functional.linear(O_flat.float().reshape(T, -1), torch.from_numpy(g["W_o"]).cuda(),
                                       torch.from_numpy(g["b_o"]).cuda())
        yerr = float((y.cpu() - torch.from_numpy(a["y"])).abs().max())
        assert yerr <= TOL_I8, f"step {s}: layer output max err {yerr:.3e}"


def test_float32_pool_golden(fa):
    """The reference kernel's CPU decode configuration with its float32 pool, passed as float32."""
    g = load_golden("attn_cfg1_fp32.npz")
    K = torch.from_numpy(g["K"].astype(np.float32)).cuda()
    V = torch.from_numpy(g["V"].astype(np.float32)).cuda()
    Q = torch.from_numpy(g["Q"].astype(np.float32)).cuda()
    O, L = fa.flash_attention_forward(Q, K, V, torch.from_numpy(g["q_len"]).cuda(),
                                      torch.from_numpy(g["block_table"]).cuda(), torch.from_numpy(g["num_blocks"]).cuda(),
                                      int(g["block_size"]), torch.from_numpy(g["kv_len"]).cuda(), None, None)
    torch.cuda.synchronize()
    err = _max_err(O, g["O_ref"].astype(np.float32), g["q_len"])
    assert err <= TOL_F16 + 1e-3, f"max |O - reference kernel| = {err:.3e}"


def test_float32_pool_write_then_attend(fa):
    """write_kv_cache into a float32 pool stores the rows exactly; attention reads them back."""
    from pie_b200 import ops

    gen = torch.Generator().manual_seed(5)
    T, H, D, BS, NB = 40, 2, 128, 16, 6
    k_new = torch.randn(T, H, D, generator=gen)
    v_new = torch.randn(T, H, D, generator=gen)
    bt = torch.tensor([[4, 1, 3]], dtype=torch.int32)
    kc = torch.zeros(NB, BS, H, D, device="cuda")
    vc = torch.zeros_like(kc)
    seq = torch.zeros(T, dtype=torch.int32)
    pos = torch.arange(T, dtype=torch.int32)
    fa.write_kv_cache(k_new.cuda(), v_new.cuda(), bt.cuda(), seq.cuda(), pos.cuda(), kc, vc)
    torch.cuda.synchronize()
    for t in range(T):
        blk, slot = int(bt[0, t // BS]), t % BS
        assert torch.equal(kc[blk, slot].cpu(), k_new[t]) and torch.equal(vc[blk, slot].cpu(), v_new[t])
    q = torch.randn(1, 4, 1, D, generator=gen)
    one = torch.ones(1, dtype=torch.int32, device="cuda")
    O, _ = fa.flash_attention_forward(q.cuda(), kc, vc, one, bt.cuda(), torch.tensor([3], dtype=torch.int32).cuda(),
                                      BS, torch.tensor([T], dtype=torch.int32).cuda(), None, None)
    torch.cuda.synchronize()
    O_or, _ = orc.paged_attention(q.numpy(), kc.cpu().numpy(), vc.cpu().numpy(), [1], bt.numpy(), [3], BS, [T])
    assert _max_err(O, O_or, [1]) <= TOL_F16
    # the split-K decode entry point refuses float32 pools explicitly
    with pytest.raises(Exception, match="fp32|float32|fp16, bf16 or int8"):
        ops.paged_attention(q.cuda(), kc, vc, one, bt.cuda(), torch.tensor([3], dtype=torch.int32).cuda(), BS,
                            torch.tensor([T], dtype=torch.int32).cuda(), mode="decode")
