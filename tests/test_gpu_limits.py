"""Parity at the size limits of the kernels.

* 8192 sequences, the most one decode launch takes, and 8193 and 20000,
  which the decode path serves in launches of at most 8192 sequences that
  share one workspace;
* the decode / prefill switch at exactly 16 packed columns
  (max_q_len * Hq / Hkv = 16 decodes, 20 does not);
* one sequence of 131072 keys (8192 blocks of 16).

Each output is checked against the oracle (on a sample of the sequences where
there are thousands).
"""
import numpy as np
import pytest
import torch

from oracle import paged_attention as orc

pytestmark = pytest.mark.gpu

TOL_F16 = 2e-3


def _check(b, O, L, rows, q_len, tol=TOL_F16):
    """Oracle on the sequences `rows` of batch b (a PagedBatch on the CPU)."""
    sel = np.asarray(rows)
    K = b.K.float().numpy() if b.K.dtype != torch.int8 else b.K.numpy()
    V = b.V.float().numpy() if b.V.dtype != torch.int8 else b.V.numpy()
    O_or, L_or = orc.paged_attention(b.Q[sel].float().numpy(), K, V, np.asarray(q_len)[sel],
                                     b.block_table[sel].numpy(), b.num_blocks[sel].numpy(), b.block_size,
                                     b.kv_len[sel].numpy(), None if b.k_scale is None else b.k_scale.numpy(),
                                     None if b.v_scale is None else b.v_scale.numpy())
    got = O[sel].float().cpu().numpy()
    for i, bi in enumerate(sel):
        n = int(q_len[bi])
        err = np.abs(got[i, :, :n] - O_or[i, :, :n]).max()
        assert err <= tol, f"sequence {bi}: max err {err:.3e}"
        np.testing.assert_allclose(L[bi, :, :n].float().cpu().numpy(), L_or[i, :, :n], atol=1e-2, rtol=1e-3)


@pytest.mark.parametrize("B,kv_dtype", [(8192, torch.float16), (8193, torch.float16), (20000, torch.float16),
                                         (8200, torch.int8)])
def test_most_sequences_per_launch(B, kv_dtype):
    from kernels.flash_attention import flash_attention_forward
    from pie_b200 import ops
    from pie_b200.workloads import make_decode_batch

    gen = np.random.default_rng(B)
    ctx = [int(c) for c in gen.integers(1, 48, size=B)]
    b = make_decode_batch(B, B, 8, 2, 128, 16, ctx, kv_dtype=kv_dtype)
    g = b.to("cuda")
    O, L = flash_attention_forward(g.Q, g.K, g.V, g.q_len, g.block_table, g.num_blocks, 16, g.kv_len, g.k_scale,
                                   g.v_scale)
    torch.cuda.synchronize()
    rows = sorted(set([0, 1, 8191, 8192, B // 2, B - 2, B - 1] + [int(x) for x in gen.integers(0, B, size=120)]))
    rows = [r for r in rows if r < B]
    tol = 2e-2 if kv_dtype == torch.int8 else TOL_F16
    _check(b, O, L, rows, b.q_len.numpy(), tol=tol)
    # the decode entry point itself takes the whole batch (no switch to the prefill kernel)
    O2, L2 = ops.paged_attention(g.Q, g.K, g.V, g.q_len, g.block_table, g.num_blocks, 16, g.kv_len, g.k_scale,
                                 g.v_scale, mode="decode")
    torch.cuda.synchronize()
    assert torch.equal(O, O2) and torch.equal(L, L2)


@pytest.mark.parametrize("qmax", [4, 5])
def test_decode_prefill_switch(qmax):
    """Hq / Hkv = 4: four query rows (16 packed columns) still decode, five go to the prefill kernel."""
    from kernels.flash_attention import flash_attention_forward
    from pie_b200.workloads import make_decode_batch

    ctx = [5, 70, 300, 1000, 2049]
    b = make_decode_batch(60 + qmax, len(ctx), 16, 4, 128, 16, ctx, q_len=qmax, outliers=0.0)
    q_len = [1, 2, qmax, qmax, 3]
    b.q_len = torch.tensor(q_len, dtype=torch.int32)
    g = b.to("cuda")
    O, L = flash_attention_forward(g.Q, g.K, g.V, g.q_len, g.block_table, g.num_blocks, 16, g.kv_len)
    torch.cuda.synchronize()
    _check(b, O, L, range(len(ctx)), q_len)


@pytest.mark.parametrize("kv_dtype", [torch.float16, torch.int8])
def test_one_sequence_of_131072_keys(kv_dtype):
    from kernels.flash_attention import flash_attention_forward
    from pie_b200.workloads import make_decode_batch

    b = make_decode_batch(77, 1, 8, 2, 128, 16, [131072], kv_dtype=kv_dtype, outliers=0.0)
    g = b.to("cuda")
    O, L = flash_attention_forward(g.Q, g.K, g.V, g.q_len, g.block_table, g.num_blocks, 16, g.kv_len, g.k_scale,
                                   g.v_scale)
    torch.cuda.synchronize()
    _check(b, O, L, [0], b.q_len.numpy(), tol=2e-2 if kv_dtype == torch.int8 else TOL_F16)
