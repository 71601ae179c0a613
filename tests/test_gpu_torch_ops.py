"""GPU: the registered torch ops (torch.ops.pie_b200.*) against the ctypes C-ABI path.

Both paths fill the same C structs and launch the same kernels, so outputs
must agree bit for bit; library errors surface as RuntimeError through
TORCH_CHECK.  (The other GPU tests exercise the torch-op path, the default
backend of pie_b200.ops, against the oracle.)
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture
def ops_mod():
    from pie_b200 import ops
    assert torch.cuda.is_available()
    return ops


def _both(ops_mod, fn):
    saved = ops_mod.BACKEND
    try:
        ops_mod.BACKEND = "torch"
        a = fn()
        ops_mod.BACKEND = "ctypes"
        b = fn()
    finally:
        ops_mod.BACKEND = saved
    torch.cuda.synchronize()
    return a, b


@pytest.mark.parametrize("kv", [torch.float16, torch.bfloat16, torch.int8])
@pytest.mark.parametrize("q_len", [1, 3, 200])
def test_paged_attention_paths_agree(ops_mod, kv, q_len):
    from pie_b200.workloads import make_decode_batch

    ctx = [300, 17, 1000, 256]
    b = make_decode_batch(3, len(ctx), 8, 2, 128, 16, ctx, kv_dtype=kv, q_dtype=torch.bfloat16 if kv ==
                          torch.bfloat16 else torch.float16, q_len=q_len)
    b.q_len = torch.tensor([min(q_len, c) for c in ctx], dtype=torch.int32)
    g = b.to("cuda")
    (O1, L1), (O2, L2) = _both(ops_mod, lambda: ops_mod.paged_attention(
        g.Q, g.K, g.V, g.q_len, g.block_table, g.num_blocks, 16, g.kv_len, g.k_scale, g.v_scale))
    for i, n in enumerate(b.q_len.tolist()):
        assert torch.equal(O1[i, :, :n], O2[i, :, :n]) and torch.equal(L1[i, :, :n], L2[i, :, :n])


def test_varlen_and_write_paths_agree(ops_mod):
    from pie_b200.workloads import empty_head_major_scales

    gen = torch.Generator().manual_seed(4)
    T, Hkv, D, BS, NB = 90, 2, 128, 16, 12
    k_new = torch.randn(T, Hkv, D, generator=gen).half().cuda()
    v_new = torch.randn(T, Hkv, D, generator=gen).half().cuda()
    bt = torch.tensor([[3, 7, 1, 0], [9, 4, 11, 2]], dtype=torch.int32, device="cuda")
    seq = torch.tensor([0] * 50 + [1] * 40, dtype=torch.int32, device="cuda")
    pos = torch.cat([torch.arange(50), torch.arange(40)]).to(torch.int32).cuda()
    pools = []
    for _ in range(2):
        K = torch.zeros(NB, BS, Hkv, D, dtype=torch.int8, device="cuda")
        V = torch.zeros_like(K)
        ks = empty_head_major_scales(NB, BS, Hkv, device="cuda").zero_()
        vs = empty_head_major_scales(NB, BS, Hkv, device="cuda").zero_()
        pools.append((K, V, ks, vs))
    it = iter(pools)

    def write():
        K, V, ks, vs = next(it)
        ops_mod.write_kv(k_new, v_new, bt, seq, pos, K, V, ks, vs)
        return K, V, ks, vs

    a, b = _both(ops_mod, write)
    assert all(torch.equal(x, y) for x, y in zip(a, b))
    K, V, ks, vs = a
    q = torch.randn(T, 8, D, generator=gen).half().cuda()
    cu = torch.tensor([0, 50, 90], dtype=torch.int32, device="cuda")
    nb = torch.tensor([4, 3], dtype=torch.int32, device="cuda")
    kl = torch.tensor([50, 40], dtype=torch.int32, device="cuda")
    (O1, L1), (O2, L2) = _both(ops_mod, lambda: ops_mod.paged_attention_varlen(q, cu, K, V, bt, nb, BS, kl, ks, vs,
                                                                               max_q_len=50))
    assert torch.equal(O1, O2) and torch.equal(L1, L2)


def test_library_errors_raise_through_torch_check(ops_mod):
    """A problem only the C ABI rejects (head_dim 96 is not compiled) raises RuntimeError with its message."""
    tops = __import__("pie_b200._torch_ext", fromlist=["ops"]).ops()
    Q = torch.zeros(1, 2, 1, 96, dtype=torch.float16, device="cuda")
    K = torch.zeros(2, 16, 2, 96, dtype=torch.float16, device="cuda")
    one = torch.ones(1, dtype=torch.int32, device="cuda")
    bt = torch.zeros(1, 1, dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError, match="head_dim 96"):
        tops.paged_attention(Q, K, K, one, bt, one, one, None, None, False, 0.0, 0, None)


def test_registered_op_replays_in_a_cuda_graph(ops_mod):
    """The functional op allocates its outputs from the graph's pool; replays equal eager calls."""
    from pie_b200.workloads import make_decode_batch

    b = make_decode_batch(8, 4, 8, 2, 128, 16, [100, 600, 31, 2000])
    g = b.to("cuda")
    tops = __import__("pie_b200._torch_ext", fromlist=["ops"]).ops()
    args = (g.Q, g.K, g.V, g.q_len, g.block_table, g.num_blocks, g.kv_len, None, None, False, 0.0, 0, None)
    O_ref, L_ref = tops.paged_attention(*args)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        tops.paged_attention(*args)  # warm the workspace outside the capture
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        O_g, L_g = tops.paged_attention(*args)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(O_g, O_ref) and torch.equal(L_g, L_ref)
