"""GPU: the persistent paired-head prefill kernel under concurrent launches.

Its CTAs take work items from a launch-wide counter kept in device memory
(one slot per launch generation, zeroed by the launch's last CTA).  Launches
in flight at the same time on different streams must not share items, and a
slot must be ready again for the next launch.  Each problem here is run alone
first, then all of them concurrently on their own streams, twice, and every
output row must equal its solo run bit for bit (rows past a sequence's
q_len are left unwritten, as by the reference launcher, and not compared).
"""
import pytest
import torch

from pie_b200.workloads import block_tables

pytestmark = pytest.mark.gpu


def _problem(seed, lens, Hq=8, Hkv=2, D=128, BS=16, dtype=torch.bfloat16):
    gen = torch.Generator().manual_seed(seed)
    bt, nblk, NB = block_tables(gen, lens, BS)
    dev = torch.device("cuda")
    Q = torch.randn(len(lens), Hq, max(lens), D, generator=gen).to(dtype).to(dev)
    K = torch.randn(NB, BS, Hkv, D, generator=gen).to(dtype).to(dev)
    V = torch.randn(NB, BS, Hkv, D, generator=gen).to(dtype).to(dev)
    L = torch.tensor(lens, dtype=torch.int32, device=dev)
    return Q, K, V, L, bt.to(dev), nblk.to(dev), BS


def _same(a, b, lens):
    """Equal on every sequence's valid query rows ([B, H, q, ...] tensors)."""
    return all(torch.equal(a[i, :, :n], b[i, :, :n]) for i, n in enumerate(lens))


def _run(prob):
    from kernels.flash_attention import flash_attention_forward

    Q, K, V, L, bt, nb, BS = prob
    O, lse = flash_attention_forward(Q, K, V, L, bt, nb, BS, L)
    return O, lse


def test_concurrent_prefill_launches_match_solo_runs():
    lens = [[700, 1500, 130], [2048, 64], [999] * 6, [3000]]
    probs = [_problem(1 + i, ln) for i, ln in enumerate(lens)]
    solo = [_run(pr) for pr in probs]
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream() for _ in probs]
    for _ in range(2):
        outs = [None] * len(probs)
        cur = torch.cuda.current_stream()
        for i, (pr, st) in enumerate(zip(probs, streams)):
            st.wait_stream(cur)
            with torch.cuda.stream(st):
                outs[i] = _run(pr)
        for st in streams:
            cur.wait_stream(st)
        torch.cuda.synchronize()
        for i, ((O, lse), (O0, lse0)) in enumerate(zip(outs, solo)):
            assert _same(O, O0, lens[i]), f"problem {i}: output differs from its solo run"
            assert _same(lse, lse0, lens[i]), f"problem {i}: LSE differs from its solo run"


def test_back_to_back_launches_reuse_the_work_counter():
    """Hundreds of launches in a row (the counter slots wrap around) still cover every item."""
    lens = [513, 257, 1025]
    prob = _problem(5, lens)
    O0, _ = _run(prob)
    torch.cuda.synchronize()
    for _ in range(300):
        O, _ = _run(prob)
    torch.cuda.synchronize()
    assert _same(O, O0, lens)
