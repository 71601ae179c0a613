"""GPU: the captured decode step (pie_b200.decode_step) against eager calls and the oracle.

Sequences are prefilled eagerly through the device block pool, then decoded
step by step by graph replays while the batch changes (a sequence leaves, a
new one joins, fewer sequences than graph rows).  Each step's output must
equal the eager attention call on the same cache and match the oracle on a
host mirror of the cache; the new rows land at position len - 1 (the
corrected decode position).
"""
import numpy as np
import pytest
import torch

from oracle import paged_attention as orc

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kv_dtype", [torch.float16, torch.int8])
def test_decode_step_graph(kv_dtype):
    from kernels.flash_attention import flash_attention_forward, write_kv_cache
    from pie_b200.block_pool import DeviceBlockManager
    from pie_b200.decode_step import DecodeStepGraph
    from pie_b200.workloads import empty_head_major_scales

    gen = torch.Generator().manual_seed(17)
    dev = torch.device("cuda")
    NB, BS, Hq, Hkv, D = 64, 16, 8, 2, 128
    pool = DeviceBlockManager(NB, BS, max_seqs=8, max_blocks_per_seq=8, device=dev)
    K = torch.zeros(NB, BS, Hkv, D, dtype=kv_dtype, device=dev)
    V = torch.zeros_like(K)
    ks = vs = None
    if kv_dtype == torch.int8:
        ks = empty_head_major_scales(NB, BS, Hkv, device=dev).zero_()
        vs = empty_head_major_scales(NB, BS, Hkv, device=dev).zero_()
    lens = {}

    def prefill(sid, n):
        assert pool.allocate(sid, -(-n // BS)).status.value == 0
        inp = pool.step_inputs([sid], [n], [n])
        k = torch.randn(n, Hkv, D, generator=gen).half().to(dev)
        v = torch.randn(n, Hkv, D, generator=gen).half().to(dev)
        write_kv_cache(k, v, inp["block_table"], inp["token_seq"], inp["positions"], K, V, ks, vs)
        lens[sid] = n

    for sid, n in ((0, 40), (1, 15), (2, 77)):
        prefill(sid, n)
    g = DecodeStepGraph(pool, K, V, ks, vs, Hq, max_seqs=4)
    tol = 2e-2 if kv_dtype == torch.int8 else 2e-3
    for step in range(6):
        if step == 3:
            assert pool.release_blocks(1).value == 0
            del lens[1]
            prefill(5, 33)
        ids = sorted(lens)
        for sid in ids:
            lens[sid] += 1
        n = len(ids)
        q = torch.randn(n, Hq, D, generator=gen).half().to(dev)
        kn = torch.randn(n, Hkv, D, generator=gen).half().to(dev)
        vn = torch.randn(n, Hkv, D, generator=gen).half().to(dev)
        O = g.step(ids, [lens[s] for s in ids], q, kn, vn).clone()
        torch.cuda.synchronize()
        # eager attention over the same cache, block tables read back from the pool
        tab = pool.block_table
        W = max(len(tab[s]) for s in ids)
        bt = torch.tensor([tab[s] + [0] * (W - len(tab[s])) for s in ids], dtype=torch.int32)
        nb = torch.tensor([len(tab[s]) for s in ids], dtype=torch.int32)
        kl = torch.tensor([lens[s] for s in ids], dtype=torch.int32)
        one = torch.ones(n, dtype=torch.int32)
        Oe, _ = flash_attention_forward(q.unsqueeze(2), K, V, one.to(dev), bt.to(dev), nb.to(dev), BS, kl.to(dev), ks,
                                        vs)
        torch.cuda.synchronize()
        assert torch.equal(O, Oe[:, :, 0]), f"step {step}: graph replay differs from the eager call"
        # the new rows sit at position len - 1
        for i, s in enumerate(ids):
            p = lens[s] - 1
            blk, slot = tab[s][p // BS], p % BS
            if kv_dtype == torch.int8:
                q8 = torch.round(kn[i].float() / (kn[i].float().abs().amax(-1, keepdim=True) / 127)).clamp(-127, 127)
                assert torch.equal(K[blk, slot].float(), q8), f"step {step}: K row of sequence {s}"
            else:
                assert torch.equal(K[blk, slot], kn[i]), f"step {step}: K row of sequence {s}"
        O_or, _ = orc.paged_attention(q.unsqueeze(2).float().cpu().numpy(), K.cpu().numpy(), V.cpu().numpy(),
                                      one.numpy(), bt.numpy(), nb.numpy(), BS, kl.numpy(),
                                      None if ks is None else ks.cpu().numpy(), None if vs is None else vs.cpu().numpy())
        err = float(np.abs(O.float().cpu().numpy() - O_or[:, :, 0]).max())
        assert err <= tol, f"step {step}: max |O - oracle| = {err:.3e}"
    g.check()
