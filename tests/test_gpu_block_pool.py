"""GPU: the device-resident block pool against the reference's own scheduler trace.

Bit-exact requirements (integer work): after every scheduling step of
``block_trace.npz`` the device free list and per-sequence block lists equal
the reference BlockManager's, every call's device status equals the
reference's, and the step inputs built on the device (padded block table,
num_blocks_per_seq, positions, token rows) equal what
transformer/model.py:126-152 and core/model_runner.py:66-107 build.
"""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import block_manager as obm
from oracle import paged_attention as orc

pytestmark = pytest.mark.gpu


def _step(g, s):
    return {k[len(f"s{s}_"):]: v for k, v in g.items() if k.startswith(f"s{s}_")}


@pytest.fixture(scope="module")
def bp():
    from pie_b200 import block_pool
    assert torch.cuda.is_available()
    return block_pool


def test_device_pool_replays_the_reference_trace(bp):
    g = load_golden("block_trace.npz")
    NB = int(g["num_blocks"])
    dm = bp.DeviceBlockManager(NB, int(g["block_size"]), max_seqs=64, max_blocks_per_seq=16, device="cuda")
    ops = g["ops"]
    checked = 0
    for s in range(int(g["steps"])):
        want_dev = []
        for _, kind, sid, n, status in ops[ops[:, 0] == s]:
            if kind == 0:
                st = dm.allocate(int(sid), int(n)).status
            else:
                st = dm.release_blocks(int(sid))
            assert st == bp.AllocStatus(int(status)), f"step {s}: host status"
            if status == 0:
                want_dev.append(0)
        dm.flush(keep_results=True)
        if want_dev:
            assert dm.last_results.cpu().tolist() == want_dev, f"step {s}: device statuses"
        a = _step(g, s)
        assert dm.free_list() == a["stack"].tolist(), f"step {s}: free list"
        tab = dm.block_table
        ids = a["table_ids"].tolist()
        off = 0
        assert sorted(tab) == a["table_seq"].tolist()
        for sid, n in zip(a["table_seq"], a["table_len"]):
            assert tab[int(sid)] == ids[off:off + n], f"step {s}: blocks of sequence {sid}"
            off += n
        # the step's attention inputs, built on the device
        seqs = a["sequence_id"].tolist()
        if not seqs:
            continue
        inp = dm.step_inputs(seqs, a["q_len"].tolist(), a["kv_len"].tolist())
        torch.cuda.synchronize()
        assert np.array_equal(inp["block_table"].cpu().numpy(), a["block_table"]), f"step {s}: block table"
        assert inp["num_blocks_per_seq"].cpu().tolist() == a["num_blocks"].tolist()
        assert inp["positions"].cpu().tolist() == a["position_ids"].tolist(), f"step {s}: positions"
        rows = inp["token_seq"].cpu().numpy()
        assert np.array_equal(np.asarray(seqs)[rows], a["pos_seq_id"]), f"step {s}: token rows"
        assert inp["cu_seqlens"].cpu().tolist()[:-1] == a["offset"].tolist()
        checked += 1
    assert int(dm.status.item()) == 0
    assert checked > 40


def test_device_pool_interleaved_allocation(bp):
    """tests/test_block_manager.py:4-37 of the reference on the device pool: statuses, no double allocation."""
    dm = bp.DeviceBlockManager(1000, 20, max_seqs=8, max_blocks_per_seq=512, device="cuda")
    ref = obm.BlockManager(1000, 20)
    seen, owned = set(), {}

    def alloc(seq, n, expect):
        r = dm.allocate(seq, n)
        assert r.status.value == expect == ref.allocate(seq, n)[0]
        if r.status == bp.AllocStatus.SUCCESS:
            dm.flush()
            ids = r.block_ids.cpu().tolist()
            assert ids == ref.block_table[seq][-n:]
            assert not (set(ids) & seen)
            seen.update(ids)
            owned[seq] = ids
        assert dm.num_free_blocks() + len(seen) == 1000

    def release(seq, expect):
        assert dm.release_blocks(seq).value == expect == ref.release_blocks(seq)
        if expect == 0:
            seen.difference_update(owned.pop(seq))
        assert dm.num_free_blocks() + len(seen) == 1000

    alloc(0, 200, 0)
    alloc(1, 130, 0)
    alloc(2, 320, 0)
    release(1, 0)
    alloc(3, 500, 1)
    alloc(3, 300, 0)
    release(6, 2)
    assert dm.free_list() == ref.st


def test_device_pool_raw_statuses(bp):
    """The device reports INSUFFICIENT_SPACE / FAILURE / ROW_FULL / INVALID itself (ops sent straight to the C ABI)."""
    import ctypes

    from pie_b200 import _lib

    dm = bp.DeviceBlockManager(10, 16, max_seqs=4, max_blocks_per_seq=6, device="cuda")
    ops = torch.tensor([[0, 0, 4], [0, 1, 7], [1, 2, 0], [0, 0, 3], [0, 5, 1], [0, 1, 6], [1, 0, 0], [0, 2, 0],
                        [1, 2, 0]], dtype=torch.int32, device="cuda")
    res = torch.full((ops.shape[0],), -9, dtype=torch.int32, device="cuda")
    lib = _lib.load()
    _lib.check("block_pool_apply", lib.block_pool_apply(ctypes.byref(dm._desc), ops.data_ptr(), ops.shape[0],
                                                        res.data_ptr(), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    # alloc 4 (ok), alloc 7 > 6 free (insufficient), release empty slot (failure), alloc 3 -> 7 > row 6 (row full),
    # slot 5 (invalid), alloc 6 (ok: 6 free), release slot 0 (ok), alloc 0 to slot 2 (ok, empty entry), release it
    assert res.cpu().tolist() == [0, 1, 2, 3, 4, 0, 0, 0, 0]
    assert int(dm.free_top.item()) == 4


def test_step_inputs_feed_the_attention_path(bp):
    """One prefill + decode step driven only by device-built inputs: write the new rows, attend, no host sync.

    Uses the corrected decode positions (the new token of a sequence holding
    n tokens sits at n - 1): the oracle attends over exactly the rows written.
    """
    from kernels.flash_attention import flash_attention_varlen, write_kv_cache
    from pie_b200.workloads import empty_head_major_scales

    gen = torch.Generator().manual_seed(9)
    NB, BS, Hq, Hkv, D = 64, 16, 8, 2, 128
    dm = bp.DeviceBlockManager(NB, BS, max_seqs=8, max_blocks_per_seq=16, device="cuda")
    K = torch.zeros(NB, BS, Hkv, D, dtype=torch.int8, device="cuda")
    V = torch.zeros_like(K)
    ks = empty_head_major_scales(NB, BS, Hkv, device="cuda").zero_()
    vs = empty_head_major_scales(NB, BS, Hkv, device="cuda").zero_()
    Kh = np.zeros((NB, BS, Hkv, D), np.int8)
    Vh = np.zeros_like(Kh)
    ksh = np.zeros((NB, BS, Hkv), np.float16)
    vsh = np.zeros_like(ksh)
    lens = {0: 0, 1: 0, 2: 0}
    prompts = {0: 37, 1: 5, 2: 70}
    for step in range(3):
        seqs, ql, kl = [], [], []
        for sid in sorted(lens):
            n_new = prompts[sid] if lens[sid] == 0 else 1
            need = -(-(lens[sid] + n_new) // BS) - dm.blocks_of(sid)
            if need > 0:
                assert dm.allocate(sid, need).status == bp.AllocStatus.SUCCESS
            seqs.append(sid)
            ql.append(n_new)
            kl.append(lens[sid] + n_new)
        inp = dm.step_inputs(seqs, ql, kl)
        T = sum(ql)
        want_pos = [lens[sid] + i for sid, n in zip(seqs, ql) for i in range(n)]
        assert inp["positions"].cpu().tolist() == want_pos
        k_new = torch.randn(T, Hkv, D, generator=gen).half()
        v_new = torch.randn(T, Hkv, D, generator=gen).half()
        q = torch.randn(T, Hq, D, generator=gen).half()
        write_kv_cache(k_new.cuda(), v_new.cuda(), inp["block_table"], inp["token_seq"], inp["positions"], K, V, ks,
                       vs)
        O, _ = flash_attention_varlen(q.cuda(), inp["cu_seqlens"], K, V, inp["block_table"],
                                      inp["num_blocks_per_seq"], BS, inp["kv_len"], ks, vs, max_q_len=max(ql))
        torch.cuda.synchronize()
        bt = inp["block_table"].cpu().numpy()
        orc.write_kv_cache(k_new.float().numpy(), v_new.float().numpy(), bt, inp["token_seq"].cpu().numpy(),
                           inp["positions"].cpu().numpy(), Kh, Vh, ksh, vsh)
        assert np.array_equal(K.cpu().numpy(), Kh) and np.array_equal(ks.cpu().numpy(), ksh)
        cu = [0] + list(np.cumsum(ql))
        for k in range(len(seqs)):
            qk = q[cu[k]:cu[k + 1]].transpose(0, 1).unsqueeze(0).float().numpy()  # [1, Hq, q, D]
            O_or, _ = orc.paged_attention(qk, Kh, Vh, [ql[k]], bt[k:k + 1], [inp["num_blocks_per_seq"][k].item()], BS,
                                          [kl[k]], ksh, vsh)
            got = O[cu[k]:cu[k + 1]].transpose(0, 1).float().cpu().numpy()
            assert np.abs(got - O_or[0]).max() <= 2e-2, f"step {step} seq {k}"
        for sid, n in zip(seqs, ql):
            lens[sid] += n
        if step == 1:
            assert dm.release_blocks(1) == bp.AllocStatus.SUCCESS
            del lens[1]
