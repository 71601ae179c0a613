"""Block bookkeeping on the CPU: the oracle and the host ledger against the reference's own trace.

``block_trace.npz`` records the reference's Scheduler and BlockManager
(core/scheduler.py, core/block_manager.py) over a seeded request trace: every
allocate / release call with its status, and after each scheduling step the
free list, the per-sequence block lists, the step metadata
(core/model_runner.py:66-107) and the padded block table
(transformer/model.py:126-152).
"""
import numpy as np

from conftest import load_golden
from oracle import block_manager as obm


def _step(g, s):
    return {k[len(f"s{s}_"):]: v for k, v in g.items() if k.startswith(f"s{s}_")}


def test_oracle_replays_the_reference_trace():
    g = load_golden("block_trace.npz")
    bm = obm.BlockManager(int(g["num_blocks"]), int(g["block_size"]))
    ops = g["ops"]
    for s in range(int(g["steps"])):
        for _, kind, sid, n, status in ops[ops[:, 0] == s]:
            got = bm.allocate(int(sid), int(n))[0] if kind == 0 else bm.release_blocks(int(sid))
            assert got == status, f"step {s}: op ({kind}, {sid}, {n}) gave {got}, reference {status}"
        a = _step(g, s)
        assert bm.st == a["stack"].tolist(), f"step {s}: free list"
        ids = a["table_ids"].tolist()
        off = 0
        assert sorted(bm.block_table) == a["table_seq"].tolist()
        for sid, n in zip(a["table_seq"], a["table_len"]):
            assert bm.block_table[int(sid)] == ids[off:off + n]
            off += n


def test_oracle_step_metadata_and_padded_table():
    g = load_golden("block_trace.npz")
    bm = obm.BlockManager(int(g["num_blocks"]), int(g["block_size"]))
    ops = g["ops"]
    seen_decode = seen_prefill = 0
    for s in range(int(g["steps"])):
        for _, kind, sid, n, _st in ops[ops[:, 0] == s]:
            if kind == 0:
                bm.allocate(int(sid), int(n))
            else:
                bm.release_blocks(int(sid))
        a = _step(g, s)
        info = a["seq_info"]
        pre = [tuple(int(x) for x in r[:3]) for r in info if r[3] == 1]
        dec = [tuple(int(x) for x in r[:3]) for r in info if r[3] == 0]
        seen_prefill += len(pre)
        seen_decode += len(dec)
        md = obm.step_metadata(pre, dec)
        for k in ("sequence_id", "q_len", "offset", "position_ids", "pos_seq_id", "kv_len"):
            assert md[k] == a[k].tolist(), f"step {s}: {k}"
        rows, nblk = obm.padded_block_table(bm.block_table, md["sequence_id"])
        assert nblk == a["num_blocks"].tolist()
        assert np.array_equal(np.asarray(rows, np.int32).reshape(a["block_table"].shape), a["block_table"])
        # the single rule the device builder uses: position = kv_len - q_len + i
        pos = [kl - ql + i for ql, kl in zip(md["q_len"], md["kv_len"]) for i in range(ql)]
        assert pos == md["position_ids"]
    assert seen_prefill > 10 and seen_decode > 100


def test_fixed_decode_positions():
    """fixed_positions: the decode token sits at len(token_ids) - 1 and attends to len(token_ids) keys."""
    md = obm.step_metadata([(0, 5, 5)], [(1, 4, 9)], fixed_positions=True)
    assert md["position_ids"] == [0, 1, 2, 3, 4, 8]
    assert md["kv_len"] == [5, 9]
    md = obm.step_metadata([(0, 5, 5)], [(1, 4, 9)])
    assert md["position_ids"][-1] == 9 and md["kv_len"][-1] == 10  # core/model_runner.py:96-97


def test_oracle_interleaved_allocation():
    """tests/test_block_manager.py:4-37 of the reference, restated on the oracle."""
    bm = obm.BlockManager(1000, 20)
    seen, owned = set(), {}

    def alloc(seq, n, expect):
        st, ids = bm.allocate(seq, n)
        assert st == expect
        if st == obm.SUCCESS:
            assert not (set(ids) & seen)
            seen.update(ids)
            owned[seq] = ids
        assert bm.num_free_blocks() + len(seen) == bm.num_blocks

    def release(seq, expect):
        assert bm.release_blocks(seq) == expect
        if expect == obm.SUCCESS:
            seen.difference_update(owned.pop(seq))
        assert bm.num_free_blocks() + len(seen) == bm.num_blocks

    alloc(0, 200, obm.SUCCESS)
    alloc(1, 130, obm.SUCCESS)
    alloc(2, 320, obm.SUCCESS)
    release(1, obm.SUCCESS)
    alloc(3, 500, obm.INSUFFICIENT_SPACE)
    alloc(3, 300, obm.SUCCESS)
    release(6, obm.FAILURE)


def test_host_ledger_matches_the_reference_statuses():
    """The host half of the device pool decides every call of the trace as the reference did."""
    from pie_b200.block_pool import AllocStatus, BlockLedger

    g = load_golden("block_trace.npz")
    led = BlockLedger(int(g["num_blocks"]), max_seqs=64, max_blocks_per_seq=16)
    ref = obm.BlockManager(int(g["num_blocks"]), int(g["block_size"]))
    n_ops = 0
    for _, kind, sid, n, status in g["ops"]:
        if kind == 0:
            st = led.allocate(int(sid), int(n))[0]
            ref.allocate(int(sid), int(n))
        else:
            st = led.release(int(sid))
            ref.release_blocks(int(sid))
        assert st == AllocStatus(int(status))
        assert led.free == ref.num_free_blocks()
        assert {k: v for k, v in led.blocks.items()} == {k: len(v) for k, v in ref.block_table.items()}
        n_ops += len(led.take_ops())
    assert n_ops == int((g["ops"][:, 4] == 0).sum())  # only successful calls reach the device
