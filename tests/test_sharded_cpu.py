"""World-size-2 gloo tests of the KV-head sharded decode host logic (CPU).

Each rank holds only its KV heads' pool and runs the oracle as its local
attention; the all-gather must reassemble exactly the full-head result.
A rank that fails before the collective makes the other rank's collective
end with an error after a short process-group timeout (no hang).
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import PKG, ROOT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_attention(Q, K, V, q_len, bt, nblk, bs, kv_len, ks, vs):
    from oracle import paged_attention as orc

    O, L = orc.paged_attention(Q.float().numpy(), K.numpy(), V.numpy(), q_len.numpy(), bt.numpy(), nblk.numpy(), bs,
                               kv_len.numpy(), None if ks is None else ks.numpy(), None if vs is None else vs.numpy())
    return torch.from_numpy(O).half(), torch.from_numpy(L).half()


def _worker(rank, world, port, result_path, fail_rank, q_len=1):
    import sys

    for p in (ROOT, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    # Rendezvous through a store with a generous wait (spawned ranks import torch at their own pace); the
    # process group's own 10 s limit then bounds the collectives, so a rank that never joins one ends the
    # other ranks' wait quickly.
    store = torch.distributed.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=120))
    torch.distributed.init_process_group("gloo", store=store, rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=10))
    from pie_b200.sharded import KVHeadShardedDecoder
    from pie_b200.workloads import make_decode_batch

    Hq, Hkv, D = 8, 4, 64
    # same full batch everywhere; q_len > 1: prefill / chunked-prefill rows
    b = make_decode_batch(4, 3, Hq, Hkv, D, 16, [40, 17, 100], kv_dtype=torch.int8, q_len=q_len)
    b.q_len = torch.tensor([min(q_len, c) for c in (40, 17, 100)], dtype=torch.int32)
    dec = KVHeadShardedDecoder(Hq, Hkv, D, attention_fn=_oracle_attention)
    lo, hi = dec.kv_lo, dec.kv_hi
    K, V = b.K[:, :, lo:hi].contiguous(), b.V[:, :, lo:hi].contiguous()
    ks, vs = b.k_scale[:, :, lo:hi].contiguous(), b.v_scale[:, :, lo:hi].contiguous()
    try:
        if rank == fail_rank:
            raise RuntimeError("injected failure before the collective")
        O = dec.forward(dec.local_q(b.Q).contiguous(), K, V, b.q_len, b.block_table, b.num_blocks, 16, b.kv_len,
                        ks, vs)
        full, _ = _oracle_attention(b.Q, b.K, b.V, b.q_len, b.block_table, b.num_blocks, 16, b.kv_len, b.k_scale,
                                    b.v_scale)
        ok = torch.equal(O, full)
        msg = "ok" if ok else f"max diff {(O.float() - full.float()).abs().max().item()}"
    except Exception as e:  # noqa: BLE001
        msg = f"error: {type(e).__name__}"
    with open(f"{result_path}.{rank}", "w") as f:
        f.write(msg)
    try:
        torch.distributed.destroy_process_group()
    except Exception:  # noqa: BLE001
        pass


def _run(world, fail_rank, tmp_path, q_len=1):
    ctx = mp.get_context("spawn")
    port = _free_port()
    out = str(tmp_path / "res")
    procs = [ctx.Process(target=_worker, args=(r, world, port, out, fail_rank, q_len)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode is not None, "rank did not exit"
    return [open(f"{out}.{r}").read() for r in range(world)]


def test_head_range_split():
    from pie_b200.sharded import head_range

    assert [head_range(8, 4, r) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        head_range(8, 3, 0)


def test_kv_head_sharded_gather_matches_full(tmp_path):
    res = _run(2, -1, tmp_path)
    assert res == ["ok", "ok"], res


def test_kv_head_sharded_prefill_matches_full(tmp_path):
    """Prefill rows (q_len up to 33, bottom-right causal) through the same sharded layer."""
    res = _run(2, -1, tmp_path, q_len=33)
    assert res == ["ok", "ok"], res


def test_failed_rank_does_not_hang_the_other(tmp_path):
    res = _run(2, 1, tmp_path)
    assert res[1].startswith("error"), res
    assert res[0].startswith("error"), res  # the surviving rank's all_gather fails instead of hanging
