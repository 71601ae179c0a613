"""Fused head-output exchange (stores into peer buffers) against the NCCL all-gather.

Two ranks on two GPUs of one box, each holding half of the KV heads of a
long-context INT8 pool.  Three decode steps with different queries (the peer
path alternates between its two output buffers) must give, on every rank, the
same bytes as the NCCL all-gather path.  Skipped where fewer than two GPUs are
visible (the single-GPU runs of this suite).
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port):
    import datetime
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "paged-inference-engine_b200"))
    import torch.distributed as dist
    from pie_b200.sharded import KVHeadShardedDecoder, build_rank_pool

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        Bn, Hq, Hkv, D, BS = 16, 16, 4, 128, 16
        ctx = [300 + 97 * i for i in range(Bn)]
        K, V, ks, vs, bt, nblk, NB = build_rank_pool(ctx, Hkv // world, D, BS, 500 + rank, dev)
        ql = torch.ones(Bn, dtype=torch.int32, device=dev)
        kl = torch.tensor(ctx, dtype=torch.int32, device=dev)
        ref = KVHeadShardedDecoder(Hq, Hkv, D)
        peer = KVHeadShardedDecoder(Hq, Hkv, D, exchange="peer")
        for step in range(3):
            Qf = torch.randn(Bn, Hq, 1, D, generator=torch.Generator().manual_seed(70 + step)).half().to(dev)
            Ql = ref.local_q(Qf).contiguous()
            want = ref.forward(Ql, K, V, ql, bt, nblk, BS, kl, ks, vs).clone()
            got = peer.forward(Ql, K, V, ql, bt, nblk, BS, kl, ks, vs).clone()
            torch.cuda.synchronize()
            assert torch.equal(got, want), f"rank {rank} step {step}: max diff {(got.float() - want.float()).abs().max()}"
        peer.close()
        dist.barrier()
    finally:
        torch.cuda.synchronize()
        dist.destroy_process_group()


def _rank_prefill(rank, world, port):
    import datetime
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "paged-inference-engine_b200"))
    import torch.distributed as dist
    from kernels.flash_attention import flash_attention_forward
    from pie_b200.sharded import KVHeadShardedAttention
    from pie_b200.workloads import make_decode_batch

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        Hq, Hkv, D = 16, 4, 128
        ctx = [700, 1300, 257]
        b = make_decode_batch(31, len(ctx), Hq, Hkv, D, 16, ctx, q_len=300)  # the same batch on every rank
        b.q_len = torch.tensor([300, 300, 257], dtype=torch.int32)
        g = b.to(dev)
        sh = KVHeadShardedAttention(Hq, Hkv, D)
        lo, hi = sh.kv_lo, sh.kv_hi
        K, V = g.K[:, :, lo:hi].contiguous(), g.V[:, :, lo:hi].contiguous()
        got = sh.forward(sh.local_q(g.Q).contiguous(), K, V, g.q_len, g.block_table, g.num_blocks, 16, g.kv_len)
        want, _ = flash_attention_forward(g.Q, g.K, g.V, g.q_len, g.block_table, g.num_blocks, 16, g.kv_len)
        torch.cuda.synchronize()
        for i, n in enumerate(b.q_len.tolist()):
            assert torch.equal(got[i, :, :n], want[i, :, :n]), f"rank {rank} sequence {i}"
        dist.barrier()
    finally:
        torch.cuda.synchronize()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs of one box")
def test_kv_head_sharded_prefill_matches_one_gpu():
    """Prefill sharded over two GPUs by KV head equals the one-GPU call bit for bit."""
    mp.spawn(_rank_prefill, args=(2, _free_port()), nprocs=2, join=True)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs of one box")
def test_peer_exchange_matches_all_gather():
    mp.spawn(_rank, args=(2, _free_port()), nprocs=2, join=True)


def _barrier(flags_local, flag_ptrs, n, rank, epoch, status):
    import ctypes
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "paged-inference-engine_b200"))
    from pie_b200 import _lib

    lib = _lib.load()
    peers = (ctypes.c_void_p * n)(*flag_ptrs)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check("paged_attn_peer_barrier",
               lib.paged_attn_peer_barrier(flags_local.data_ptr(), peers, n, rank, epoch, status.data_ptr(), stream))


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_peer_barrier_gives_up_on_a_silent_peer():
    """One GPU, two ranks' worth of flags: peer 1's slot is a local array nobody posts to.

    The bounded wait must run out, set the peer-timeout status bit and return
    (the context stays usable); rank 0's own post still lands in both arrays.
    """
    import time

    from pie_b200 import _lib

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    local = torch.zeros(64, dtype=torch.int32, device=dev)
    silent = torch.zeros(64, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _barrier(local, [local.data_ptr(), silent.data_ptr()], 2, 0, 1, status)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert int(status.item()) & _lib.PA_STATUS_PEER_TIMEOUT, "the wait on the silent peer did not report a timeout"
    assert dt < 20.0, f"bounded wait took {dt:.1f} s"
    assert int(local[0].item()) == 1 and int(silent[0].item()) == 1, "rank 0 did not post its epoch"
    # the context is still usable
    x = torch.arange(10, device=dev).sum()
    assert int(x.item()) == 45


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_peer_barrier_accepts_a_peer_one_epoch_ahead():
    """A peer that already passed this barrier and posted the next epoch ends the wait at once."""
    from pie_b200 import _lib

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    local = torch.zeros(64, dtype=torch.int32, device=dev)
    peer = torch.zeros(64, dtype=torch.int32, device=dev)
    local[1] = 6  # peer 1 has posted epoch 6 into this rank's slot 1
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    _barrier(local, [local.data_ptr(), peer.data_ptr()], 2, 0, 5, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert int(local[0].item()) == 5 and int(peer[0].item()) == 5
    assert int(status.item()) & _lib.PA_STATUS_PEER_TIMEOUT == 0
