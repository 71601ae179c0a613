"""Generate the golden fixtures in tests/golden/ from the reference itself.

Runs in the build container only (it needs the reference checkout at
/root/reference, read-only); the fixtures it writes are committed and the GPU
tests read those, never the reference.

* ``quant_reference.npz``   -- the reference's own ``quantize`` function
  (tests/pre_quantize_test.py:3-12) on the seed-0 inputs of that script and
  applied row by row to a seeded [T, H, D] tensor.
* ``attn_*.npz``            -- the reference's own Triton kernel
  ``flash_attention_kernel`` (kernels/flash_attention.py:19-136) executed by
  the Triton interpreter (TRITON_INTERPRET=1) on CPU, called through ``.fn``
  with the launcher's argument list and stride convention (:155-170).

Decode and chunked-prefill cases use the "last rows" arrangement: the q_len
new queries are placed in rows kv_len-q_len .. kv_len-1 of a zero-padded Q and
q_len_per_seq is set to kv_len, so the reference's top-left mask (:97) gives
each of them exactly the keys a bottom-right aligned mask would.  GQA cases
expand the KV heads with repeat_interleave because the reference kernel has no
GQA.  INT8 per-token cases feed the reference kernel the dequantised pool
(int8 * scale, float32) with unit scales, which is the arithmetic of its
dequantise step (:83-84).

* ``model_layer_steps.npz`` -- three steps of the reference's own
  ``MultiHeadAttention.forward`` (transformer/model.py:69-173) driven by its
  own Scheduler and BlockManager (core/scheduler.py, core/block_manager.py)
  with the step metadata built as core/model_runner.py:66-107 builds it.  The
  layer's call of ``FlashAttentionFunction.apply`` is captured (its exact
  arguments: float32 Q, the model's [num_blocks, heads, block_size, d_k] INT8
  pools with float32 per-block scales) and answered by the oracle reading the
  pools in the model's own layout (bottom-right mask); the layer output after
  W_o is recorded too.

Usage:  python tests/golden/make_golden.py [--ref PATH] [case ...]
        (PATH defaults to $PIE_REFERENCE_ROOT; with no case every fixture is
        regenerated)
"""
from __future__ import annotations

import importlib.util
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

def _ref_root() -> str:
    if "--ref" in sys.argv:
        i = sys.argv.index("--ref")
        root = sys.argv[i + 1]
        del sys.argv[i:i + 2]
        return root
    root = os.environ.get("PIE_REFERENCE_ROOT")
    if not root:
        sys.exit("make_golden.py: pass --ref PATH or set PIE_REFERENCE_ROOT to the reference checkout")
    return root


REF = os.path.abspath(_ref_root())
OUT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REF)
sys.path.insert(0, os.path.dirname(os.path.dirname(OUT)))

import kernels.flash_attention as ref_fa  # noqa: E402  (the reference module)
from oracle import paged_attention as orc  # noqa: E402

assert ref_fa.__file__.startswith(REF), ref_fa.__file__


def _load_ref_quantize():
    spec = importlib.util.spec_from_file_location("ref_pre_quantize", os.path.join(REF, "tests", "pre_quantize_test.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.quantize


def run_ref_kernel(Q, K, V, q_len, block_table, num_blocks, block_size, kv_len, k_scale, v_scale):
    """flash_attention_forward's launch (kernels/flash_attention.py:142-170) without the CUDA assert."""
    B, H, maxq, D = Q.shape
    # The reference kernel dots the Q tile with the float32 dequantised K tile
    # (kernels/flash_attention.py:83,88); tl.dot needs equal operand dtypes, so
    # Q must be float32 (as transformer/model.py passes it).  fp16 inputs are
    # widened exactly.
    Q = Q.float()
    O = torch.zeros(B, H, maxq, D, dtype=torch.float16)
    L = torch.zeros(B, H, maxq, dtype=torch.float16)
    BLOCK_M = 32
    grid = (B, H, -(-int(q_len.max()) // BLOCK_M))
    ref_fa.flash_attention_kernel.fn[grid](
        Q, K, V, O, L,
        Q.stride(0), Q.stride(1), Q.stride(2), Q.stride(3),
        K.stride(0), K.stride(2), K.stride(1), K.stride(3),
        V.stride(0), V.stride(2), V.stride(1), V.stride(3),
        O.stride(0), O.stride(1), O.stride(2), O.stride(3),
        L.stride(0), L.stride(1), L.stride(2),
        block_table, num_blocks,
        q_len,
        block_table.stride(0), block_table.stride(1),
        kv_len,
        k_scale, v_scale,
        k_scale.stride(0), k_scale.stride(1),
        v_scale.stride(0), v_scale.stride(1),
        block_size, D, BLOCK_M=BLOCK_M)
    return O, L


def last_rows_ref(Qnew, K, V, q_len, block_table, num_blocks, block_size, kv_len, k_scale, v_scale):
    """Bottom-right aligned attention of Qnew [B, H, maxq_new, D] via the reference kernel."""
    B, H, mq, D = Qnew.shape
    maxkv = int(kv_len.max())
    Qpad = torch.zeros(B, H, maxkv, D, dtype=Qnew.dtype)
    for b in range(B):
        ql, kl = int(q_len[b]), int(kv_len[b])
        Qpad[b, :, kl - ql:kl] = Qnew[b, :, :ql]
    O, L = run_ref_kernel(Qpad, K, V, kv_len.clone(), block_table, num_blocks, block_size, kv_len, k_scale, v_scale)
    Oo = torch.zeros(B, H, mq, D, dtype=torch.float16)
    Lo = torch.zeros(B, H, mq, dtype=torch.float16)
    for b in range(B):
        ql, kl = int(q_len[b]), int(kv_len[b])
        Oo[b, :, :ql] = O[b, :, kl - ql:kl]
        Lo[b, :, :ql] = L[b, :, kl - ql:kl]
    return Oo, Lo


def seeded_tables(gen, B, ctx, block_size, pool_blocks):
    nblk = [-(-c // block_size) for c in ctx]
    perm = torch.randperm(pool_blocks, generator=gen)
    bt = torch.zeros(B, max(nblk), dtype=torch.int32)
    cur = 0
    for b in range(B):
        bt[b, :nblk[b]] = perm[cur:cur + nblk[b]].to(torch.int32)
        cur += nblk[b]
    return bt, torch.tensor(nblk, dtype=torch.int32)


def case_reference_test():
    """tests/test_flash_attention.py:6-96 inputs (seed 0, generated on CPU), fixed call (unit scales)."""
    torch.manual_seed(0)
    B, H, D, BS = 3, 4, 64, 16
    kv_len = torch.tensor([20, 35, 16], dtype=torch.int32)
    q_len = kv_len.clone()
    maxq = int(q_len.max())
    nb_needed = sum(-(-int(l) // BS) for l in kv_len)
    nb_total = nb_needed + 5
    Kp = torch.randn(nb_total, BS, H, D, dtype=torch.float16)
    Vp = torch.randn(nb_total, BS, H, D, dtype=torch.float16)
    ids = torch.randperm(nb_total)[:nb_needed]
    bt = torch.zeros(B, -(-int(kv_len.max()) // BS), dtype=torch.int32)
    cur = 0
    assign = []
    for i in range(B):
        n = -(-int(kv_len[i]) // BS)
        bt[i, :n] = ids[cur:cur + n].to(torch.int32)
        assign.append(ids[cur:cur + n])
        cur += n
    nblk = torch.tensor([-(-int(l) // BS) for l in kv_len], dtype=torch.int32)
    Q = torch.randn(B, H, maxq, D, dtype=torch.float16)
    ones = torch.ones(nb_total, H, dtype=torch.float32)
    O, L = run_ref_kernel(Q, Kp, Vp, q_len, bt, nblk, BS, kv_len, ones, ones)
    # the test's own comparator: gathered SDPA (tests/test_flash_attention.py:67-83)
    O_sdpa = torch.zeros(B, H, maxq, D, dtype=torch.float32)
    for i in range(B):
        ql, kl = int(q_len[i]), int(kv_len[i])
        Ks = Kp[assign[i]].reshape(-1, H, D)[:kl].permute(1, 0, 2).unsqueeze(0).float()
        Vs = Vp[assign[i]].reshape(-1, H, D)[:kl].permute(1, 0, 2).unsqueeze(0).float()
        O_sdpa[i, :, :ql] = torch.nn.functional.scaled_dot_product_attention(
            Q[i:i + 1, :, :ql].float(), Ks, Vs, is_causal=True)[0]
    for i in range(B):
        ql = int(q_len[i])
        assert torch.allclose(O[i, :, :ql].float(), O_sdpa[i, :, :ql], atol=1e-2, rtol=1e-3)
    np.savez_compressed(os.path.join(OUT, "attn_reference_test.npz"), Q=Q.numpy(), K=Kp.numpy(), V=Vp.numpy(),
                        block_table=bt.numpy(), num_blocks=nblk.numpy(), q_len=q_len.numpy(),
                        kv_len=kv_len.numpy(), block_size=BS, O_ref=O.numpy(), L_ref=L.numpy(),
                        O_sdpa=O_sdpa.numpy())
    print("attn_reference_test", O.float().abs().max().item())


def case_cfg1(variant):
    """The CPU decode shape: B=4, ctx [17,64,100,128], H=8, D=64, BS=16, 64-block pool."""
    gen = torch.Generator().manual_seed(1)
    B, H, D, BS, NB = 4, 8, 64, 16, 64
    ctx = [17, 64, 100, 128]
    bt, nblk = seeded_tables(gen, B, ctx, BS, NB)
    kv_len = torch.tensor(ctx, dtype=torch.int32)
    # values stored in fp16 so the fixture is half the size; the reference
    # computes on the float32 pool made from them.
    K16 = torch.randn(NB, BS, H, D, generator=gen).to(torch.float16)
    V16 = torch.randn(NB, BS, H, D, generator=gen).to(torch.float16)
    Q16 = torch.randn(B, H, 1, D, generator=gen).to(torch.float16)
    q_len = torch.ones(B, dtype=torch.int32)
    extra = {}
    if variant == "fp32":
        Kr, Vr = K16.float(), V16.float()
        ks = vs = torch.ones(NB, H, dtype=torch.float32)
    elif variant == "int8_block":
        kq, ksc = orc.quantize_blocks(K16.float().numpy())
        vq, vsc = orc.quantize_blocks(V16.float().numpy())
        Kr, Vr = torch.from_numpy(kq), torch.from_numpy(vq)
        ks, vs = torch.from_numpy(ksc), torch.from_numpy(vsc)
        extra = dict(K_i8=kq, V_i8=vq, k_scale=ksc, v_scale=vsc)
    elif variant == "int8_token":
        kq, ksc = orc.quantize_rows(K16.float().numpy())  # [NB,BS,H,D], [NB,BS,H]
        vq, vsc = orc.quantize_rows(V16.float().numpy())
        ksc16, vsc16 = ksc.astype(np.float16), vsc.astype(np.float16)
        Kr = torch.from_numpy(kq.astype(np.float32) * ksc16.astype(np.float32)[..., None])
        Vr = torch.from_numpy(vq.astype(np.float32) * vsc16.astype(np.float32)[..., None])
        ks = vs = torch.ones(NB, H, dtype=torch.float32)
        extra = dict(K_i8=kq, V_i8=vq, k_scale=ksc16, v_scale=vsc16)
    else:
        raise ValueError(variant)
    O, L = last_rows_ref(Q16, Kr, Vr, q_len, bt, nblk, BS, kv_len, ks, vs)
    pools = dict(K=K16.numpy(), V=V16.numpy()) if not extra else {}
    np.savez_compressed(os.path.join(OUT, f"attn_cfg1_{variant}.npz"), Q=Q16.numpy(), **pools,
                        block_table=bt.numpy(), num_blocks=nblk.numpy(), q_len=q_len.numpy(), kv_len=kv_len.numpy(),
                        block_size=BS, O_ref=O.numpy(), L_ref=L.numpy(), **extra)
    print(f"attn_cfg1_{variant}", O.float().abs().max().item())


def case_gqa(name, H_q, H_kv, D, BS, ctx, q_lens, int8, seed):
    """GQA decode / chunked prefill (bottom-right), fp16 or per-token INT8."""
    gen = torch.Generator().manual_seed(seed)
    B = len(ctx)
    nblk_l = [-(-c // BS) for c in ctx]
    NB = sum(nblk_l) + 3
    bt, nblk = seeded_tables(gen, B, ctx, BS, NB)
    kv_len = torch.tensor(ctx, dtype=torch.int32)
    q_len = torch.tensor(q_lens, dtype=torch.int32)
    K16 = torch.randn(NB, BS, H_kv, D, generator=gen).to(torch.float16)
    V16 = torch.randn(NB, BS, H_kv, D, generator=gen).to(torch.float16)
    Q16 = torch.randn(B, H_q, max(q_lens), D, generator=gen).to(torch.float16)
    G = H_q // H_kv
    extra = {}
    if int8:
        kq, ksc = orc.quantize_rows(K16.float().numpy())
        vq, vsc = orc.quantize_rows(V16.float().numpy())
        ksc16, vsc16 = ksc.astype(np.float16), vsc.astype(np.float16)
        Kr = torch.from_numpy(kq.astype(np.float32) * ksc16.astype(np.float32)[..., None])
        Vr = torch.from_numpy(vq.astype(np.float32) * vsc16.astype(np.float32)[..., None])
        extra = dict(K_i8=kq, V_i8=vq, k_scale=ksc16, v_scale=vsc16)
    else:
        Kr, Vr = K16, V16
    Kx = Kr.repeat_interleave(G, dim=2)
    Vx = Vr.repeat_interleave(G, dim=2)
    ones = torch.ones(NB, H_q, dtype=torch.float32)
    O, L = last_rows_ref(Q16, Kx, Vx, q_len, bt, nblk, BS, kv_len, ones, ones)
    pools = dict(K=K16.numpy(), V=V16.numpy()) if not extra else {}
    np.savez_compressed(os.path.join(OUT, f"attn_{name}.npz"), Q=Q16.numpy(), **pools,
                        block_table=bt.numpy(), num_blocks=nblk.numpy(), q_len=q_len.numpy(), kv_len=kv_len.numpy(),
                        block_size=BS, O_ref=O.numpy(), L_ref=L.numpy(), **extra)
    print(f"attn_{name}", O.float().abs().max().item())


def case_top_left():
    """Raw reference semantics: q_len < kv_len with the reference's own (top-left) mask."""
    gen = torch.Generator().manual_seed(7)
    B, H, D, BS = 3, 2, 64, 16
    ctx = [40, 33, 16]
    q_lens = [1, 5, 16]
    nblk_l = [-(-c // BS) for c in ctx]
    NB = sum(nblk_l) + 2
    bt, nblk = seeded_tables(gen, B, ctx, BS, NB)
    kv_len = torch.tensor(ctx, dtype=torch.int32)
    q_len = torch.tensor(q_lens, dtype=torch.int32)
    K16 = torch.randn(NB, BS, H, D, generator=gen).to(torch.float16)
    V16 = torch.randn(NB, BS, H, D, generator=gen).to(torch.float16)
    Q16 = torch.randn(B, H, max(q_lens), D, generator=gen).to(torch.float16)
    ones = torch.ones(NB, H, dtype=torch.float32)
    O, L = run_ref_kernel(Q16, K16, V16, q_len, bt, nblk, BS, kv_len, ones, ones)
    np.savez_compressed(os.path.join(OUT, "attn_top_left.npz"), Q=Q16.numpy(), K=K16.numpy(), V=V16.numpy(),
                        block_table=bt.numpy(), num_blocks=nblk.numpy(), q_len=q_len.numpy(), kv_len=kv_len.numpy(),
                        block_size=BS, O_ref=O.numpy(), L_ref=L.numpy())
    print("attn_top_left", O.float().abs().max().item())


def case_quant():
    quantize = _load_ref_quantize()
    torch.manual_seed(0)
    x1 = torch.randn(1000) * 2.0
    q1, s1 = quantize(x1)
    x2 = torch.zeros(100)
    q2, s2 = quantize(x2)
    x3 = torch.randn(100) * 0.1
    x3[0] = 50.0
    q3, s3 = quantize(x3)
    # per-row application to fp16-valued rows [T, H, D] with outliers
    gen = torch.Generator().manual_seed(3)
    rows = torch.randn(24, 4, 128, generator=gen)
    rows = rows * torch.where(torch.rand(rows.shape, generator=gen) < 0.01, 8.0, 1.0)
    rows = rows.to(torch.float16).float()
    rows[5, 2] = 0.0  # all-zero row: scale 1.0
    qr = torch.zeros(rows.shape, dtype=torch.int8)
    sr = torch.zeros(rows.shape[:2], dtype=torch.float32)
    for t in range(rows.shape[0]):
        for h in range(rows.shape[1]):
            q, s = quantize(rows[t, h])
            qr[t, h] = q
            sr[t, h] = s
    np.savez_compressed(os.path.join(OUT, "quant_reference.npz"),
                        x1=x1.numpy(), q1=q1.numpy(), s1=np.float32(s1), x2=x2.numpy(), q2=q2.numpy(),
                        s2=np.float32(s2), x3=x3.numpy(), q3=q3.numpy(), s3=np.float32(s3),
                        rows=rows.numpy(), rows_q=qr.numpy(), rows_scale=sr.numpy())
    print("quant", s1, s3)


def step_metadata(prefill_seqs, decode_seqs):
    """The per-step lists core/model_runner.py:66-107 builds (its F6 decode position included)."""
    sequence_id, length, offset, position_ids, pos_seq_id, kv_len = [], [], [], [], [], []
    cnt = 0
    for seq in prefill_seqs:
        n = len(seq.prompt_token_ids)
        sequence_id.append(seq.seq_id)
        length.append(n)
        offset.append(cnt)
        cnt += n
        pos_seq_id.extend([seq.seq_id] * n)
        position_ids.extend(range(len(seq.token_ids)))
        kv_len.append(n)
    for seq in decode_seqs:
        sequence_id.append(seq.seq_id)
        length.append(1)
        offset.append(cnt)
        cnt += 1
        pos_seq_id.append(seq.seq_id)
        position_ids.append(len(seq.token_ids))
        kv_len.append(len(seq.token_ids) + 1)
    i32 = lambda v: torch.tensor(v, dtype=torch.int32)  # noqa: E731
    return dict(sequence_id=i32(sequence_id), length=i32(length), offset=i32(offset),
                position_ids=i32(position_ids), pos_seq_id=i32(pos_seq_id), kv_len=i32(kv_len))


def case_model_layer():
    """The reference attention layer's own call of the kernel, captured over three scheduler steps."""
    import core.config as core_config

    # the layer sizes its pools from this dict at construction: a small pool
    core_config.core_configurations.update(block_size=16, num_blocks=24)
    import transformer.model as tm
    from core.block_manager import BlockManager
    from core.scheduler import Scheduler
    from core.sequence import Sequence

    assert tm.__file__.startswith(REF), tm.__file__
    torch.manual_seed(21)
    d_model, heads, BS = 128, 2, 16
    layer = tm.MultiHeadAttention(d_model, heads).eval()
    bm = BlockManager(24, BS)
    sched = Scheduler(bm, BS, 100, skip_threshold=3, lookahead=5)
    gen = torch.Generator().manual_seed(22)
    prompts = [[int(t) for t in torch.randint(0, 1000, (n,), generator=gen)] for n in (20, 7, 33)]
    for i, pr in enumerate(prompts):
        sched.add_request(Sequence(seq_id=i, prompt_token_ids=pr))

    captured = []

    class Capture:
        """Stands in for FlashAttentionFunction: records the call, answers with the oracle."""

        @staticmethod
        def apply(Q, K, V, q_len, block_table, num_blocks, block_size, kv_len, k_scale, v_scale):
            Kn = K.numpy().transpose(0, 2, 1, 3)  # the model writes [block, head, slot, d]
            Vn = V.numpy().transpose(0, 2, 1, 3)
            O, L = orc.paged_attention(Q.numpy(), Kn, Vn, q_len.numpy(), block_table.numpy(), num_blocks.numpy(),
                                       int(block_size), kv_len.numpy(), k_scale.numpy(), v_scale.numpy())
            captured.append(dict(Q=Q.clone().numpy(), K=K.clone().numpy(), V=V.clone().numpy(),
                                 q_len=q_len.clone().numpy(), block_table=block_table.clone().numpy(),
                                 num_blocks=num_blocks.clone().numpy(), kv_len=kv_len.clone().numpy(),
                                 k_scale=k_scale.clone().numpy(), v_scale=v_scale.clone().numpy(), O_ref=O,
                                 block_size=np.int32(block_size)))
            return torch.from_numpy(O).to(torch.float16)

    tm.FlashAttentionFunction = Capture
    out = {}
    for step in range(3):
        if step == 2:
            sched.add_request(Sequence(seq_id=3, prompt_token_ids=[5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16]))
        so = sched.schedule()
        md = step_metadata(so.prefill_seqs, so.decode_seqs)
        T = int(md["length"].sum())
        x = torch.randn(T, d_model, generator=gen)
        with torch.no_grad():
            y = layer(x, x, x, bm.block_table, md["length"], md["kv_len"], md["sequence_id"], md["offset"],
                      md["length"], md["position_ids"], md["pos_seq_id"])
        c = captured[-1]
        for k, v in c.items():
            out[f"s{step}_{k}"] = v
        out[f"s{step}_y"] = y.numpy()
        out[f"s{step}_offset"] = md["offset"].numpy()
        out[f"s{step}_length"] = md["length"].numpy()
        for seq in so.prefill_seqs + so.decode_seqs:  # core/model_runner.py:140-155, no EOS
            seq.token_ids.append(int(torch.randint(0, 1000, (1,), generator=gen)))
        print(f"model_layer step {step}: {len(so.prefill_seqs)} prefill, {len(so.decode_seqs)} decode, "
              f"max|O| {np.abs(c['O_ref']).max():.3f}")
    out["W_o"] = layer.W_o.weight.detach().numpy()
    out["b_o"] = layer.W_o.bias.detach().numpy()
    out["steps"] = np.int32(3)
    np.savez_compressed(os.path.join(OUT, "model_layer_steps.npz"), **out)


def case_block_trace():
    """The reference's own Scheduler + BlockManager over a seeded request trace.

    Records every allocate / release call (with its status), and after each
    scheduling step the free list, the per-sequence block lists, the step's
    metadata (core/model_runner.py:66-107) and the padded block table
    (transformer/model.py:126-152).  A small pool makes INSUFFICIENT_SPACE,
    skipped admissions and the scheduler's blocking mode occur.
    """
    from core.block_manager import BlockManager
    from core.scheduler import Scheduler
    from core.sequence import Sequence

    sys.path.insert(0, os.path.dirname(OUT))
    from oracle import block_manager as obm

    NB, BS, MAXLEN, STEPS = 48, 16, 100, 70
    bm = BlockManager(NB, BS)
    ops = []  # (step, kind 0 = allocate / 1 = release, seq_id, n, status)
    cur = [0]
    alloc0, rel0 = bm.allocate, bm.release_blocks

    def alloc(seq_id, n):
        r = alloc0(seq_id, n)
        ops.append((cur[0], 0, seq_id, n, r.status.value))
        return r

    def rel(seq_id):
        r = rel0(seq_id)
        ops.append((cur[0], 1, seq_id, 0, r.value))
        return r

    bm.allocate, bm.release_blocks = alloc, rel
    sched = Scheduler(bm, BS, MAXLEN, skip_threshold=3, lookahead=5)
    gen = torch.Generator().manual_seed(31)
    rnd = lambda lo, hi: int(torch.randint(lo, hi + 1, (1,), generator=gen))  # noqa: E731
    out = {}
    next_id = 0
    for step in range(STEPS):
        cur[0] = step
        if step < 45:
            for _ in range(rnd(0, 2)):
                sched.add_request(Sequence(seq_id=next_id, prompt_token_ids=[rnd(0, 999) for _ in range(rnd(5, 90))]))
                next_id += 1
        if step == 30:
            bm.release_blocks(10 ** 6)  # an unknown sequence: FAILURE (core/block_manager.py:49-50)
        so = sched.schedule()
        pre = [(s.seq_id, len(s.prompt_token_ids), len(s.token_ids)) for s in so.prefill_seqs]
        dec = [(s.seq_id, len(s.prompt_token_ids), len(s.token_ids)) for s in so.decode_seqs]
        md = obm.step_metadata(pre, dec)
        rows, nblk = obm.padded_block_table(bm.block_table, md["sequence_id"])
        W = max(nblk) if nblk else 0
        out[f"s{step}_stack"] = np.asarray(bm.st, np.int32)
        seqs = sorted(bm.block_table)
        out[f"s{step}_table_seq"] = np.asarray(seqs, np.int32)
        out[f"s{step}_table_len"] = np.asarray([len(bm.block_table[q]) for q in seqs], np.int32)
        out[f"s{step}_table_ids"] = np.asarray([b for q in seqs for b in bm.block_table[q]], np.int32)
        out[f"s{step}_seq_info"] = np.asarray([(sid, npr, ntk, 1) for sid, npr, ntk in pre] +
                                              [(sid, npr, ntk, 0) for sid, npr, ntk in dec], np.int32).reshape(-1, 4)
        for k, v in md.items():
            out[f"s{step}_{k}"] = np.asarray(v, np.int32)
        out[f"s{step}_block_table"] = np.asarray(rows, np.int32).reshape(len(rows), W)
        out[f"s{step}_num_blocks"] = np.asarray(nblk, np.int32)
        for s_ in so.prefill_seqs + so.decode_seqs:  # one new token; some sequences end (EOS)
            if rnd(0, 99) < 7:
                s_.is_finished = True
            else:
                s_.token_ids.append(rnd(0, 999))
    out["ops"] = np.asarray(ops, np.int32)
    out["steps"] = np.int32(STEPS)
    out["num_blocks"] = np.int32(NB)
    out["block_size"] = np.int32(BS)
    st = out["ops"][:, 4]
    print(f"block_trace: {len(ops)} ops, {int((st == 1).sum())} insufficient, {int((st == 2).sum())} failure, "
          f"{next_id} sequences")
    np.savez_compressed(os.path.join(OUT, "block_trace.npz"), **out)


CASES = {
    "quant": case_quant,
    "reference_test": case_reference_test,
    "cfg1_fp32": lambda: case_cfg1("fp32"),
    "cfg1_int8_block": lambda: case_cfg1("int8_block"),
    "cfg1_int8_token": lambda: case_cfg1("int8_token"),
    "gqa_decode_d128": lambda: case_gqa("gqa_decode_d128", 8, 2, 128, 16, [37, 128, 200, 16, 1], [1, 1, 1, 1, 1],
                                        False, 11),
    "gqa_chunked_d64": lambda: case_gqa("gqa_chunked_d64", 8, 2, 64, 16, [40, 70, 16], [3, 16, 16], False, 12),
    "gqa_int8_token_d128": lambda: case_gqa("gqa_int8_token_d128", 8, 2, 128, 16, [50, 97, 130], [1, 1, 1], True,
                                            13),
    "gqa_int8_chunked_bs32": lambda: case_gqa("gqa_int8_chunked_bs32", 4, 1, 128, 32, [65, 90], [7, 33], True, 14),
    "top_left": case_top_left,
    "model_layer": case_model_layer,
    "block_trace": case_block_trace,
}

if __name__ == "__main__":
    for name in (sys.argv[1:] or list(CASES)):
        CASES[name]()
