"""Benchmark of the B200 paged-attention hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload long_ctx_int8|decode_fp16|decode_int8|prefill_bf16|prefill_int8|
                                project_write_int8]
                    [--exchange nccl|peer] [--no-extra] [--no-cpu-baseline] [--no-reference-kernel]
                    [--batch B (long_ctx_int8)] [--tokens T (project_write_int8)]

One step = one pass of the hot path over one batch of seeded synthetic input
with the reference's benchmark shapes (no public dataset is involved):

  long_ctx_int8 (default, every N) B=256, 64/8 heads, D=128, block_size 16,
                ctx ~ U[8192, 32768], INT8 KV with fp16 per-token scales; the
                KV heads are sharded across the N ranks (strong scaling) and
                the per-head outputs gathered with an NCCL
                all_gather_into_tensor inside the timed step.  Metric: HBM
                GB/s of the algorithmic bytes (int8 K/V + scales of every
                attended token, Q, O), whole job.
  decode_fp16   paged decode attention, B=64, 32/8 heads, D=128, ctx ~
                U[512, 4096], fp16 KV.  Metric: HBM GB/s.
  decode_int8   the same shape with INT8 KV (fp16 per-token scales, 1% outliers
                x8): quantise-on-write of 64 new tokens per sequence, then decode.
  prefill_bf16  causal paged prefill, B=8, L ~ U[1024, 4096], 32/8 heads, bf16;
                K/V written into scattered fp16 blocks, then attention.
                Metric: TFLOP/s (causal FLOPs).
  prefill_int8  the same prefill over an INT8 pool (fp16 Q, quantise-on-write of
                the new rows); the attention call dequantises the blocks it reads
                once into fp16 scratch and runs the tcgen05 kernel.
  project_write_int8  the K/V projection of the prefill_bf16 tokens (x [T, 4096]
                bf16, W [2048, 4096]) with the INT8 cache write in its
                epilogue, one launch.  Metric: TFLOP/s of the projection.

On one GPU the line also carries, under ``workloads``, a full record (value,
roofline, e2e, clocks, cpu_baseline) for each of the other five workloads,
timed the same way in the same run.  ``roofline`` describes the dominant
launches: the attention call alone (no write kernel, no collective) on the
same inputs, timed by a second CUDA-event loop after the timed region; its
``step_*`` fields give the whole step per GPU against the same peak.  Inputs
exceed the 126 MB L2 for every workload; the timed region is bracketed by
barrier + synchronize, timed with CUDA events on the launching stream, max
over ranks.  ``e2e`` runs the same step through the public Python API with
each step's inputs copied from pinned host memory and the result read back
(for the sharded workload: every rank copies in its own query heads and
metadata, rank 0 reads back the gathered output).  ``--impl reference`` times
the reference's own path on the host CPU (the naive PyTorch paged attention,
restated in oracle/) on the same workloads and prints the same JSON line.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "paged-inference-engine_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# ----------------------------------------------------------------------------
# environment helpers
# ----------------------------------------------------------------------------
def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {k: float(d[k]) for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained")}, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int, period_ms: int = 50):
        self.index, self.period = index, period_ms
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-i", str(self.index),
                 "-lms", str(self.period)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------
# workloads
# ----------------------------------------------------------------------------
class Workload:
    """One benchmark case: device step, end-to-end step, and a CPU-oracle sample.

    step()          one pass of the hot path over device-resident inputs
    e2e_step()      the same through the public API with this step's inputs
                    copied from pinned host memory and the result copied back
                    (decode: the inputs packed into one pinned buffer and both
                    copies on their own streams, overlapping the neighbouring
                    steps' attention; every step still moves all of its bytes
                    inside the timed region)
    cpu_unit(i)     runs unit i of the reference's naive CPU path (the oracle
                    restatement) and returns the work it did (bytes or FLOPs);
                    units are small (tens of ms) so that samples stay bounded
    """

    metric = unit = dtype = bound = kernel = ""
    scale = 1.0
    scaling = "weak"
    launches = 1
    h2d = d2h = 0

    def io_bytes(self, ws: int) -> tuple[int, int]:
        """(host->device, device->host) bytes of one e2e step, summed over the ranks."""
        return self.h2d * ws, self.d2h * ws

    def cpu_sample(self, seconds: float, threads: int):
        torch.set_num_threads(threads)
        done, t, i = 0.0, 0.0, 0
        while t < seconds or i == 0:
            t0 = time.perf_counter()
            done += self.cpu_unit(i)
            t += time.perf_counter() - t0
            i += 1
        return t, done, i


def _pin(*ts):
    return [t.pin_memory() for t in ts]


class PipelinedInputs:
    """A step's host inputs packed into one pinned buffer and its result read back,
    both overlapped with the previous step's computation.

    step(fn): [h2d stream] wait until input slot s is free, one H2D copy of every
    input; [current stream] wait for it and for the read-back of output slot s
    two steps ago, out = fn(s, input views of slot s); [d2h stream] copy `out`
    into pinned host memory.  start() / end() bracket the timed region: the
    copy streams start after its opening event and its closing event follows
    the last read-back.
    """

    def __init__(self, host: list, out_host: list, device, readback: bool = True):
        self.readback = readback
        self.offs, total = [], 0
        for t in host:
            total = (total + 255) // 256 * 256
            self.offs.append(total)
            total += t.numel() * t.element_size()
        self.hbuf = torch.empty(total, dtype=torch.uint8).pin_memory()
        for t, o in zip(host, self.offs):
            n = t.numel() * t.element_size()
            self.hbuf[o:o + n].copy_(t.contiguous().view(-1).view(torch.uint8))
        self.nbytes = sum(t.numel() * t.element_size() for t in host)
        self.dbufs = [torch.empty(total, dtype=torch.uint8, device=device) for _ in range(2)]
        self.views = [[d[o:o + t.numel() * t.element_size()].view(t.dtype).view(t.shape)
                       for t, o in zip(host, self.offs)] for d in self.dbufs]
        self.out_host = out_host
        self.device = device
        self.h2d = torch.cuda.Stream(device)
        self.d2h = torch.cuda.Stream(device)
        ev = lambda: [torch.cuda.Event() for _ in range(2)]  # noqa: E731
        self.ready, self.free, self.computed, self.read = ev(), ev(), ev(), ev()
        self.i = 0

    def start(self):
        cur = torch.cuda.current_stream(self.device)
        self.h2d.wait_stream(cur)
        self.d2h.wait_stream(cur)

    def end(self):
        torch.cuda.current_stream(self.device).wait_stream(self.d2h)

    def step(self, fn):
        s = self.i & 1
        cur = torch.cuda.current_stream(self.device)
        with torch.cuda.stream(self.h2d):
            if self.i >= 2:
                self.h2d.wait_event(self.free[s])
            self.dbufs[s].copy_(self.hbuf, non_blocking=True)
            self.ready[s].record(self.h2d)
        cur.wait_event(self.ready[s])
        if self.i >= 2 and self.readback:
            cur.wait_event(self.read[s])
        out = fn(s, self.views[s])
        self.free[s].record(cur)
        self.computed[s].record(cur)
        if self.readback:
            out.record_stream(self.d2h)  # a per-call output stays allocated until it is read back
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self.computed[s])
                self.out_host[s].copy_(out, non_blocking=True)
                self.read[s].record(self.d2h)
        self.i += 1


class DecodeWorkload(Workload):
    """decode_fp16 / decode_int8: B=64, 32/8 heads, D=128, ctx ~ U[512, 4096]."""

    def __init__(self, name: str, seed: int, device, cpu_only: bool = False):
        from pie_b200.workloads import config_batch

        self.name = name
        b = config_batch(name, seed=seed)
        self.b = b
        B, Hq, _, D = b.Q.shape
        Hkv = b.K.shape[2]
        self.sum_ctx = int(b.kv_len.long().sum())
        kv_bytes = self.sum_ctx * Hkv * b.kv_bytes_per_token_head
        qo_bytes = 2 * B * Hq * D * 2 + B * Hq * 2
        self.info = {"B": B, "Hq": Hq, "Hkv": Hkv, "D": D, "block_size": b.block_size, "sum_ctx": self.sum_ctx,
                     "kv_dtype": str(b.K.dtype).replace("torch.", "")}
        self.int8 = name == "decode_int8"
        self.work = kv_bytes + qo_bytes
        self.dominant_work = self.work  # the attention launches alone
        self.write = None
        if self.int8:
            T_new = 64
            gen = torch.Generator().manual_seed(seed + 99)
            kn = (torch.randn(B * T_new, Hkv, D, generator=gen) *
                  torch.where(torch.rand(B * T_new, Hkv, D, generator=gen) < 0.01, 8.0, 1.0)).half()
            vn = torch.randn(B * T_new, Hkv, D, generator=gen).half()
            seq = torch.arange(B, dtype=torch.int32).repeat_interleave(T_new)
            pos = (b.kv_len.view(-1, 1) - T_new + torch.arange(T_new).view(1, -1)).reshape(-1).to(torch.int32)
            self.write = (kn, vn, seq, pos)
            self.work += 2 * B * T_new * Hkv * (D * 2 + D + 2)
            self.info["new_tokens_per_seq"] = T_new
        self.unit, self.scale, self.bound, self.dtype = "GB/s", 1e-9, "hbm", "i8" if self.int8 else "f16"
        self.metric = ("paged decode attention + quantise-on-write HBM GB/s (INT8 KV, B=64, 32/8 heads, D=128)"
                       if self.int8 else
                       "paged decode attention HBM GB/s (fp16 KV, B=64, 32/8 heads, D=128, ctx~U[512,4096])")
        self.kernel = "paged_attn_decode (split + merge launches)" + (" + kv_write_quant" if self.int8 else "")
        self.dominant_name = "paged_attn_decode (pa_decode_kernel + pa_decode_merge_kernel)"
        self.launches = 3 if self.int8 else 2
        if not cpu_only:
            self._device(device)

    def _device(self, device):
        from kernels.flash_attention import flash_attention_forward, write_kv_cache

        b, g = self.b, self.b.to(device)
        self.g = g
        wd = None if self.write is None else [t.to(device) for t in self.write]

        def attend(out=None):
            return flash_attention_forward(g.Q, g.K, g.V, g.q_len, g.block_table, g.num_blocks, g.block_size,
                                           g.kv_len, g.k_scale, g.v_scale, out=out)

        def step(out=None):
            if wd is not None:
                write_kv_cache(wd[0], wd[1], g.block_table, wd[2], wd[3], g.K, g.V, g.k_scale, g.v_scale)
            return attend(out)
        self.step = step
        self.dominant = attend

        outs = [torch.empty(b.Q.shape, dtype=torch.float16, device=device) for _ in range(2)]
        hO = [torch.empty(b.Q.shape, dtype=torch.float16).pin_memory() for _ in range(2)]
        pipe = PipelinedInputs([b.Q, b.block_table, b.num_blocks, b.q_len, b.kv_len, *(self.write or ())], hO,
                               device)
        self.h2d = pipe.nbytes
        self.d2h = hO[0].numel() * hO[0].element_size()

        def run(s, v):
            Q, bt, nb, ql, kl = v[:5]
            if self.write is not None:
                write_kv_cache(v[5], v[6], bt, v[7], v[8], g.K, g.V, g.k_scale, g.v_scale)
            O, _ = flash_attention_forward(Q, g.K, g.V, ql, bt, nb, g.block_size, kl, g.k_scale, g.v_scale,
                                           out=outs[s])
            return O

        self.e2e_step = lambda: pipe.step(run)
        self.e2e_start, self.e2e_end = pipe.start, pipe.end

    def cpu_unit(self, i):
        from oracle import paged_attention as orc

        b = self.b
        if not hasattr(self, "_np"):
            self._np = (b.Q.float().numpy(), b.K.numpy(), b.V.numpy(),
                        None if b.k_scale is None else b.k_scale.numpy(),
                        None if b.v_scale is None else b.v_scale.numpy(),
                        *[t.numpy() for t in (b.q_len, b.block_table, b.num_blocks, b.kv_len)])
        Q, K, V, ks, vs, ql, bt, nb, kl = self._np
        s = slice(i % len(kl), i % len(kl) + 1)
        orc.paged_attention(Q[s], K, V, ql[s], bt[s], nb[s], b.block_size, kl[s], ks, vs)
        return float(kl[s][0]) * K.shape[2] * b.kv_bytes_per_token_head

    def sample_desc(self, n, t):
        return f"{n} whole sequences of the workload, one at a time, {t:.1f} s"


class PrefillWorkload(Workload):
    """prefill_bf16: B=8, L ~ U[1024, 4096], 32/8 heads, D=128, bf16; write K/V then attend.

    prefill_int8: the same shape over an INT8 pool (fp16 Q and new rows, quantise-on-write with
    head-major fp16 per-token scales); the attention call dequantises the blocks it reads once
    into fp16 scratch, then runs the tcgen05 kernel.
    """

    ROWS = 64  # query rows per CPU unit

    def __init__(self, seed: int, device, cpu_only: bool = False, int8: bool = False):
        from pie_b200.workloads import CONFIGS, block_tables, draw_context_lengths

        self.int8 = int8
        self.name = "prefill_int8" if int8 else "prefill_bf16"
        cfg = CONFIGS["prefill_bf16"]
        gen = torch.Generator().manual_seed(seed)
        L = draw_context_lengths(gen, cfg["B"], *cfg["ctx_range"])
        B, Hq, Hkv, D, BS = cfg["B"], cfg["Hq"], cfg["Hkv"], cfg["D"], cfg["BS"]
        bt, nblk, NB = block_tables(gen, L, BS)
        maxL = max(L)
        self.L, self.BS, self.NB = L, BS, NB
        dt = torch.float16 if int8 else torch.bfloat16
        self.Q = torch.randn(B, Hq, maxL, D, generator=gen).to(dt)
        T = sum(L)
        self.kn = torch.randn(T, Hkv, D, generator=gen).to(dt)
        self.vn = torch.randn(T, Hkv, D, generator=gen).to(dt)
        self.seq = torch.cat([torch.full((l,), i, dtype=torch.int32) for i, l in enumerate(L)])
        self.pos = torch.cat([torch.arange(l, dtype=torch.int32) for l in L])
        self.bt, self.nblk = bt, nblk
        self.Lt = torch.tensor(L, dtype=torch.int32)
        self.work = sum(4.0 * Hq * D * l * (l + 1) / 2 for l in L)
        self.dominant_work = self.work
        self.info = {"B": B, "Hq": Hq, "Hkv": Hkv, "D": D, "block_size": BS, "sum_len": T,
                     "q_dtype": "float16" if int8 else "bfloat16", "kv_dtype": "int8" if int8 else "float16"}
        self.unit, self.scale, self.bound, self.dtype = "TFLOP/s", 1e-12, "tensor", "f16" if int8 else "bf16"
        if int8:
            self.metric = ("causal paged prefill TFLOP/s (INT8 KV pool, fp16 Q, B=8, L~U[1024,4096], 32/8 heads, "
                           "D=128)")
            self.kernel = "kv_write_quant + paged_attn_forward (kv_dequant_kernel + pa_prefill_tc2_kernel)"
            self.dominant_name = "paged_attn_forward, INT8 pool (kv_dequant_kernel + pa_prefill_tc2_kernel)"
        else:
            self.metric = "causal paged prefill TFLOP/s (bf16, B=8, L~U[1024,4096], 32/8 heads, D=128)"
            self.kernel = "kv_write_copy + paged_attn_prefill"
            self.dominant_name = "paged_attn_prefill (pa_prefill_tc2_kernel)"
        self.launches = 2
        self.Hq, self.D = Hq, D
        if not cpu_only:
            self._device(device)

    def _device(self, device):
        from kernels.flash_attention import flash_attention_forward, write_kv_cache

        host = _pin(self.Q, self.kn, self.vn, self.seq, self.pos, self.bt, self.nblk, self.Lt)
        dev = [t.to(device) for t in host]
        Qd, knd, vnd, seqd, posd, btd, nbd, Ld = dev
        Hkv, D = self.kn.shape[1], self.kn.shape[2]
        ks = vs = None
        if self.int8:
            from pie_b200.workloads import empty_head_major_scales

            Kc = torch.empty(self.NB, self.BS, Hkv, D, dtype=torch.int8, device=device)
            ks = empty_head_major_scales(self.NB, self.BS, Hkv, device=device)
            vs = empty_head_major_scales(self.NB, self.BS, Hkv, device=device)
        else:
            Kc = torch.empty(self.NB, self.BS, Hkv, D, dtype=torch.float16, device=device)
        Vc = torch.empty_like(Kc)
        self.dev = dict(Q=Qd, K=Kc, V=Vc, ks=ks, vs=vs, bt=btd, nb=nbd, L=Ld, kn=knd, vn=vnd, seq=seqd, pos=posd)

        def attend(out=None):
            return flash_attention_forward(Qd, Kc, Vc, Ld, btd, nbd, self.BS, Ld, ks, vs, out=out)

        def step(out=None):
            write_kv_cache(knd, vnd, btd, seqd, posd, Kc, Vc, ks, vs)
            return attend(out)
        self.step = step
        self.dominant = attend

        outs = [torch.empty(self.Q.shape, dtype=torch.float16, device=device) for _ in range(2)]
        hO = [torch.empty(self.Q.shape, dtype=torch.float16).pin_memory() for _ in range(2)]
        pipe = PipelinedInputs(host, hO, device)
        self.h2d = pipe.nbytes
        self.d2h = hO[0].numel() * hO[0].element_size()

        def run(s, v):
            Q, kn, vn, seq, pos, bt, nb, Lx = v
            write_kv_cache(kn, vn, bt, seq, pos, Kc, Vc, ks, vs)
            O, _ = flash_attention_forward(Q, Kc, Vc, Lx, bt, nb, self.BS, Lx, ks, vs, out=outs[s])
            return O

        self.e2e_step = lambda: pipe.step(run)
        self.e2e_start, self.e2e_end = pipe.start, pipe.end

    def _cpu_pool(self):
        # the copy-on-write of the new rows, done once (not timed)
        import numpy as np

        from oracle import paged_attention as orc

        Hkv, D = self.kn.shape[1], self.kn.shape[2]
        seq, pos, bt = self.seq.numpy(), self.pos.numpy(), self.bt.numpy()
        blk = bt[seq, pos // self.BS]
        ks = vs = None
        if self.int8:
            K = np.zeros((self.NB, self.BS, Hkv, D), np.int8)
            V = np.zeros_like(K)
            ks = np.ones((self.NB, self.BS, Hkv), np.float16)
            vs = np.ones_like(ks)
            for src, dst, sc in ((self.kn, K, ks), (self.vn, V, vs)):
                q, s = orc.quantize_rows(src.float().numpy())
                dst[blk, pos % self.BS] = q
                sc[blk, pos % self.BS] = s.astype(np.float16)
        else:
            K = np.zeros((self.NB, self.BS, Hkv, D), np.float16)
            V = np.zeros_like(K)
            K[blk, pos % self.BS] = self.kn.float().numpy().astype(np.float16)
            V[blk, pos % self.BS] = self.vn.float().numpy().astype(np.float16)
        units = [(b, lo) for b, l in enumerate(self.L) for lo in range(0, l, self.ROWS)]
        order = np.random.default_rng(0).permutation(len(units))
        return K, V, ks, vs, [units[j] for j in order]

    def cpu_unit(self, i):
        """Query rows [lo, lo + ROWS) of one sequence against its causal keys."""
        from oracle import paged_attention as orc

        if not hasattr(self, "_cpu"):
            self._cpu = self._cpu_pool()
        K, V, ks, vs, units = self._cpu
        b, lo = units[i % len(units)]
        l = self.L[b]
        hi = min(l, lo + self.ROWS)
        q = self.Q[b:b + 1, :, lo:hi].float().numpy()
        # bottom-right causal with kv_len = hi: row m (absolute lo + m) sees keys 0..lo+m
        orc.paged_attention(q, K, V, [hi - lo], self.bt[b:b + 1].numpy(), self.nblk[b:b + 1].numpy(), self.BS, [hi],
                            ks, vs)
        return 4.0 * self.Hq * self.D * sum(r + 1 for r in range(lo, hi))

    def sample_desc(self, n, t):
        return f"{n} blocks of {self.ROWS} query rows drawn from the workload's sequences, {t:.1f} s"


class ProjectWriteWorkload(Workload):
    """project_write_int8: the K/V projection of a prefill batch with the INT8 cache write in its epilogue.

    x [T, 4096] bf16 with T the prefill_bf16 tokens (B=8, L ~ U[1024, 4096]), W = [W_k; W_v]
    [2 * 8 * 128, 4096] bf16, fp32 bias; every token's K and V rows are quantised (one fp16 scale per
    token and head, head-major) into scattered blocks of 16 slots.  Metric: TFLOP/s of the projection.
    """

    ROWS = 64  # tokens per CPU unit

    def __init__(self, seed: int, device, cpu_only: bool = False, tokens: int = 0):
        from pie_b200.workloads import CONFIGS, block_tables, draw_context_lengths

        self.name = "project_write_int8"
        cfg = CONFIGS["prefill_bf16"]
        gen = torch.Generator().manual_seed(seed)
        L = draw_context_lengths(gen, cfg["B"], *cfg["ctx_range"])
        if tokens:  # one sequence of `tokens` new tokens (a decode-sized batch)
            L = [tokens]
        Hq, Hkv, D, BS = cfg["Hq"], cfg["Hkv"], cfg["D"], cfg["BS"]
        dm = Hq * D
        bt, nblk, NB = block_tables(gen, L, BS)
        T = sum(L)
        self.T, self.dm, self.Hkv, self.D, self.BS, self.NB = T, dm, Hkv, D, BS, NB
        self.x = torch.randn(T, dm, generator=gen).to(torch.bfloat16)
        self.w = (torch.randn(2 * Hkv * D, dm, generator=gen) / dm ** 0.5).to(torch.bfloat16)
        self.b = torch.randn(2 * Hkv * D, generator=gen) * 0.1
        self.seq = torch.cat([torch.full((l,), i, dtype=torch.int32) for i, l in enumerate(L)])
        self.pos = torch.cat([torch.arange(l, dtype=torch.int32) for l in L])
        self.bt = bt
        self.work = 2.0 * T * dm * 2 * Hkv * D
        self.dominant_work = self.work
        self.info = {"T": T, "d_model": dm, "Hkv": Hkv, "D": D, "block_size": BS, "x_dtype": "bfloat16",
                     "kv_dtype": "int8", "scales": "fp16 per (token, head), head-major"}
        self.unit, self.scale, self.bound, self.dtype = "TFLOP/s", 1e-12, "tensor", "bf16"
        self.metric = ("K/V projection with the INT8 paged-cache write in its epilogue, TFLOP/s "
                       f"(T = {'%d tokens' % tokens if tokens else 'prefill_bf16 tokens'}, d_model 4096, 8 KV heads, "
                       "D=128)")
        self.kernel = "kv_project_write (kv_project_kernel)"
        self.dominant_name = "kv_project_kernel"
        self.launches = 1
        if not cpu_only:
            self._device(device)

    def _device(self, device):
        from kernels.flash_attention import project_write_kv_cache
        from pie_b200.workloads import empty_head_major_scales

        host = _pin(self.x, self.seq, self.pos, self.bt)
        xd, seqd, posd, btd = [t.to(device) for t in host]
        wd, bd = self.w.to(device), self.b.to(device)
        KV = torch.empty(2, self.NB, self.BS, self.Hkv, self.D, dtype=torch.int8, device=device)
        ks = empty_head_major_scales(self.NB, self.BS, self.Hkv, device=device)
        vs = empty_head_major_scales(self.NB, self.BS, self.Hkv, device=device)
        self.dev = dict(x=xd, w=wd, b=bd, KV=KV)

        def step():
            project_write_kv_cache(xd, wd, bd, btd, seqd, posd, KV[0], KV[1], ks, vs)
        self.step = self.dominant = step

        hKV = [torch.empty(KV.shape, dtype=torch.int8).pin_memory() for _ in range(2)]
        pipe = PipelinedInputs(host, hKV, device)
        self.h2d = pipe.nbytes
        self.d2h = KV.numel()

        def run(s, v):
            x, seq, pos, bt = v
            project_write_kv_cache(x, wd, bd, bt, seq, pos, KV[0], KV[1], ks, vs)
            return KV

        self.e2e_step = lambda: pipe.step(run)
        self.e2e_start, self.e2e_end = pipe.start, pipe.end

    def cpu_unit(self, i):
        """The reference's path for 64 tokens: x @ W^T + b in float32 (transformer/model.py:75-82), then
        the per-(token, head) quantisation of the cache write (:85-122, restated in the oracle)."""
        from oracle import paged_attention as orc

        if not hasattr(self, "_wf"):
            self._wf = self.w.float()
        n = (self.T + self.ROWS - 1) // self.ROWS
        lo = (i * 7919 % n) * self.ROWS
        xs = self.x[lo:lo + self.ROWS].float()
        y = torch.addmm(self.b, xs, self._wf.T).view(-1, 2, self.Hkv, self.D).numpy()
        orc.quantize_rows(y[:, 0])
        orc.quantize_rows(y[:, 1])
        return 2.0 * xs.shape[0] * self.dm * 2 * self.Hkv * self.D

    def sample_desc(self, n, t):
        return f"{n} blocks of {self.ROWS} tokens (float32 projection + quantisation), {t:.1f} s"


class LongCtxWorkload(Workload):
    """long_ctx_int8: B=256, 64/8 heads, ctx ~ U[8192, 32768], INT8; KV heads sharded over ranks."""

    def __init__(self, ws: int, rank: int, device, cpu_only: bool = False, exchange: str = "nccl",
                 batch: int = 0):
        from pie_b200.workloads import CONFIGS, draw_context_lengths

        self.name = "long_ctx_int8"
        self.exchange = exchange
        cfg = dict(CONFIGS["long_ctx_int8"])
        if batch:
            cfg["B"] = batch
        self.cfg = cfg
        Bn, Hq, Hkv, D, BS = cfg["B"], cfg["Hq"], cfg["Hkv"], cfg["D"], cfg["BS"]
        gen = torch.Generator().manual_seed(0)
        self.ctx = draw_context_lengths(gen, Bn, *cfg["ctx_range"])  # same sequences on every rank
        self.sum_ctx = sum(self.ctx)
        self.work = self.sum_ctx * Hkv * (2 * D + 4) + 2 * Bn * Hq * D * 2
        self.info = {"B": Bn, "Hq": Hq, "Hkv": Hkv, "D": D, "block_size": BS, "sum_ctx": self.sum_ctx}
        self.unit, self.scale, self.bound, self.dtype = "GB/s", 1e-9, "hbm", "i8"
        self.scaling = "strong"
        self.metric = ("long-context paged decode HBM GB/s, KV heads sharded over GPUs (INT8 KV, B=256, 64/8 heads, "
                       "ctx~U[8192,32768])")
        self.kernel = ("paged_attn_decode per GPU (split + merge" +
                       (", output rows stored into peer buffers + barrier)" if exchange == "peer" and ws > 1
                        else ", + NCCL all_gather)" if ws > 1 else ")"))
        self.dominant_name = "paged_attn_decode per GPU, local heads (split + merge, no collective)"
        self.launches = 2
        self.ws, self.rank = ws, rank
        if not cpu_only:
            self._device(device)

    def _device(self, device):
        from pie_b200.sharded import KVHeadShardedDecoder, build_rank_pool

        c = self.cfg
        Bn, Hq, Hkv, D, BS = c["B"], c["Hq"], c["Hkv"], c["D"], c["BS"]
        dec = KVHeadShardedDecoder(Hq, Hkv, D, exchange=self.exchange)
        K, V, ks, vs, bt, nblk, NB = build_rank_pool(self.ctx, Hkv // self.ws, D, BS, 1000 + self.rank, device)
        Qfull = torch.randn(Bn, Hq, 1, D, generator=torch.Generator().manual_seed(5)).half()
        Ql = dec.local_q(Qfull).contiguous().to(device)
        ql = torch.ones(Bn, dtype=torch.int32, device=device)
        kl = torch.tensor(self.ctx, dtype=torch.int32, device=device)

        def step():
            return dec.forward(Ql, K, V, ql, bt, nblk, BS, kl, ks, vs)
        self.step = step
        self.dominant = lambda: dec.forward(Ql, K, V, ql, bt, nblk, BS, kl, ks, vs, gather=False)
        self.dominant_work = self.work / self.ws  # this rank's KV heads, Q and O

        # every rank copies in its own query heads and paging metadata; the
        # gathered O (all heads) is read back once, by rank 0
        hO = [torch.empty(Bn, Hq, 1, D, dtype=torch.float16).pin_memory() for _ in range(2)]
        pipe = PipelinedInputs([dec.local_q(Qfull).contiguous(), bt.cpu(), nblk.cpu(), ql.cpu(), kl.cpu()], hO,
                               device, readback=self.rank == 0)
        self.h2d = pipe.nbytes
        self.d2h = hO[0].numel() * hO[0].element_size()
        self.dec = dec

        def run(s, v):
            return dec.forward(v[0], K, V, v[3], v[1], v[2], BS, v[4], ks, vs)

        self.e2e_step = lambda: pipe.step(run)
        self.e2e_start, self.e2e_end = pipe.start, pipe.end

    def io_bytes(self, ws: int) -> tuple[int, int]:
        return self.h2d * ws, self.d2h

    def close(self):
        self.dec.close()

    def cpu_unit(self, i):
        """One sequence of the workload's shape (ctx from its range) over all 8 KV heads."""
        from oracle import paged_attention as orc
        from pie_b200.workloads import make_decode_batch

        if not hasattr(self, "_cpu"):
            c = self.cfg
            ctx = self.ctx[:4]
            b = make_decode_batch(1000, len(ctx), c["Hq"], c["Hkv"], c["D"], c["BS"], ctx, kv_dtype=torch.int8,
                                  outliers=0.01)
            self._cpu = (b, b.Q.float().numpy(), b.K.numpy(), b.V.numpy(), b.k_scale.numpy(), b.v_scale.numpy(),
                         *[t.numpy() for t in (b.q_len, b.block_table, b.num_blocks, b.kv_len)])
        b, Q, K, V, ks, vs, ql, bt, nb, kl = self._cpu
        s = slice(i % len(kl), i % len(kl) + 1)
        orc.paged_attention(Q[s], K, V, ql[s], bt[s], nb[s], b.block_size, kl[s], ks, vs)
        return float(kl[s][0]) * K.shape[2] * b.kv_bytes_per_token_head

    def sample_desc(self, n, t):
        return f"{n} sequences (4 distinct, ctx from the workload's range, all 8 KV heads), {t:.1f} s"


def make_workload(name: str, ws: int, rank: int, device, cpu_only: bool = False, exchange: str = "nccl",
                  batch: int = 0, tokens: int = 0) -> Workload:
    if name in ("prefill_bf16", "prefill_int8"):
        return PrefillWorkload(1000 + rank, device, cpu_only, int8=name == "prefill_int8")
    if name == "long_ctx_int8":
        return LongCtxWorkload(ws, rank, device, cpu_only, exchange, batch)
    if name == "project_write_int8":
        return ProjectWriteWorkload(1000 + rank, device, cpu_only, tokens)
    return DecodeWorkload(name, 1000 + rank, device, cpu_only)


# ----------------------------------------------------------------------------
# timing
# ----------------------------------------------------------------------------
def time_steps(step, steps: int, warmup: int, device, ws: int, on_start=None, on_end=None):
    for _ in range(warmup):
        step()
    torch.cuda.synchronize(device)
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(device)
    e0.record(stream)
    if on_start is not None:
        on_start()
    for _ in range(steps):
        step()
    if on_end is not None:
        on_end()
    e1.record(stream)
    torch.cuda.synchronize(device)
    if ws > 1:
        torch.distributed.barrier()
    ms = e0.elapsed_time(e1)
    if ws > 1:
        t = torch.tensor([ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def read_traffic(name: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", f"{name}.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


def measure(w: Workload, a, device, ws: int, rank: int, local: int, peaks: dict, peak_kind: str,
            cpu_baseline: bool) -> dict:
    """Time one workload: the step (``value``), its dominant launches alone (``roofline``),
    the public-API step with host buffers (``e2e``), clocks during the timed
    region, and (rank 0, one GPU) the reference's CPU path on a bounded sample."""
    if w.bound == "hbm":
        peak, punit = peaks["hbm_gbs"], "GB/s"
    else:
        peak, punit = peaks["bf16_tflops"], "TFLOP/s"
    with ClockSampler(local) as clk:
        ms = time_steps(w.step, a.steps, a.warmup, device, ws)
    ms_step = ms / a.steps
    # weak scaling: every rank runs its own batch; strong: the ranks share one
    total_work = w.work * (ws if w.scaling == "weak" else 1)
    value = total_work / (ms_step * 1e-3) * w.scale
    per_gpu = value / ws

    # the dominant launches alone (no write kernel, no collective), same inputs
    dom_ms = time_steps(w.dominant, a.steps, a.warmup, device, ws) / a.steps
    dom = w.dominant_work / (dom_ms * 1e-3) * w.scale

    e2e_steps = max(10, a.steps // 10)
    e_ms = time_steps(w.e2e_step, e2e_steps, a.warmup, device, ws, getattr(w, "e2e_start", None),
                      getattr(w, "e2e_end", None)) / e2e_steps
    e2e = {"value": round(total_work / (e_ms * 1e-3) * w.scale, 2), "unit": w.unit,
           "h2d_bytes_per_step": w.io_bytes(ws)[0], "d2h_bytes_per_step": w.io_bytes(ws)[1],
           "steps": e2e_steps, "ms_per_step": round(e_ms, 5)}
    rec = {
        "metric": w.metric, "value": round(value, 2), "unit": w.unit, "ms_per_step": round(ms_step, 5),
        "us_per_step": round(ms_step * 1e3, 2), "higher_is_better": True, "scaling": w.scaling, "dtype": w.dtype,
        "config": {"workload": w.name, **w.info,
                   "parallelism": ((f"kv-head shard x{ws} + " +
                                    ("NCCL all_gather_into_tensor" if getattr(w, "exchange", "nccl") == "nccl"
                                     else "output rows stored into peer buffers")) if w.scaling == "strong"
                                   else f"dp{ws} (one batch per rank)"),
                   "l2": "inputs larger than L2 (126 MB)"},
        "roofline": {"bound": w.bound, "achieved": round(dom, 2), "peak": peak, "unit": punit,
                     "frac": round(dom / peak, 4), "traffic": rank_traffic(w, ws),
                     "kernel": w.dominant_name, "us_per_launch": round(dom_ms * 1e3, 2),
                     "step_achieved": round(per_gpu, 2), "step_frac": round(per_gpu / peak, 4),
                     "step_kernels": w.kernel, "peak_source": f"{peak_kind} MEASURED_PEAKS"},
        "e2e": e2e,
        "gpu_launches": w.launches * a.steps,
        "clocks": clk.summary(),
    }
    if cpu_baseline and rank == 0 and ws == 1:
        threads = os.cpu_count() or 1
        t, done, n = w.cpu_sample(a.cpu_seconds, threads)
        rec["cpu_baseline"] = {"value": round(done / t * w.scale, 4), "unit": w.unit, "cores": threads,
                               "kind": "port", "sample": w.sample_desc(n, t)}
    return rec


EXTRA_WORKLOADS = ("decode_fp16", "decode_int8", "prefill_bf16", "prefill_int8", "project_write_int8")
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def load_reference_kernel_module():
    """The reference's unmodified kernels/flash_attention.py from baseline/_ref, under its own module name."""
    import importlib.util

    path = os.path.join(REF_DIR, "kernels", "flash_attention.py")
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} missing (python baseline/install_reference.py REFERENCE_ROOT)")
    spec = importlib.util.spec_from_file_location("reference_flash_attention", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def reference_kernel_leg(w: Workload, a, device) -> dict:
    """The reference's own GPU kernel on this workload, through its own launcher, on this B200.

    ``flash_attention_forward`` (kernels/flash_attention.py:139-172, Triton JIT
    for sm_100, first call autotunes) with the inputs the reference's kernel
    accepts: float32 Q (its tl.dot needs float32 operands), K/V heads expanded
    to the query heads (it has no grouped-query attention), unit float32
    per-(block, head) scales for float16 pools, per-block scales for INT8
    pools (its only scale layout).  Decode calls use q_len = 1: the kernel's
    top-left mask then lets the query see key 0 only (its output is not a
    decode result), but every program still loads and multiplies every block
    of its sequence, so the time is that of its decode.  Prefill calls are
    exact (q_len = kv_len).  Reported against the workload's own algorithmic
    work: the same bytes or causal FLOPs as ``value``.
    """
    if w.name == "project_write_int8":
        return reference_projection_leg(w, a, device)
    try:
        import triton

        ref = load_reference_kernel_module()
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    try:
        if w.name.startswith("prefill"):
            d = w.dev
            from kernels.flash_attention import write_kv_cache

            write_kv_cache(d["kn"], d["vn"], d["bt"], d["seq"], d["pos"], d["K"], d["V"], d["ks"], d["vs"])
            G = d["Q"].shape[1] // d["K"].shape[2]
            Q = d["Q"].float()
            Kx = d["K"].repeat_interleave(G, dim=2)
            Vx = d["V"].repeat_interleave(G, dim=2)
            if d["ks"] is not None:
                ks = d["ks"].float().amax(dim=1).repeat_interleave(G, dim=1).contiguous()
                vs = d["vs"].float().amax(dim=1).repeat_interleave(G, dim=1).contiguous()
                note = "prefill rows (q_len = kv_len), INT8 pool with per-(block, head) scales, heads expanded x4"
            else:
                ks = vs = torch.ones(Kx.shape[0], Kx.shape[2], dtype=torch.float32, device=device)
                note = "prefill rows (q_len = kv_len), K/V heads expanded x4, float32 Q"
            args = (Q, Kx, Vx, d["L"], d["bt"], d["nb"], w.BS, d["L"], ks, vs)
        else:
            g = w.g
            G = g.Q.shape[1] // g.K.shape[2]
            Q = g.Q.float()
            Kx = g.K.repeat_interleave(G, dim=2)
            Vx = g.V.repeat_interleave(G, dim=2)
            if g.K.dtype == torch.int8:
                ks = g.k_scale.float().amax(dim=1).repeat_interleave(G, dim=1).contiguous()
                vs = g.v_scale.float().amax(dim=1).repeat_interleave(G, dim=1).contiguous()
                note = "q_len 1 (top-left mask), INT8 pool with per-(block, head) scales, heads expanded x4"
            else:
                ks = vs = torch.ones(Kx.shape[0], Kx.shape[2], dtype=torch.float32, device=device)
                note = "q_len 1 (top-left mask), fp16 pool, heads expanded x4"
            args = (Q, Kx, Vx, g.q_len, g.block_table, g.num_blocks, g.block_size, g.kv_len, ks, vs)
        t0 = time.perf_counter()
        ref.flash_attention_forward(*args)  # compiles and autotunes
        torch.cuda.synchronize(device)
        first_s = time.perf_counter() - t0
        ms = time_steps(lambda: ref.flash_attention_forward(*args), a.steps, a.warmup, device, 1) / a.steps
        val = w.dominant_work / (ms * 1e-3) * w.scale
        best = getattr(ref.flash_attention_kernel, "best_config", None)
        return {"impl": "reference Triton kernel, unmodified (baseline/_ref/kernels/flash_attention.py)",
                "triton": triton.__version__, "value": round(val, 3), "unit": w.unit,
                "us_per_call": round(ms * 1e3, 2), "first_call_s": round(first_s, 2),
                "best_config": str(best) if best is not None else None, "inputs": note,
                "ours_over_reference": None}
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"{type(e).__name__}: {e}"[:300]}


def reference_projection_leg(w: Workload, a, device) -> dict:
    """The reference's projection on this B200: two float32 nn.Linear calls (W_k, W_v) over the same
    tokens (transformer/model.py:75-76, cuBLAS).  Its cache write that follows, a per-token Python loop
    with host synchronisations (:85-122), is not timed, so this leg is faster than the reference's path."""
    try:
        import torch.nn.functional as F

        d = w.dev
        x = d["x"].float()
        Wk, Wv = d["w"].float().chunk(2)
        bk, bv = d["b"].chunk(2)

        def ref_step():
            F.linear(x, Wk, bk)
            F.linear(x, Wv, bv)
        ms = time_steps(ref_step, a.steps, a.warmup, device, 1) / a.steps
        val = w.dominant_work / (ms * 1e-3) * w.scale
        return {"impl": "reference projection: float32 nn.Linear for W_k and W_v (cuBLAS), cache write not timed",
                "value": round(val, 3), "unit": w.unit, "us_per_call": round(ms * 1e3, 2),
                "tf32": bool(torch.backends.cuda.matmul.allow_tf32), "ours_over_reference": None}
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"{type(e).__name__}: {e}"[:300]}


def rank_traffic(w: Workload, ws: int):
    """DRAM bytes of one dominant launch on one rank (a strong-scaled rank reads 1/ws of the pool)."""
    t = read_traffic(f"{w.name}_dominant_kernel")
    if t is None:
        return None
    return round(t / ws) if w.scaling == "strong" else t


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="long_ctx_int8",
                    choices=["decode_fp16", "decode_int8", "prefill_bf16", "prefill_int8", "project_write_int8",
                             "long_ctx_int8"])
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="one GPU: skip the records of the other workloads under the 'workloads' key")
    ap.add_argument("--exchange", default="nccl", choices=["nccl", "peer"],
                    help="long_ctx_int8 head-output exchange: NCCL all-gather or stores into peer buffers")
    ap.add_argument("--no-reference-kernel", action="store_true",
                    help="one GPU: skip timing the reference's own Triton kernel on the extra workloads")
    ap.add_argument("--batch", type=int, default=0,
                    help="long_ctx_int8 with fewer sequences (same context-length draws), for small profiler "
                         "captures; 0 = the workload's 256")
    ap.add_argument("--tokens", type=int, default=0,
                    help="project_write_int8 with one sequence of this many tokens (a decode-sized batch); "
                         "0 = the prefill_bf16 tokens")
    a = ap.parse_args()
    a.warmup = max(3, a.warmup)

    ws, rank, local = dist_env()
    if a.impl == "reference":
        return run_reference(a, ws, rank)

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if ws > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    peaks, peak_kind = load_peaks()
    w = make_workload(a.workload, ws, rank, device, exchange=a.exchange, batch=a.batch, tokens=a.tokens)
    rec = measure(w, a, device, ws, rank, local, peaks, peak_kind, not a.no_cpu_baseline)
    close = getattr(w, "close", None)
    if close is not None:
        close()
    del w
    torch.cuda.empty_cache()
    line = {"metric": rec.pop("metric"), "value": rec.pop("value"), "unit": rec.pop("unit"), "n_gpus": ws,
            "steps": a.steps, "warmup": a.warmup, **rec, "vs_baseline": None,
            "data": "synthetic (seeded N(0,1), reference benchmark shapes)"}
    if ws == 1 and not a.no_extra:
        # the other configurations of the reference's measurement plan, timed the same way in this run
        line["workloads"] = {}
        for name in EXTRA_WORKLOADS:
            if name == a.workload:
                continue
            wx = make_workload(name, ws, rank, device)
            rx = measure(wx, a, device, ws, rank, local, peaks, peak_kind, not a.no_cpu_baseline)
            if not a.no_reference_kernel:
                rk = reference_kernel_leg(wx, a, device)
                if "value" in rk:
                    rk["ours_over_reference"] = round(rx["roofline"]["achieved"] / rk["value"], 2)
                rx["reference_gpu_kernel"] = rk
            line["workloads"][name] = rx
            del wx
            torch.cuda.empty_cache()
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))


def run_reference(a, ws, rank):
    """Reference arm: the reference's own path for this hot path on the host CPU.

    The reference's naive PyTorch paged attention (restated in oracle/; the
    reference's Triton kernel needs a GPU build of the reference) runs on all
    host threads, one bounded sample of the workload per step.  Under torchrun
    only rank 0 runs it.
    """
    if rank != 0:
        return
    threads = os.cpu_count() or 1

    def timed(name, budget):
        w = make_workload(name, ws, rank, None, cpu_only=True)
        for _ in range(a.warmup):
            w.cpu_sample(0.0, threads)
        t_tot, done_tot, n_tot = 0.0, 0.0, 0
        for _ in range(a.steps):
            t, done, n = w.cpu_sample(budget, threads)
            t_tot, done_tot, n_tot = t_tot + t, done_tot + done, n_tot + n
        val = done_tot / t_tot * w.scale
        sample = f"{a.steps} steps of {budget * 1e3:.0f} ms: " + w.sample_desc(n_tot, t_tot)
        return {"impl": "reference", "metric": w.metric, "value": round(val, 4), "unit": w.unit, "n_gpus": ws,
                "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(t_tot / a.steps * 1e3, 3),
                "higher_is_better": True, "scaling": w.scaling, "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded N(0,1), reference benchmark shapes)",
                "config": {"workload": name, **w.info, "threads": threads},
                "cpu_baseline": {"value": round(val, 4), "unit": w.unit, "cores": threads, "kind": "port",
                                 "sample": sample},
                "e2e": {"value": round(val, 4), "unit": w.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}

    line = timed(a.workload, min(2.0, 120.0 / max(1, a.steps + a.warmup)))
    if ws == 1 and not a.no_extra:
        line["workloads"] = {n: timed(n, min(0.5, 30.0 / max(1, a.steps + a.warmup)))
                             for n in EXTRA_WORKLOADS if n != a.workload}
    print(json.dumps(line))


if __name__ == "__main__":
    main()
