"""Benchmark of the B200 paged-attention hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode_fp16|decode_int8|prefill_bf16|long_ctx_int8]

One step = one pass of the hot path over one batch of seeded synthetic input
with the reference's benchmark shapes (no public dataset is involved):

  decode_fp16   (default) paged decode attention, B=64, 32/8 heads, D=128,
                block_size 16, ctx ~ U[512, 4096], fp16 KV.  Metric: HBM GB/s of
                the algorithmic bytes (K/V of every attended token + Q + O).
  decode_int8   the same shape with INT8 KV (fp16 per-token scales, 1% outliers
                x8): quantise-on-write of 64 new tokens per sequence, then decode.
  prefill_bf16  causal paged prefill, B=8, L ~ U[1024, 4096], 32/8 heads, bf16;
                K/V written into scattered fp16 blocks, then attention.
                Metric: TFLOP/s (causal FLOPs).
  long_ctx_int8 B=256, 64/8 heads, ctx ~ U[8192, 32768], INT8 KV; KV heads are
                sharded across the N ranks and the per-head outputs gathered
                with an NCCL all-gather (strong scaling).

Decode workloads under torchrun run one batch per rank (seed + rank, weak
scaling, no collective).  Inputs exceed the 126 MB L2 for every workload; the
timed region is bracketed by barrier + synchronize, timed with CUDA events on
the launching stream, max over ranks.  ``--impl reference`` times the
reference's own path on the host CPU (the naive PyTorch paged attention,
restated in oracle/) on the same workload and prints the same JSON line.
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
def decode_workload(name: str, seed: int, device):
    """Build the decode batch (on `device`) and the per-step call."""
    from kernels.flash_attention import flash_attention_forward, write_kv_cache
    from pie_b200.workloads import config_batch

    b = config_batch(name, seed=seed)
    g = b.to(device)
    B, Hq, _, D = b.Q.shape
    Hkv = b.K.shape[2]
    sum_ctx = int(b.kv_len.long().sum())
    kv_bytes = sum_ctx * Hkv * b.kv_bytes_per_token_head
    qo_bytes = 2 * B * Hq * D * 2 + B * Hq * 2
    info = {"B": B, "Hq": Hq, "Hkv": Hkv, "D": D, "block_size": b.block_size, "sum_ctx": sum_ctx,
            "kv_dtype": str(b.K.dtype).replace("torch.", "")}
    write = None
    if name == "decode_int8":
        T_new = 64
        gen = torch.Generator().manual_seed(seed + 99)
        kn = (torch.randn(B * T_new, Hkv, D, generator=gen) *
              torch.where(torch.rand(B * T_new, Hkv, D, generator=gen) < 0.01, 8.0, 1.0)).half().to(device)
        vn = torch.randn(B * T_new, Hkv, D, generator=gen).half().to(device)
        seq = torch.arange(B, dtype=torch.int32).repeat_interleave(T_new).to(device)
        pos = (b.kv_len.view(-1, 1) - T_new + torch.arange(T_new).view(1, -1)).reshape(-1).to(torch.int32).to(device)
        write = (kn, vn, seq, pos)
        w_bytes = 2 * B * T_new * Hkv * (D * 2 + D + 2)
        info["new_tokens_per_seq"] = T_new
        kv_bytes += w_bytes

    def step(out=None):
        if write is not None:
            write_kv_cache(write[0], write[1], g.block_table, write[2], write[3], g.K, g.V, g.k_scale, g.v_scale)
        return flash_attention_forward(g.Q, g.K, g.V, g.q_len, g.block_table, g.num_blocks, g.block_size, g.kv_len,
                                       g.k_scale, g.v_scale, out=out)

    launches = 2 + (1 if write is not None else 0)
    return b, g, step, kv_bytes + qo_bytes, info, launches


def prefill_workload(seed: int, device):
    from kernels.flash_attention import flash_attention_forward, write_kv_cache
    from pie_b200.workloads import CONFIGS, block_tables, draw_context_lengths

    cfg = CONFIGS["prefill_bf16"]
    gen = torch.Generator().manual_seed(seed)
    L = draw_context_lengths(gen, cfg["B"], *cfg["ctx_range"])
    B, Hq, Hkv, D, BS = cfg["B"], cfg["Hq"], cfg["Hkv"], cfg["D"], cfg["BS"]
    bt, nblk, NB = block_tables(gen, L, BS)
    maxL = max(L)
    Q = torch.randn(B, Hq, maxL, D, generator=gen).to(torch.bfloat16)
    T = sum(L)
    kn = torch.randn(T, Hkv, D, generator=gen).to(torch.bfloat16)
    vn = torch.randn(T, Hkv, D, generator=gen).to(torch.bfloat16)
    seq = torch.cat([torch.full((l,), i, dtype=torch.int32) for i, l in enumerate(L)])
    pos = torch.cat([torch.arange(l, dtype=torch.int32) for l in L])
    d = lambda t: t.to(device)  # noqa: E731
    Qd, knd, vnd, seqd, posd, btd, nbd = map(d, (Q, kn, vn, seq, pos, bt, nblk))
    Ld = torch.tensor(L, dtype=torch.int32, device=device)
    Kc = torch.empty(NB, BS, Hkv, D, dtype=torch.float16, device=device)
    Vc = torch.empty_like(Kc)

    def step(out=None):
        write_kv_cache(knd, vnd, btd, seqd, posd, Kc, Vc)
        return flash_attention_forward(Qd, Kc, Vc, Ld, btd, nbd, BS, Ld, None, None, out=out)

    flops = sum(4.0 * Hq * D * l * (l + 1) / 2 for l in L)
    info = {"B": B, "Hq": Hq, "Hkv": Hkv, "D": D, "block_size": BS, "sum_len": T, "q_dtype": "bfloat16",
            "kv_dtype": "float16"}
    host = {"Q": Q, "kn": kn, "vn": vn, "seq": seq, "pos": pos, "bt": bt, "nblk": nblk, "L": torch.tensor(L)}
    return host, step, flops, info


# ----------------------------------------------------------------------------
# timing
# ----------------------------------------------------------------------------
def time_steps(step, steps: int, warmup: int, device, ws: int):
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
    for _ in range(steps):
        step()
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


def cpu_baseline_decode(b, seconds: float, threads: int):
    """The reference's naive paged attention (oracle restatement) on the host CPU."""
    from oracle import paged_attention as orc

    torch.set_num_threads(threads)
    Qn = b.Q.float().numpy()
    Kn, Vn = b.K.numpy(), b.V.numpy()
    ks = None if b.k_scale is None else b.k_scale.numpy()
    vs = None if b.v_scale is None else b.v_scale.numpy()
    meta = [t.numpy() for t in (b.q_len, b.block_table, b.num_blocks, b.kv_len)]
    B = Qn.shape[0]
    times, seqs_done, t_end = [], 0, time.perf_counter() + seconds
    i = 0
    while time.perf_counter() < t_end or not times:
        sl = slice(i % B, i % B + 1)
        t0 = time.perf_counter()
        orc.paged_attention(Qn[sl], Kn, Vn, meta[0][sl], meta[1][sl], meta[2][sl], b.block_size, meta[3][sl], ks, vs)
        times.append((time.perf_counter() - t0, int(meta[3][sl][0])))
        seqs_done += 1
        i += 1
    t = sum(x[0] for x in times)
    ctx = sum(x[1] for x in times)
    return t, ctx, seqs_done


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode_fp16",
                    choices=["decode_fp16", "decode_int8", "prefill_bf16", "long_ctx_int8"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    a = ap.parse_args()
    a.warmup = max(3, a.warmup)

    ws, rank, local = dist_env()
    if a.impl == "reference":
        return run_reference(a, ws, rank)
    if a.workload == "long_ctx_int8":
        from pie_b200.sharded import bench_long_ctx
        return bench_long_ctx(a, ws, rank, local)

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if ws > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=device)
    peaks, peak_kind = load_peaks()
    seed = 1000 + rank

    if a.workload == "prefill_bf16":
        host, step, work, info, launches = *prefill_workload(seed, device), 2
        unit, metric = "TFLOP/s", "causal paged prefill TFLOP/s (bf16, B=8, L~U[1024,4096], 32/8 heads, D=128)"
        scale = 1e-12
        bound, peak, punit = "tensor", peaks["bf16_tflops"], "TFLOP/s"
    else:
        b, g, step, work, info, launches = decode_workload(a.workload, seed, device)
        unit = "GB/s"
        metric = ("paged decode attention HBM GB/s (fp16 KV, B=64, 32/8 heads, D=128, ctx~U[512,4096])"
                  if a.workload == "decode_fp16" else
                  "paged decode attention + quantise-on-write HBM GB/s (INT8 KV, B=64, 32/8 heads, D=128)")
        scale = 1e-9
        bound, peak, punit = "hbm", peaks["hbm_gbs"], "GB/s"

    with ClockSampler(local) as clk:
        ms = time_steps(step, a.steps, a.warmup, device, ws)
    ms_step = ms / a.steps
    value = ws * work / (ms_step * 1e-3) * scale

    # e2e: host buffers in, result back to host, through the public API
    e2e = e2e_measure(a, step, device, ws, (b if a.workload != "prefill_bf16" else None),
                      (g if a.workload != "prefill_bf16" else None), work, scale)

    achieved = work / (ms_step * 1e-3) * scale
    traffic = read_traffic(f"{a.workload}_dominant_kernel")
    line = {
        "metric": metric, "value": round(value, 2), "unit": unit, "n_gpus": ws, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(ms_step, 5), "us_per_step": round(ms_step * 1e3, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16" if a.workload == "decode_fp16" else ("i8" if a.workload == "decode_int8" else "bf16"),
        "data": "synthetic (seeded N(0,1), reference benchmark shapes)",
        "config": {"workload": a.workload, **info, "parallelism": f"dp{ws} (one batch per rank)",
                   "l2": "inputs larger than L2 (126 MB)"},
        "roofline": {"bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": punit,
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "kernel": "paged_attn_decode (split + merge launches)" if bound == "hbm" else
                               "kv_write_copy + paged_attn_prefill", "peak_source": f"{peak_kind} MEASURED_PEAKS"},
        "e2e": e2e,
        "gpu_launches": launches * a.steps,
        "clocks": clk.summary(),
    }
    if rank == 0 and ws == 1 and not a.no_cpu_baseline and a.workload != "prefill_bf16":
        threads = os.cpu_count() or 1
        t, ctx, nseq = cpu_baseline_decode(b, a.cpu_seconds, threads)
        kvb = ctx * info["Hkv"] * b.kv_bytes_per_token_head
        line["cpu_baseline"] = {"value": round(kvb / t * 1e-9, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                                "sample": f"{nseq} sequences of the workload, one at a time, {t:.1f} s"}
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))


def e2e_measure(a, step, device, ws, b, g, work, scale):
    """Same metric through the public API with host-resident step inputs.

    Per step: pinned host -> device copy of the step's inputs (Q and the paging
    metadata; the KV pool is device-resident state), the call, and the
    device -> host copy of O.  Timed with CUDA events like the device number.
    """
    if b is None:
        return None
    from kernels.flash_attention import flash_attention_forward

    hQ = b.Q.pin_memory()
    hbt, hnb, hql, hkl = (t.pin_memory() for t in (b.block_table, b.num_blocks, b.q_len, b.kv_len))
    hO = torch.empty(b.Q.shape, dtype=torch.float16).pin_memory()
    dQ = torch.empty_like(g.Q)
    dbt, dnb, dql, dkl = (torch.empty_like(t) for t in (g.block_table, g.num_blocks, g.q_len, g.kv_len))
    h2d = sum(t.numel() * t.element_size() for t in (hQ, hbt, hnb, hql, hkl))
    d2h = hO.numel() * hO.element_size()

    def e2e_step():
        for h, d in ((hQ, dQ), (hbt, dbt), (hnb, dnb), (hql, dql), (hkl, dkl)):
            d.copy_(h, non_blocking=True)
        O, _ = flash_attention_forward(dQ, g.K, g.V, dql, dbt, dnb, g.block_size, dkl, g.k_scale, g.v_scale)
        hO.copy_(O, non_blocking=True)

    steps = max(10, a.steps // 10)
    ms = time_steps(e2e_step, steps, a.warmup, device, ws)
    val = ws * work / (ms / steps * 1e-3) * scale
    return {"value": round(val, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "steps": steps, "ms_per_step": round(ms / steps, 5)}


def run_reference(a, ws, rank):
    """Reference arm: the reference's CPU path (naive PyTorch paged attention) on the host."""
    if rank != 0:
        return
    from pie_b200.workloads import config_batch

    threads = os.cpu_count() or 1
    if a.workload in ("decode_fp16", "decode_int8"):
        b = config_batch(a.workload, seed=1000)
        ms_list, bytes_list = [], []
        for _ in range(a.warmup):
            cpu_baseline_decode(b, 0.0, threads)
        for _ in range(a.steps):
            t, ctx, n = cpu_baseline_decode(b, min(2.0, 120.0 / max(1, a.steps)), threads)
            ms_list.append(t)
            bytes_list.append(ctx * b.K.shape[2] * b.kv_bytes_per_token_head)
        t = sum(ms_list)
        val = sum(bytes_list) / t * 1e-9
        unit = "GB/s"
        metric = ("paged decode attention HBM GB/s (fp16 KV, B=64, 32/8 heads, D=128, ctx~U[512,4096])"
                  if a.workload == "decode_fp16" else
                  "paged decode attention + quantise-on-write HBM GB/s (INT8 KV, B=64, 32/8 heads, D=128)")
        sample = f"{a.steps} samples of whole sequences of the workload, {t:.1f} s total"
    else:
        print(json.dumps({"impl": "reference", "unavailable": f"reference CPU arm covers decode workloads only"}))
        return
    line = {"impl": "reference", "metric": metric, "value": round(val, 4), "unit": unit, "n_gpus": ws,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(t / a.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1), reference benchmark shapes)",
            "config": {"workload": a.workload, "threads": threads},
            "cpu_baseline": {"value": round(val, 4), "unit": unit, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": round(val, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


if __name__ == "__main__":
    main()
