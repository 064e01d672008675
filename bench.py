#!/usr/bin/env python
"""Benchmark of the NVFP4 cached linear on B200 (one JSON line on rank 0).

Metric: cached-linear TFLOPS and % of the dense-FP4 peak at
M x N x K = 2048 x 2880 x 7680 (configs[1]; BF16 activations ~N(0,1), weights
~N(0,0.02) quantized once, bias ~N(0,0.01)), plus the standalone quantizer's
HBM GB/s on the config-4 tensor (16384 x 16384 Student-t stress input).

A step = one cached linear call: quantize the activations + block-scaled GEMM
with the fused bias, on inputs already in HBM.  L2 (126 MB > the 55 MB
working set) is flushed by writing a 256 MiB buffer before every timed step;
each step is timed alone with CUDA events on the launching stream.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU (torchrun, one rank per GPU): data-parallel M-split with weak
scaling -- every rank runs the full per-GPU workload on its own activations,
no collective on the data path; the reported value is all ranks' FLOPs over
the slowest rank's time.  `--impl reference` times the reference's CPU path
(its own quantizer compiled for the host + fp32 matmul of the dequantized
operands) on the host cores, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "fp4-gemm-blackwell_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "cached-linear TFLOPS & % dense-FP4 peak @2048x2880x7680; quantize HBM GB/s"
FP4_DATASHEET_TFLOPS = 9000.0   # B200 dense FP4 (NVIDIA datasheet; 18 PF is with 2:4 sparsity)
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
PUBLISHED_GB10_TFLOPS = 129.0   # reference README.md:17, DGX Spark GB10, same metric and shape


def load_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS, "source": "fallback"}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks/throttle sampling in the background during timed regions."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.2)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(s):
            try:
                return float(s)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1])]
        mx = [num(r[2]) for r in rows if num(r[2])]
        pw = [num(r[3]) for r in rows if num(r[3])]
        loaded = [s for s, p in zip(sm, pw) if p and p > 250] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(pw) if pw else None, "samples": len(rows), "reasons": reasons}


# ------------------------------------------------------------------------------ timing
class L2Flusher:
    def __init__(self, dev, mib: int = 256):
        self.buf = torch.empty(mib * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def __call__(self):
        self.buf.fill_(1.0)


def time_launches(fn, steps: int, warmup: int, flush=None, stream=None) -> list[float]:
    """Per-call device milliseconds (CUDA events on `stream`), L2 flushed before each."""
    stream = stream or torch.cuda.current_stream()
    for _ in range(warmup):
        if flush:
            flush()
        fn()
    torch.cuda.synchronize()
    times = []
    pairs = []
    for _ in range(steps):
        if flush:
            flush()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        fn()
        e.record(stream)
        pairs.append((s, e))
    torch.cuda.synchronize()
    for s, e in pairs:
        times.append(s.elapsed_time(e))
    return times


# ------------------------------------------------------------------------------ CPU reference path
def cpu_reference_step(x_bits, w_dq, bias, rows: int):
    """The reference's path on the host: its quantizer (oracle/_ref when built, else
    the C restatement), dequantize, fp32 matmul (+ bias).  Returns fp32 [rows, N]."""
    from oracle import nvfp4_oracle as O
    xs = x_bits[:rows]
    k_pad = w_dq.shape[1]
    m_pad = O.round_up(rows, 128)
    padded = torch.zeros(m_pad, k_pad, dtype=torch.int16).numpy().view("uint16")
    padded[:rows, :xs.shape[1]] = xs
    if O.ref_available():
        q, s = O.ref_quantize(padded)
    else:
        q, s = O.quantize(padded)
    a = torch.from_numpy(O.dequantize(q, s, m_pad, k_pad))[:rows]
    out = a @ w_dq.t()
    if bias is not None:
        out = out.to(torch.bfloat16).float() + bias.float()
    return out


def cpu_baseline(m, n, k, target_s: float = 15.0) -> dict:
    from oracle import nvfp4_oracle as O
    from tests import workloads as W
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    x, w, b = W.cached_linear_inputs(m, n, k, seed=0)
    n_pad, k_pad = O.round_up(n, 128), O.round_up(k, 128)
    wq, ws = O.quantize(O.bf16_bits(w), n_pad, k_pad)
    w_dq = torch.from_numpy(O.dequantize(wq, ws, n_pad, k_pad))[:n]
    x_bits = O.bf16_bits(x)
    rows = min(m, 256)
    t0 = time.perf_counter()
    cpu_reference_step(x_bits, w_dq, b, rows)
    dt = time.perf_counter() - t0
    rows = max(128, min(m, int(rows * max(1.0, 2.0 / max(dt, 1e-3)))))  # ~2 s per repetition
    reps, elapsed = 0, 0.0
    while elapsed < target_s and reps < 50:
        t0 = time.perf_counter()
        cpu_reference_step(x_bits, w_dq, b, rows)
        elapsed += time.perf_counter() - t0
        reps += 1
    tflops = 2.0 * rows * n * k * reps / elapsed / 1e12
    return {"value": tflops, "unit": "TFLOPS", "cores": threads,
            "kind": "reference" if O.ref_available() else "port",
            "sample": f"{reps} x {rows} of {m} rows at {m}x{n}x{k}: reference quantizer on the host "
                      f"(oracle/_ref) + dequantize + torch fp32 mm + bias, {elapsed:.1f} s"}


def run_reference_arm(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    from oracle import nvfp4_oracle as O
    from tests import workloads as W
    m, n, k = W.HEADLINE_SHAPE
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    x, w, b = W.cached_linear_inputs(m, n, k, seed=0)
    n_pad, k_pad = O.round_up(n, 128), O.round_up(k, 128)
    wq, wsf = O.quantize(O.bf16_bits(w), n_pad, k_pad)
    w_dq = torch.from_numpy(O.dequantize(wq, wsf, n_pad, k_pad))[:n]
    x_bits = O.bf16_bits(x)
    # Size each step so that warmup + steps take about a minute.
    t0 = time.perf_counter()
    cpu_reference_step(x_bits, w_dq, b, 128)
    per_row = (time.perf_counter() - t0) / 128
    budget = 60.0 / max(1, args.steps + args.warmup)
    rows = int(max(128, min(m, budget / max(per_row, 1e-9))) // 128 * 128) or 128
    for _ in range(args.warmup):
        cpu_reference_step(x_bits, w_dq, b, rows)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cpu_reference_step(x_bits, w_dq, b, rows)
        times.append(time.perf_counter() - t0)
    t = sum(times) / len(times)
    tflops = 2.0 * rows * n * k / t / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": tflops, "unit": "TFLOPS", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"cached-linear {m}x{n}x{k} + bias on host CPU (sample {rows} rows per step)",
                   "parallelism": "host threads"},
        "cpu_baseline": {"value": tflops, "unit": "TFLOPS", "cores": threads,
                         "kind": "reference" if O.ref_available() else "port",
                         "sample": f"{rows} of {m} rows per step; reference quantizer (oracle/_ref) + "
                                   f"dequantize + torch fp32 mm + bias"},
        "e2e": {"value": tflops, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------ our arm
def run_ours(args):
    import torch.distributed as dist

    import fp4_gemm
    from tests import workloads as W

    ws, rank, local = dist_env()
    if ws > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=300))
    dev = torch.device("cuda", local if ws > 1 else 0)
    torch.cuda.set_device(dev)
    peaks = load_peaks()
    fp4_peak = 4.0 * peaks["bf16_tflops"]

    m, n, k = W.HEADLINE_SHAPE
    x, w, b = W.cached_linear_inputs(m, n, k, seed=rank)
    xd, wd, bd = x.to(dev), w.to(dev), b.to(dev)
    cache = fp4_gemm.FP4WeightCache(wd, bd)
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    flush = L2Flusher(dev)
    lib = fp4_gemm._lib
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream

    def step():
        rc = lib.fp4b_run_cached_ex(xd.data_ptr(), m, k, k, cache._handle, n, None, 0, out.data_ptr(), n,
                                    bd.data_ptr(), 1.0, 0.0, sptr)
        if rc != 0:
            raise RuntimeError(f"cached linear failed: {rc} {fp4_gemm._last_error()}")

    # kernel-level pieces for the roofline: quantize of A alone, GEMM alone
    k_pad = cache.K
    aq, asf = fp4_gemm.quantize_to_buffers(xd, None, k_pad)
    wsd = cache.state_dict()

    def quant_only():
        lib.fp4b_quantize(xd.data_ptr(), m, k, k, aq.data_ptr(), asf.data_ptr(), aq.shape[0], k_pad, sptr)

    def gemm_only():
        lib.fp4b_gemm_prequant(aq.data_ptr(), asf.data_ptr(), m, aq.shape[0], wsd["fp4"].data_ptr(),
                               wsd["sf"].data_ptr(), n, cache.N, k_pad, None, 0, out.data_ptr(), n, bd.data_ptr(),
                               1.0, 0.0, sptr)

    clocks = ClockSampler(dev.index if ws == 1 else local)
    clocks.start()
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    step_ms = time_launches(step, args.steps, args.warmup, flush, stream)
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    gemm_ms = time_launches(gemm_only, args.steps, args.warmup, flush, stream)
    quant_ms = time_launches(quant_only, args.steps, args.warmup, flush, stream)
    clk = clocks.stop()

    total_step_ms = sum(step_ms)
    if ws > 1:
        t = torch.tensor([total_step_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_step_ms = float(t.item())
    ms_per_step = total_step_ms / args.steps
    flops = 2.0 * m * n * k
    value = ws * flops / (ms_per_step * 1e-3) / 1e12

    gemm_avg = sum(gemm_ms) / len(gemm_ms)
    quant_avg = sum(quant_ms) / len(quant_ms)
    gemm_tflops = flops / (gemm_avg * 1e-3) / 1e12
    quant_bytes = m * k * 2 + aq.shape[0] * k_pad // 2 + aq.shape[0] * k_pad // 16

    result = None
    if rank == 0:
        # standalone quantizer, config 4 (input 512 MiB > L2, no flush needed)
        q4 = W.quantizer_stress(16384, 16384, seed=0).to(dev)
        q4_fp4 = torch.empty(16384, 8192, dtype=torch.uint8, device=dev)
        q4_sf = torch.empty(16384 * 1024, dtype=torch.uint8, device=dev)

        def quant4():
            lib.fp4b_quantize(q4.data_ptr(), 16384, 16384, 16384, q4_fp4.data_ptr(), q4_sf.data_ptr(), 16384,
                              16384, sptr)
        q4_ms = time_launches(quant4, max(10, args.steps // 2), 3, None, stream)
        q4_bytes = 16384 * 16384 * (2 + 0.5 + 0.0625)
        q4_gbs = q4_bytes / (statistics.mean(q4_ms) * 1e-3) / 1e9
        del q4, q4_fp4, q4_sf

        # shape sweep of configs[1] (and config 1), cached linear with bias
        sweep = {}
        for (sm_, sn, sk) in [W.CFG1_SHAPE] + [s for s in W.CACHED_SHAPES if s != W.HEADLINE_SHAPE]:
            sx, sw, sb = W.cached_linear_inputs(sm_, sn, sk, seed=1)
            sxd, sbd = sx.to(dev), sb.to(dev)
            sc = fp4_gemm.FP4WeightCache(sw.to(dev), sbd)
            so = torch.empty(sm_, sn, dtype=torch.bfloat16, device=dev)

            def sstep():
                lib.fp4b_run_cached_ex(sxd.data_ptr(), sm_, sk, sk, sc._handle, sn, None, 0, so.data_ptr(), sn,
                                       sbd.data_ptr(), 1.0, 0.0, sptr)
            st = time_launches(sstep, max(10, args.steps // 2), 3, flush, stream)
            ms = statistics.mean(st)
            sweep[f"{sm_}x{sn}x{sk}"] = {"ms": ms, "tflops": 2.0 * sm_ * sn * sk / (ms * 1e-3) / 1e12}
            sc.free()

        # end to end through the public API: pinned host in, pinned host out
        x_host = x.pin_memory()
        y_host = torch.empty(m, n, dtype=torch.bfloat16).pin_memory()

        def e2e_step():
            xg = x_host.to(dev, non_blocking=True)
            y = cache.forward(xg, sync=False)
            y_host.copy_(y, non_blocking=True)
        e2e_ms = time_launches(e2e_step, args.steps, args.warmup, flush, stream)
        e2e_avg = statistics.mean(e2e_ms)

        cpu = cpu_baseline(m, n, k) if ws == 1 else None
        traffic = None
        tp = os.path.join(ROOT, "profiles", "roofline_traffic.json")
        if os.path.exists(tp):
            traffic = json.load(open(tp)).get("gemm_2048x2880x7680_bytes_per_launch")
        result = {
            "metric": METRIC,
            "value": value,
            "unit": "TFLOPS",
            "n_gpus": ws,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": value / PUBLISHED_GB10_TFLOPS,
            "vs_baseline_note": "reference's published 129 TFLOPS for this shape is on DGX Spark GB10 (README.md:17)",
            "dtype": "nvfp4",
            "data": "synthetic",
            "config": {"workload": f"cached-linear {m}x{n}x{k} + bias (configs[1]); quantize activations + "
                                   "tcgen05 block-scaled GEMM per step, weights quantized once",
                       "M": m, "N": n, "K": k, "parallelism": f"dp{ws} (M-split, no collective)",
                       "l2": "flushed (256 MiB write) before every timed step"},
            "pct_fp4_peak_datasheet": 100.0 * value / FP4_DATASHEET_TFLOPS,
            "pct_fp4_peak_4x_measured_bf16": 100.0 * (value / ws) / fp4_peak,
            "kernels": {"quantize_activations_us": quant_avg * 1e3, "gemm_us": gemm_avg * 1e3,
                        "step_us": ms_per_step * 1e3, "quantize_activations_gbs": quant_bytes / (quant_avg * 1e-3) / 1e9},
            "roofline": {"bound": "tensor", "kernel": "nvf4_gemm_kernel (2048x2880x7680)",
                         "achieved": gemm_tflops, "peak": fp4_peak, "unit": "TFLOP/s",
                         "frac": gemm_tflops / fp4_peak, "traffic": traffic,
                         "peak_source": f"4 x bf16 dense burst ({peaks['source']}, MEASURED_PEAKS.json): "
                                        "B200 dense FP4 = 4 x dense BF16",
                         "frac_of_datasheet_9pf": gemm_tflops / FP4_DATASHEET_TFLOPS},
            "quantize": {"workload": "config 4: 16384x16384 bf16 Student-t stress, bit-exact",
                         "value": q4_gbs, "unit": "GB/s", "ms": statistics.mean(q4_ms),
                         "roofline": {"bound": "hbm", "achieved": q4_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                      "frac": q4_gbs / peaks["hbm_gbs"],
                                      "algorithmic_bytes": q4_bytes}},
            "sweep": sweep,
            "e2e": {"value": flops / (e2e_avg * 1e-3) / 1e12, "unit": "TFLOPS",
                    "h2d_bytes_per_step": m * k * 2, "d2h_bytes_per_step": m * n * 2,
                    "path": "fp4_gemm.FP4WeightCache.forward(sync=False) with pinned host in/out copies"},
            "gpu_launches": 2 * args.steps,
            "clocks": clk,
        }
        if cpu is not None:
            result["cpu_baseline"] = cpu
    cache.free()
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        run_reference_arm(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
