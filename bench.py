#!/usr/bin/env python
"""Benchmark of the NVFP4 cached linear on B200 (one JSON line on rank 0).

Metric: cached-linear TFLOPS and % of the dense-FP4 peak at
M x N x K = 2048 x 2880 x 7680 (configs[1]; BF16 activations ~N(0,1), weights
~N(0,0.02) quantized once, bias ~N(0,0.01)), plus the standalone quantizer's
HBM GB/s on the config-4 tensor (16384 x 16384 Student-t stress input).

A step = one cached linear call: quantize the activations + block-scaled GEMM
with the fused bias, on inputs already in HBM.  One step's working set (55 MB)
fits in L2 (126 MB), so the timed loop rotates through enough independent
input/weight/output sets to move more than twice L2 per pass ("inputs larger
than L2"); K steps run back to back between one pair of CUDA events on the
launching stream (an event pair per step would add ~4 us of event overhead to
every step on this GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU (torchrun, one rank per GPU): the headline is data-parallel with
weak scaling -- every rank runs the full per-GPU workload on its own
activations, no collective on the data path; the reported value is all ranks'
FLOPs over the slowest rank's time.  The same line carries config 5 (the
decoder-layer linear stack, M = 8192) run in every mode on the same ranks:
"single" (each rank the whole stack alone: the 1-GPU time), "tp_p2p",
"tp_epilogue" and "tp_nccl" (weights N-sharded, output columns assembled on
every rank by copy-engine pushes over NVLink, by the GEMM epilogue's NVLink
stores, or by an NCCL all-gather), and "dp" (rows split), with strong-scaling efficiency, the bytes each rank receives per step
and a byte-for-byte check of a column-parallel linear against one GPU
(`tp_bytes_equal`).  `--impl reference` times the reference's CPU path (its
own quantizer compiled for the host + fp32 matmul of the dequantized
operands) on the host cores, on rank 0 only.

Roofline denominator for the GEMM and the step: the larger of NVIDIA's dense
NVFP4 figure (9 PFLOP/s) and the dense NVFP4 MMA rate measured in the same run
by fp4b_mma_rate (`--config fp4peak` prints that measurement alone, with the
GEMM mainloop's MMA mixes).
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
L2_BYTES = 126 * 1024 * 1024


def sets_needed(bytes_per_set: int) -> int:
    """Distinct buffer sets so that one pass over them moves more than twice L2."""
    return max(2, -(-2 * L2_BYTES // max(1, bytes_per_set)))


def time_rotating(fns, steps: int, warmup: int, stream=None) -> float:
    """Average device milliseconds per call of K back-to-back calls, call i
    using buffer set i % len(fns); the sets together exceed L2, so every call
    reads its inputs from HBM.  One CUDA-event pair brackets the K calls (an
    event pair per call would add ~4 us of event overhead to each), and the
    GPU is parked on a sleep while the host enqueues them."""
    stream = stream or torch.cuda.current_stream()
    for i in range(warmup):
        fns[i % len(fns)]()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        torch.cuda._sleep(int(2e6) * (steps + 10))
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(steps):
        fns[i % len(fns)]()
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


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


# ------------------------------------------------------------------------------ peak and roofline
def measured_fp4_peak() -> dict | None:
    """Dense NVFP4 MMA rate of this GPU (fp4b_mma_rate: N = 256, operands resident
    in shared memory, no loads), or None when the measurement fails."""
    import fp4_gemm
    try:
        return fp4_gemm.mma_rate(256, 0, False, 0, stages=8192, reps=5)
    except RuntimeError:
        return None


def fp4_roofline_peak(measured: dict | None) -> tuple[float, str]:
    """(denominator, its source): the larger of the 9 PF datasheet figure and the measured rate."""
    if measured and measured["tflops"] > FP4_DATASHEET_TFLOPS:
        return measured["tflops"], "dense NVFP4 MMA rate measured in this run (fp4b_mma_rate, N=256)"
    return FP4_DATASHEET_TFLOPS, "NVIDIA B200 dense NVFP4 datasheet (9 PFLOP/s; above the rate measured in this run)"


def roofline_entry(achieved: float, peak: float, peak_source: str, measured: dict | None, fp4_4x_bf16: float,
                   **extra) -> dict:
    d = {"bound": "tensor", **extra, "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
         "peak_source": peak_source, "frac_of_datasheet_9pf": achieved / FP4_DATASHEET_TFLOPS,
         "frac_of_4x_measured_bf16": achieved / fp4_4x_bf16}
    if measured:
        d["frac_of_measured_mma_peak"] = achieved / measured["tflops"]
    return d


# ------------------------------------------------------------------------------ config 5: decoder stack
STACK_LINEARS = (("qkv", 5120, 2880), ("o", 2880, 4096), ("gate_up", 15360, 2880), ("down", 2880, 7680))
STACK_M = 8192


def stack_flops(layers: int) -> float:
    return 2.0 * STACK_M * layers * sum(n * k for _, n, k in STACK_LINEARS)


def stack_weight(layer: int, j: int, dev) -> torch.Tensor:
    """Weight of linear j of a layer: N(0, 0.02) BF16, from a seed of its own
    (the same bytes on every rank and every GPU)."""
    _, n, k = STACK_LINEARS[j]
    g = torch.Generator(device=dev).manual_seed(1000 * layer + j)
    return (torch.randn(n, k, generator=g, device=dev) * 0.02).to(torch.bfloat16)


def stack_activations(dev, r0: int, r1: int) -> dict:
    """Fresh N(0,1) activations per input width (the stack's shapes do not chain); rows [r0, r1)."""
    g = torch.Generator(device=dev).manual_seed(7)
    return {k: torch.randn(STACK_M, k, generator=g, device=dev).to(torch.bfloat16)[r0:r1].contiguous()
            for k in sorted({k for _, _, k in STACK_LINEARS})}


def time_stack(mode: str, layers: int, steps: int, warmup: int, ws: int, rank: int, dev) -> float:
    """Milliseconds per stack step (max over ranks).  mode: "single" (this rank
    runs the whole stack alone), "dp" (rows split over the ranks), "tp_p2p" /
    "tp_epilogue" / "tp_nccl" (weights N-sharded, output columns assembled on
    every rank by copy-engine pushes, by the GEMM epilogue's stores, or by an
    NCCL all-gather)."""
    import torch.distributed as dist

    import fp4_gemm
    import fp4_gemm_dist as D
    r0, r1 = D.row_range(STACK_M, ws, rank) if mode == "dp" else (0, STACK_M)
    mods = []
    for li in range(layers):
        lin = []
        for j in range(len(STACK_LINEARS)):
            w = stack_weight(li, j, dev)
            if mode.startswith("tp"):
                lin.append(D.ColumnParallelFP4Linear(w, None, mode=mode[3:]))
            else:
                lin.append(fp4_gemm.FP4WeightCache(w))
            del w
        mods.append(lin)
    xs = stack_activations(dev, r0, r1)
    stream = torch.cuda.current_stream(dev)

    def step():
        for lin in mods:
            for mod, (_, _, k) in zip(lin, STACK_LINEARS):
                if mode.startswith("tp"):
                    mod.forward(xs[k])
                else:
                    mod.forward(xs[k], sync=False)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    if ws > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    for lin in mods:
        for mod in lin:
            mod.free()
    del mods, xs
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    return ms


def stack_recv_bytes(ws: int, layers: int) -> int:
    """Bytes of output columns the busiest receiver takes in per tensor-parallel step."""
    import fp4_gemm_dist as D
    total = 0
    for _, n, _ in STACK_LINEARS:
        shards = D.plan_column_shards(n, ws)
        total += STACK_M * (n - min(s.cols for s in shards)) * 2
    return total * layers


def tp_bytes_equal(ws: int, dev) -> bool:
    """One column-parallel linear (the stack's QKV shape, 2048 rows, BF16 bias),
    in both assembly modes, equals the single-GPU cache byte for byte on every rank."""
    import torch.distributed as dist

    import fp4_gemm
    import fp4_gemm_dist as D
    w = stack_weight(0, 0, dev)
    g = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn(2048, w.shape[1], generator=g, device=dev).to(torch.bfloat16)
    b = (torch.randn(w.shape[0], generator=g, device=dev) * 0.01).to(torch.bfloat16)
    single = fp4_gemm.FP4WeightCache(w, b)
    ref = single.forward(x, sync=True)
    ok = True
    for mode in ("p2p", "epilogue", "nccl"):
        tp = D.ColumnParallelFP4Linear(w, b, mode=mode)
        ok = ok and bool(torch.equal(tp.forward(x), ref))
        tp.free()
    single.free()
    flag = torch.tensor([1 if ok else 0], device=dev, dtype=torch.int32)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    return bool(flag.item())


def stack_report(args, ws: int, rank: int, dev) -> dict:
    """Config 5 in every mode that applies at this world size (see the module docstring)."""
    layers = args.layers
    flops = stack_flops(layers)
    modes = ["single"] + (["tp_p2p", "tp_epilogue", "tp_nccl", "dp"] if ws > 1 else [])
    out = {"workload": f"config 5: {layers} layers x (QKV 2880->5120, O 4096->2880, gate_up 2880->15360, "
                       f"down 7680->2880), M={STACK_M} tokens, weights N(0,0.02) cached as NVFP4, fresh N(0,1) "
                       "activations per linear (quantized every call), no bias",
           "tflop_per_step": flops / 1e12, "steps": args.steps, "warmup": args.warmup, "modes": {}}
    t_single = None
    for mode in modes:
        ms = time_stack(mode, layers, args.steps, args.warmup, ws, rank, dev)
        entry = {"ms_per_step": ms}
        if mode == "single":
            t_single = ms
            entry["tflops"] = flops / (ms * 1e-3) / 1e12
            entry["note"] = "every rank runs the whole stack on its own GPU; the 1-GPU time (max over ranks)"
        else:
            entry["tflops"] = flops / (ms * 1e-3) / 1e12
            entry["efficiency_vs_1gpu"] = t_single / (ws * ms)
            if mode.startswith("tp"):
                rb = stack_recv_bytes(ws, layers)
                entry["recv_bytes_per_step_per_rank"] = rb
                entry["nvlink_gbs_per_rank"] = rb / (ms * 1e-3) / 1e9
        out["modes"][mode] = entry
    if ws > 1:
        out["tp_bytes_equal"] = tp_bytes_equal(ws, dev)
    return out


# ------------------------------------------------------------------------------ our arm
def headline_sets(m, n, k, rank, dev):
    import fp4_gemm
    from tests import workloads as W
    per_set = m * k * 2 + (n + 64) * k * 9 // 16 + m * n * 2 + m * k * 9 // 16
    nsets = sets_needed(per_set)
    sets = []
    for i in range(nsets):
        x, w, b = W.cached_linear_inputs(m, n, k, seed=1000 * rank + i)
        xd, bd = x.to(dev), b.to(dev)
        cache = fp4_gemm.FP4WeightCache(w.to(dev), bd)
        out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        aq, asf = fp4_gemm.quantize_to_buffers(xd, None, cache.K)
        sets.append(dict(x=xd, b=bd, cache=cache, out=out, aq=aq, asf=asf, wsd=cache.state_dict()))
    return sets, per_set


def gemm_fn(lib, st, m, n, sptr):
    kp = st["cache"].K
    return lambda: lib.fp4b_gemm_prequant(st["aq"].data_ptr(), st["asf"].data_ptr(), m, st["aq"].shape[0],
                                          st["wsd"]["fp4"].data_ptr(), st["wsd"]["sf"].data_ptr(), n,
                                          st["cache"].N, kp, None, 0, st["out"].data_ptr(), n,
                                          st["b"].data_ptr(), 1.0, 0.0, sptr)


def run_ours(args):
    import datetime

    import torch.distributed as dist

    import fp4_gemm
    from tests import workloads as W

    ws, rank, local = dist_env()
    if ws > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=300))
    dev = torch.device("cuda", local if ws > 1 else 0)
    torch.cuda.set_device(dev)
    peaks = load_peaks()
    fp4_4x_bf16 = 4.0 * peaks["bf16_tflops"]
    lib = fp4_gemm._lib
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream
    clocks = ClockSampler(dev.index if ws == 1 else local)
    clocks.start()
    mma_peak = measured_fp4_peak()
    fp4_peak, fp4_peak_source = fp4_roofline_peak(mma_peak)

    # --- headline: cached linear 2048 x 2880 x 7680 + bias, buffer sets rotated past L2
    m, n, k = W.HEADLINE_SHAPE
    sets, per_set = headline_sets(m, n, k, rank, dev)
    nsets = len(sets)

    def make_step(st):
        def step():
            rc = lib.fp4b_run_cached_ex(st["x"].data_ptr(), m, k, k, st["cache"]._handle, n, None, 0,
                                        st["out"].data_ptr(), n, st["b"].data_ptr(), 1.0, 0.0, sptr)
            if rc != 0:
                raise RuntimeError(f"cached linear failed: {rc} {fp4_gemm._last_error()}")
        return step

    def make_quant(st):
        kp = st["cache"].K
        return lambda: lib.fp4b_quantize(st["x"].data_ptr(), m, k, k, st["aq"].data_ptr(), st["asf"].data_ptr(),
                                         st["aq"].shape[0], kp, sptr)

    steps_fns = [make_step(st) for st in sets]
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms_per_step = time_rotating(steps_fns, args.steps, args.warmup, stream)
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    gemm_ms = time_rotating([gemm_fn(lib, st, m, n, sptr) for st in sets], args.steps, args.warmup, stream)
    quant_ms = time_rotating([make_quant(st) for st in sets], args.steps, args.warmup, stream)

    if ws > 1:
        t = torch.tensor([ms_per_step], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_per_step = float(t.item())
    flops = 2.0 * m * n * k
    value = ws * flops / (ms_per_step * 1e-3) / 1e12
    gemm_tflops = flops / (gemm_ms * 1e-3) / 1e12
    step_tflops = flops / (ms_per_step * 1e-3) / 1e12
    aq0 = sets[0]["aq"]
    quant_bytes = m * k * 2 + aq0.shape[0] * aq0.shape[1] + aq0.shape[0] * aq0.shape[1] // 8
    tile = fp4_gemm.gemm_tile_width(m, n, k, torch.cuda.get_device_properties(dev).multi_processor_count)

    # --- config 5 on every rank (all modes that apply at this world size)
    stack = stack_report(args, ws, rank, dev)

    # --- end to end through the public API on every rank at once: pinned host in,
    # pinned host out, every step (FP4WeightCache.forward_host overlaps the row
    # chunks' copies with their GEMMs); the whole job's rate, max time over ranks
    x_host = W.cached_linear_inputs(m, n, k, seed=0)[0].pin_memory()
    y_host = torch.empty(m, n, dtype=torch.bfloat16).pin_memory()
    cache0 = sets[0]["cache"]

    def e2e_step():
        cache0.forward_host(x_host, out=y_host)
    if ws > 1:
        dist.barrier()
    e2e_ms = time_rotating([e2e_step], args.steps, args.warmup, stream)
    if ws > 1:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    result = None
    if rank == 0:
        # standalone quantizer, config 4 (input 512 MiB > L2)
        q4 = W.quantizer_stress(16384, 16384, seed=0).to(dev)
        q4_fp4 = torch.empty(16384, 8192, dtype=torch.uint8, device=dev)
        q4_sf = torch.empty(16384 * 1024, dtype=torch.uint8, device=dev)

        def quant4():
            lib.fp4b_quantize(q4.data_ptr(), 16384, 16384, 16384, q4_fp4.data_ptr(), q4_sf.data_ptr(), 16384,
                              16384, sptr)
        q4_ms = time_rotating([quant4], max(10, args.steps // 2), 3, stream)
        q4_bytes = 16384 * 16384 * (2 + 0.5 + 0.0625)
        q4_gbs = q4_bytes / (q4_ms * 1e-3) / 1e9
        del q4, q4_fp4, q4_sf

        # shape sweep of configs[1] (and config 1), cached linear with bias
        sweep = {}
        for (sm_, sn, sk) in [W.CFG1_SHAPE] + [sh for sh in W.CACHED_SHAPES if sh != W.HEADLINE_SHAPE]:
            sbytes = sm_ * sk * 2 + sn * sk * 9 // 16 + sm_ * sn * 2
            ssets = []
            for i in range(sets_needed(sbytes)):
                sx, sw, sb = W.cached_linear_inputs(sm_, sn, sk, seed=2000 + i)
                ssets.append((sx.to(dev), fp4_gemm.FP4WeightCache(sw.to(dev), sb.to(dev)), sb.to(dev),
                              torch.empty(sm_, sn, dtype=torch.bfloat16, device=dev)))

            def mk(t):
                sxd, sc, sbd, so = t
                return lambda: lib.fp4b_run_cached_ex(sxd.data_ptr(), sm_, sk, sk, sc._handle, sn, None, 0,
                                                      so.data_ptr(), sn, sbd.data_ptr(), 1.0, 0.0, sptr)
            sms_ = time_rotating([mk(t) for t in ssets], max(10, args.steps // 2), 3, stream)
            sweep[f"{sm_}x{sn}x{sk}"] = {"ms": sms_, "tflops": 2.0 * sm_ * sn * sk / (sms_ * 1e-3) / 1e12}
            for t in ssets:
                t[1].free()

        # config 3: dynamic matmul, both operands quantized every call (8192^3 and 16384^3)
        dynamic = {}
        for dn in (8192, 16384):
            g = torch.Generator(device=dev).manual_seed(3)
            da = torch.randn(dn, dn, generator=g, device=dev).to(torch.bfloat16)
            db = torch.randn(dn, dn, generator=g, device=dev).to(torch.bfloat16)
            dd = torch.empty(dn, dn, dtype=torch.bfloat16, device=dev)

            def dyn(da=da, db=db, dd=dd, dn=dn):
                rc = lib.fp4b_run_ex(da.data_ptr(), dn, dn, dn, db.data_ptr(), dn, dn, None, 0, dd.data_ptr(), dn,
                                     None, 1.0, 0.0, sptr)
                if rc != 0:
                    raise RuntimeError(f"dynamic matmul failed: {rc} {fp4_gemm._last_error()}")
            dms = time_rotating([dyn], max(3, args.steps // 10), 3, stream)
            dtf = 2.0 * dn ** 3 / (dms * 1e-3) / 1e12
            dynamic[f"{dn}^3"] = {"ms": dms, "tflops": dtf, "frac_of_roofline_peak": dtf / fp4_peak}
            del da, db, dd

    clk = clocks.stop()

    if rank == 0:
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
                       "l2": f"inputs larger than L2: {nsets} independent input/weight/output sets rotated "
                             f"({nsets * per_set / 2**20:.0f} MiB per pass), K steps back to back"},
            "pct_fp4_peak_datasheet": 100.0 * (value / ws) / FP4_DATASHEET_TFLOPS,
            "pct_fp4_peak_4x_measured_bf16": 100.0 * (value / ws) / fp4_4x_bf16,
            "measured_mma_peak": mma_peak,
            "kernels": {"quantize_activations_us": quant_ms * 1e3, "gemm_us": gemm_ms * 1e3,
                        "step_us": ms_per_step * 1e3,
                        "quantize_activations_gbs": quant_bytes / (quant_ms * 1e-3) / 1e9,
                        "quantize_activations_frac_hbm": quant_bytes / (quant_ms * 1e-3) / 1e9 / peaks["hbm_gbs"]},
            "roofline": roofline_entry(
                gemm_tflops, fp4_peak, fp4_peak_source, mma_peak, fp4_4x_bf16,
                kernel=f"nvf4_gemm_pair_kernel (2048x2880x7680, {tile}-wide CTA-pair tiles)", traffic=traffic),
            "roofline_step": roofline_entry(
                step_tflops, fp4_peak, fp4_peak_source, mma_peak, fp4_4x_bf16,
                what="whole cached-linear step: activation quantize + GEMM + fused bias, per GPU"),
            "quantize": {"workload": "config 4: 16384x16384 bf16 Student-t stress, bit-exact",
                         "value": q4_gbs, "unit": "GB/s", "ms": q4_ms,
                         "roofline": {"bound": "hbm", "achieved": q4_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                      "frac": q4_gbs / peaks["hbm_gbs"], "algorithmic_bytes": q4_bytes,
                                      "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peaks['source']})"}},
            "sweep": sweep,
            "dynamic": {"workload": "config 3: fp4_matmul path (quantize A and B, GEMM) per call, N(0,1) operands, "
                                    "inputs larger than L2", **dynamic},
            "stack": stack,
            "e2e": {"value": ws * flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOPS",
                    "h2d_bytes_per_step": ws * m * k * 2, "d2h_bytes_per_step": ws * m * n * 2,
                    "ms_per_step": e2e_ms,
                    "path": "fp4_gemm.FP4WeightCache.forward_host(pinned x, out=pinned y) on every rank at once: "
                            "512-row chunks, host-to-device copy / quantize+GEMM / device-to-host copy overlapped "
                            "on three streams; whole job, max time over ranks"},
            "gpu_launches": 2 * args.steps,
            "clocks": clk,
        }
        if cpu is not None:
            result["cpu_baseline"] = cpu
    for st in sets:
        st["cache"].free()
    if ws > 1:
        import fp4_gemm_dist as D
        D.PeerFlagBarrier.close_all()
        dist.barrier()
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)


def run_stack(args):
    """Config 5 alone (`--config stack`): every mode that applies at this world size, one JSON line."""
    import datetime

    import torch.distributed as dist

    ws, rank, local = dist_env()
    dev = torch.device("cuda", local if ws > 1 else 0)
    torch.cuda.set_device(dev)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    rep = stack_report(args, ws, rank, dev)
    if rank == 0:
        best = max(rep["modes"].values(), key=lambda e: e["tflops"])
        print(json.dumps({"metric": "decoder-stack TFLOPS (config 5)", "value": best["tflops"], "unit": "TFLOPS",
                          "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": best["ms_per_step"], "higher_is_better": True, "scaling": "strong",
                          "dtype": "nvfp4", "data": "synthetic", "stack": rep}), flush=True)
    if ws > 1:
        import fp4_gemm_dist as D
        D.PeerFlagBarrier.close_all()
        dist.barrier()
        dist.destroy_process_group()


def run_quantize(args):
    """Config 4 alone: the standalone quantizer on the 16384 x 16384 Student-t
    stress tensor (512 MiB in, inputs larger than L2), one JSON line.  The
    headline run reports the same figure under "quantize"; this entry point
    exists so that the kernel can be timed or profiled without the rest."""
    import fp4_gemm
    from tests import workloads as W

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = fp4_gemm._lib
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    q4 = W.quantizer_stress(16384, 16384, seed=0).to(dev)
    q4_fp4 = torch.empty(16384, 8192, dtype=torch.uint8, device=dev)
    q4_sf = torch.empty(16384 * 1024, dtype=torch.uint8, device=dev)

    def quant4():
        rc = lib.fp4b_quantize(q4.data_ptr(), 16384, 16384, 16384, q4_fp4.data_ptr(), q4_sf.data_ptr(), 16384,
                               16384, sptr)
        if rc != 0:
            raise RuntimeError(f"fp4b_quantize failed ({rc})")
    ms = time_rotating([quant4], args.steps, args.warmup, stream)
    nbytes = 16384 * 16384 * (2 + 0.5 + 0.0625)
    gbs = nbytes / (ms * 1e-3) / 1e9
    peaks = load_peaks()
    peak = peaks["hbm_gbs"]
    print(json.dumps({"metric": "quantize HBM GB/s (config 4)", "value": gbs, "unit": "GB/s", "n_gpus": 1,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                      "dtype": "bf16->nvfp4", "data": "synthetic",
                      "config": {"workload": "config 4: 16384x16384 bf16 Student-t stress, bit-exact",
                                 "l2": "input 512 MiB > L2"},
                      "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                                   "frac": gbs / peak, "algorithmic_bytes": nbytes,
                                   "peak_source": peaks["source"]},
                      "gpu_launches": args.steps}), flush=True)


def run_gemm(args):
    """One GEMM alone (`--config gemm`): the headline 2048 x 2880 x 7680 + bias,
    or `--shape MxNxK`, on operands quantized beforehand, buffer sets rotated
    past L2, one JSON line.  The command the GEMM's ncu captures run (one kernel
    per step, nothing else in the timed loop)."""
    import fp4_gemm
    from tests import workloads as W

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = fp4_gemm._lib
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    m, n, k = tuple(int(v) for v in args.shape.split("x")) if args.shape else W.HEADLINE_SHAPE
    sets, per_set = headline_sets(m, n, k, 0, dev)
    ms = time_rotating([gemm_fn(lib, st, m, n, sptr) for st in sets], args.steps, args.warmup, stream)
    tflops = 2.0 * m * n * k / (ms * 1e-3) / 1e12
    tile = fp4_gemm.gemm_tile_width(m, n, k, torch.cuda.get_device_properties(dev).multi_processor_count)
    what = "headline GEMM" if (m, n, k) == tuple(W.HEADLINE_SHAPE) else "GEMM"
    print(json.dumps({"metric": f"{what} TFLOPS ({m}x{n}x{k} + bias, operands pre-quantized)",
                      "value": tflops, "unit": "TFLOPS", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": ms, "higher_is_better": True, "dtype": "nvfp4", "data": "synthetic",
                      "config": {"workload": f"GEMM {m}x{n}x{k} + bias, {tile}-wide CTA-pair tiles",
                                 "l2": f"{len(sets)} buffer sets rotated ({len(sets) * per_set / 2**20:.0f} MiB)"},
                      "frac_of_datasheet_9pf": tflops / FP4_DATASHEET_TFLOPS,
                      "gpu_launches": args.steps}), flush=True)
    for st in sets:
        st["cache"].free()


# (n0, n1, scale copies, scale-B atoms per k-block): the dense peak, then the
# per-k-block MMA work of the GEMM's tile widths with and without their
# scale copies.
MMA_MIXES = [(256, 0, False, 0), (128, 0, False, 0), (192, 0, False, 0), (128, 192, False, 0),
             (192, 192, False, 0), (128, 0, True, 1), (192, 0, True, 2), (256, 0, True, 2), (128, 192, True, 3),
             (192, 192, True, 3), (128, 192, True, 2)]


def run_fp4peak(args):
    """`--config fp4peak`: the dense NVFP4 MMA rate of this GPU (the GEMM
    roofline's measured denominator) and the tensor-pipe rate of the GEMM
    mainloop's MMA mixes, operands resident in shared memory (no loads)."""
    import fp4_gemm
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    clocks = ClockSampler(0)
    clocks.start()
    mixes = {}
    for n0, n1, cp, atoms in MMA_MIXES:
        r = fp4_gemm.mma_rate(n0, n1, cp, atoms, stages=8192, reps=3)
        key = f"N={n0}" + (f"+{n1}" if n1 else "") + (f", {1 + atoms} scale copies per k-block" if cp else "")
        mixes[key] = {"tflops": r["tflops"], "ms": r["ms"], "pairs": r["pairs"]}
    clk = clocks.stop()
    peak = mixes["N=256"]["tflops"]
    print(json.dumps({"metric": "dense NVFP4 MMA rate (tcgen05.mma.cta_group::2.kind::mxf4nvf4.block16, M=256, "
                                "K=64, operands resident in shared memory)",
                      "value": peak, "unit": "TFLOP/s", "n_gpus": 1, "higher_is_better": True,
                      "frac_of_datasheet_9pf": peak / FP4_DATASHEET_TFLOPS, "mixes": mixes,
                      "gpu_launches": 4 * len(MMA_MIXES), "clocks": clk}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["headline", "stack", "quantize", "gemm", "fp4peak"], default="headline",
                    help="stack: config 5 decoder-layer linear stack; quantize: config 4 quantizer alone; gemm: "
                         "the headline GEMM alone; fp4peak: the measured NVFP4 MMA rate (none of these is the "
                         "headline metric)")
    ap.add_argument("--layers", type=int, default=12)
    ap.add_argument("--shape", default=None, help="--config gemm: MxNxK (default the headline 2048x2880x7680)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.config == "stack":
        run_stack(args)
    elif args.config == "quantize":
        run_quantize(args)
    elif args.config == "gemm":
        run_gemm(args)
    elif args.config == "fp4peak":
        run_fp4peak(args)
    elif args.impl == "reference":
        run_reference_arm(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
