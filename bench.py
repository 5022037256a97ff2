#!/usr/bin/env python3
"""Benchmark of the quantized-inference hot path (pplmx/nova cuda::quantize on B200).

Headline workload: dense FP8 E4M3 GEMM, M=N=K=4096,
A and B pre-quantized from fp32 ~N(0,1) with per-tensor scales amax/448, fp32
accumulation, bf16 output with the scales folded into the epilogue; B in the
reference's K x N layout (FP8GEMM::forward).  One step = one GEMM launch.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 (torchrun): every rank runs the same GEMM on its own GPU (replicas, no
collective on the data path); value = all ranks' FLOPs / max-over-ranks time.

Output: rank 0 prints the secondary workloads (quantize bandwidth sweep, C3,
C4) on a line of their own starting with "secondary ", then ONE JSON line
whose last key, "tp_mlp", times BASELINE configs[4] -- the tensor-parallel
FP8 SwiGLU MLP with tp = N (strong scaling, T = 16384 tokens at every N,
GEMM-fused bf16 all-reduce of the row-parallel output) -- with a parity check
of sampled output rows and, for N > 1, the tp = 1 time measured in the same
run on every GPU.
--impl reference times the reference algorithm on the host cores (the CPU
oracle port of FP8GEMM::forward's naive kernel, fp8_gemm.cu:64-86, on all
host threads), rank 0 only, plus the reference's own host code on one core.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M = N = K = 4096
FLOPS = 2.0 * M * N * K
L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2
METRIC = "FP8 GEMM TFLOPS (4096^3 E4M3, bf16 out)"


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def profile_traffic(name):
    """DRAM bytes per launch from the committed ncu summary, or None."""
    try:
        txt = open(os.path.join(ROOT, "profiles", name)).read()
    except OSError:
        return None
    m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", txt)
    return float(m.group(1)) if m else None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    def __init__(self, index, period=0.002):
        self.index, self.period = index, period
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._t = None

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nv = nv
            self.h = nv.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
        except Exception:
            self.nv = None
            return self
        names = {
            "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
            "hw_power_brake_slowdown": 0x80, "sw_power_cap": 0x4, "sync_boost": 0x10,
        }

        def run():
            while not self._stop.is_set():
                try:
                    self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                    r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                    for k, bit in names.items():
                        if r & bit:
                            self.reasons.add(k)
                except Exception:
                    pass
                time.sleep(self.period)

        self._t = threading.Thread(target=run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples),
                "source": "nvml"}


def dist_init(gpus):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def spin_up(fn, seconds):
    """Runs fn back to back for about `seconds` so that the clocks have left
    their idle state before anything is timed (an idle B200 sits at ~120 MHz
    SM clock, and a few launches after idle time memory-bound kernels at
    60-75% of the bandwidth they reach once the GPU is busy)."""
    import torch
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end:
        for _ in range(20):
            fn()
        torch.cuda.synchronize()


def make_operands(seed_a=2, seed_b=3):
    """A, B ~ N(0,1) quantized on the GPU with per-tensor amax/448 scales
    (nq_calibrate_quantize: amax -> scale -> OCP E4M3 codes)."""
    import torch
    import nova_b200.capi as nq
    s = torch.cuda.current_stream().cuda_stream
    out = []
    for seed in (seed_a, seed_b):
        g = torch.Generator(device="cuda").manual_seed(seed)
        x = torch.randn(M, K, device="cuda", generator=g)
        q = torch.empty(M * K, dtype=torch.uint8, device="cuda")
        sc = torch.empty(2, dtype=torch.float32, device="cuda")
        nq.calibrate_quantize(x.data_ptr(), nq.F32, q.data_ptr(), x.numel(), nq.E4M3, sc.data_ptr(), s)
        torch.cuda.synchronize()
        out.append((q, float(sc[1].item())))
        del x
    return out


def ref_host_lib():
    """The reference's own host code (pplmx/nova's fp8_types.hpp,
    quantize_tensor.hpp and quantize_ops.hpp compiled from the reference tree
    into oracle/_ref/libnova_ref_host.so by oracle/Makefile), or None."""
    import ctypes as C
    path = os.path.join(ROOT, "oracle", "_ref", "libnova_ref_host.so")
    if not os.path.exists(path):
        return None
    lib = C.CDLL(path)
    lib.ref_e4m3_encode_array.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t]
    lib.ref_e4m3_encode_array.restype = None
    lib.ref_from_float_int8.argtypes = [C.c_void_p, C.c_size_t, C.c_float, C.c_void_p, C.c_void_p]
    lib.ref_from_float_int8.restype = C.c_int
    lib.ref_quantized_matmul.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_float,
                                         C.c_float]
    lib.ref_quantized_matmul.restype = None
    return lib


def cpu_reference_host():
    """Times the reference's OWN host code on one core (single-threaded by
    construction): FP8E4M3(float) over an array (fp8_types.hpp:64-97, the loop
    of benchmark_fp8_roundtrip, benchmark.cpp:308-335),
    QuantizedTensor<int8_t>::FromFloat (quantize_tensor.hpp:160-191: amax and
    round-half-away quantize) and QuantizedMatmul::forward
    (quantize_ops.hpp:54-81) at the C1 shape and on row slices of the C4
    decode shape (scaled linearly to M = 16).  Bytes per element as the GPU
    kernels count them: quantize 5 B (4 read + 1 write); C4 K*N + M*K + 2*M*N
    + 4*(M+N)."""
    import ctypes as C
    import numpy as np
    lib = ref_host_lib()
    if lib is None:
        return {"unavailable": "oracle/_ref/libnova_ref_host.so not built (needs the pplmx/nova source tree)"}
    vp = lambda a: a.ctypes.data_as(C.c_void_p)
    rng = np.random.default_rng(13)
    res = []
    for n in (1 << 20, 56 << 20):
        x = rng.standard_normal(n, dtype=np.float32)
        q = np.empty(n, np.uint8)
        t0 = time.perf_counter()
        lib.ref_e4m3_encode_array(vp(x), vp(q), n)
        dt = time.perf_counter() - t0
        res.append({"code": "FP8E4M3(float) array encode", "n": n, "s": round(dt, 4),
                    "GB/s": round(5.0 * n / dt / 1e9, 3), "Melem/s": round(n / dt / 1e6, 1)})
        qi = np.empty(n, np.int8)
        sc = np.zeros(1, np.float32)
        t0 = time.perf_counter()
        lib.ref_from_float_int8(vp(x), n, 0.0, vp(qi), vp(sc))
        dt = time.perf_counter() - t0
        res.append({"code": "QuantizedTensor<int8_t>::FromFloat (amax + quantize)", "n": n, "s": round(dt, 4),
                    "GB/s": round(5.0 * n / dt / 1e9, 3), "Melem/s": round(n / dt / 1e6, 1)})
        del x, q, qi
    m, k, n = 128, 1024, 1024
    a = rng.integers(-127, 128, (m, k), dtype=np.int8)
    b = rng.integers(-127, 128, (k, n), dtype=np.int8)
    o = np.empty((m, n), np.int8)
    t0 = time.perf_counter()
    lib.ref_quantized_matmul(vp(a), vp(b), vp(o), m, k, n, 0.01, 0.01)
    dt = time.perf_counter() - t0
    res.append({"code": "QuantizedMatmul::forward", "shape": [m, k, n], "s": round(dt, 4),
                "GOP/s": round(2.0 * m * k * n / dt / 1e9, 3)})
    kd, nd, rows = 8192, 28672, 1                                 # BASELINE configs[3], M = 16 scaled from 1 row
    a = rng.integers(-127, 128, (rows, kd), dtype=np.int8)
    b = rng.integers(-127, 128, (kd, nd), dtype=np.int8)
    o = np.empty((rows, nd), np.int8)
    t0 = time.perf_counter()
    lib.ref_quantized_matmul(vp(a), vp(b), vp(o), rows, kd, nd, 0.01, 0.01)
    dt = time.perf_counter() - t0
    t16 = dt * 16 / rows
    c4_bytes = kd * nd + 16 * kd + 2 * 16 * nd + 4 * (16 + nd)
    res.append({"code": "QuantizedMatmul::forward", "shape": [16, kd, nd], "sample_rows": rows,
                "s_scaled_to_m16": round(t16, 3), "GB/s": round(c4_bytes / t16 / 1e9, 4),
                "GOP/s": round(2.0 * 16 * kd * nd / t16 / 1e9, 3)})
    return {"cores": 1, "kind": "reference", "host_nproc": os.cpu_count(), "results": res}


def cpu_reference_sample(rows, threads):
    """Times the oracle port of the reference FP8 GEMM (naive kernel order,
    compat decode, fp32 FMA) on `rows` rows of the 4096^3 problem."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib as O
    rng = np.random.default_rng(0)
    a = rng.integers(0, 256, (rows, K), dtype=np.uint8)
    b = rng.integers(0, 256, (K, N), dtype=np.uint8)
    c = np.empty((rows, N), np.float32)
    t0 = time.perf_counter()
    used = O.lib.orc_fp8_gemm_reference_rows_mt(O.ptr(a), O.ptr(b), O.ptr(c), rows, K, N, 1.0, 1.0, 1.0, 0, rows,
                                                threads)
    dt = time.perf_counter() - t0
    return dt, used


def cpu_baseline(target_s=8.0):
    """The headline metric on ONE host core: the oracle port of the
    reference's FP8GEMM::forward (its naive kernel's order, decode and FMA,
    fp8_gemm.cu:64-86; the reference has no host FP8 GEMM of its own) on a
    row slice of the 4096^3 problem, plus the reference's own host code
    (cpu_reference_host) for the quantize and INT8 GEMM paths."""
    dt, used = cpu_reference_sample(4, 1)                       # calibration
    rate = (2.0 * 4 * N * K) / dt
    rows = int(max(4, min(M, target_s * rate / (2.0 * N * K))))
    dt, used = cpu_reference_sample(rows, 1)
    tflops = 2.0 * rows * N * K / dt / 1e12
    return {"value": tflops, "unit": "TFLOP/s", "cores": used, "kind": "port",
            "sample": f"{rows} of 4096 rows of the 4096^3 FP8 GEMM (naive reference order, 1 thread), {dt:.1f} s",
            "reference_host_code": cpu_reference_host()}


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    rows = max(threads, 8)
    for _ in range(args.warmup):
        cpu_reference_sample(rows, threads)
    times = []
    used = threads
    for _ in range(args.steps):
        dt, used = cpu_reference_sample(rows, threads)
        times.append(dt)
    per_step = sum(times) / len(times)
    tflops = 2.0 * rows * N * K / per_step / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": tflops, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "e4m3 in, fp32 accumulate", "data": "synthetic",
        "config": {"workload": "fp8_gemm_4096 (BASELINE configs[1]), host sample", "m": M, "n": N, "k": K,
                   "rows_per_step": rows},
        "cpu_baseline": {"value": tflops, "unit": "TFLOP/s", "cores": used, "kind": "port",
                         "sample": f"{rows} of 4096 rows per step (oracle port of fp8_gemm.cu:64-86)",
                         "reference_host_code": cpu_reference_host()},
        "e2e": {"value": tflops, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch
    world, rank, local = dist_init(args.gpus)
    import nova_b200.capi as nq
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    (qa, sa), (qb, sb) = make_operands()
    alpha = float(__import__("numpy").float32(sa) * __import__("numpy").float32(sb))
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    desc = nq.make_desc(M, N, K, nq.E4M3, nq.E4M3, nq.B_KN, nq.BF16, alpha)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")

    def gemm():
        nq.gemm(desc, qa.data_ptr(), qb.data_ptr(), out.data_ptr(), sh)

    spin_up(lambda: (flush.zero_(), gemm()), 0.3)
    for _ in range(args.warmup):
        flush.zero_()
        gemm()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        r0.record(stream)
        for i in range(args.steps):
            flush.zero_()                     # L2 flush between timed launches
            starts[i].record(stream)
            gemm()
            ends[i].record(stream)
        r1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    launch_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    mean_ms = sum(launch_ms) / len(launch_ms)
    region_ms = r0.elapsed_time(r1)
    mean_ms_max = max_over_ranks(mean_ms, world)
    value = world * FLOPS / (mean_ms_max * 1e-3) / 1e12
    assert nq.device_error_flags() == 0, "a kernel reported a timed-out wait"

    # ---- end to end through the C ABI with host buffers -------------------
    # Every step uploads its A and B from pinned host memory, runs the GEMM and
    # downloads its bf16 C, as a serving pipeline does: uploads on one copy
    # stream, downloads on another, two buffer sets, so step i+1's upload and
    # step i-1's download overlap step i's GEMM (each buffer is rewritten only
    # after the step that last used it is done with it).
    ha = torch.empty(M * K, dtype=torch.uint8, pin_memory=True)
    hb = torch.empty(K * N, dtype=torch.uint8, pin_memory=True)
    ha.copy_(qa.cpu())
    hb.copy_(qb.cpu())
    bufs = [(torch.empty_like(qa), torch.empty_like(qb), torch.empty_like(out),
             torch.empty(M, N, dtype=torch.bfloat16, pin_memory=True)) for _ in range(2)]
    s_up, s_down = torch.cuda.Stream(), torch.cuda.Stream()
    ev = {k: [torch.cuda.Event() for _ in range(2)] for k in ("up", "gemm", "down")}
    e2e_steps = max(3, min(args.steps, 50))

    def e2e_step(i):
        j = i % 2
        da, db, dc, hc = bufs[j]
        with torch.cuda.stream(s_up):
            if i >= 2:
                s_up.wait_event(ev["gemm"][j])        # step i-2's GEMM has read da, db
            da.copy_(ha, non_blocking=True)
            db.copy_(hb, non_blocking=True)
            ev["up"][j].record(s_up)
        stream.wait_event(ev["up"][j])
        if i >= 2:
            stream.wait_event(ev["down"][j])          # step i-2's download has read dc
        nq.gemm(desc, da.data_ptr(), db.data_ptr(), dc.data_ptr(), sh)
        ev["gemm"][j].record(stream)
        with torch.cuda.stream(s_down):
            s_down.wait_event(ev["gemm"][j])
            hc.copy_(dc, non_blocking=True)
            ev["down"][j].record(s_down)

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_up)
    for i in range(e2e_steps):
        e2e_step(i)
    e1.record(s_down)                                 # after the last download, which follows everything
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps, world)
    e2e_value = world * FLOPS / (e2e_ms * 1e-3) / 1e12
    del bufs, flush
    torch.cuda.empty_cache()
    tp_res = None
    if not args.no_tp_mlp:
        # a failure of the secondary TP block must not cost the headline line
        try:
            tp_res = tp_mlp_bench(world, rank, max(3, min(args.steps, 10)), args.warmup if args.warmup < 5 else 5,
                                  chunks=args.tp_chunks, overlap=args.tp_overlap, allreduce=args.tp_allreduce)
        except Exception as e:  # reported in the JSON line instead
            tp_res = {"error": f"{type(e).__name__}: {e}"[:300]}
            torch.cuda.synchronize()

    if rank != 0:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return 0
    pk = peaks()
    fp8_peak = 2.0 * pk["bf16_tflops"]
    achieved = FLOPS / (mean_ms * 1e-3) / 1e12
    traffic = profile_traffic("fp8_gemm_4096.md")
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": mean_ms_max, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "e4m3 in, fp32 accumulate, bf16 out", "data": "synthetic",
        "config": {"workload": "fp8_gemm_4096 (BASELINE configs[1])", "m": M, "n": N, "k": K,
                   "b_layout": "K x N row-major (FP8GEMM::forward)", "parallelism": f"replicas x{world}",
                   "l2": "256 MiB buffer written between timed launches", "timed_region_ms": region_ms},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": fp8_peak, "unit": "TFLOP/s",
                     "frac": achieved / fp8_peak, "traffic": traffic,
                     "peak_source": f"2 x bf16_tflops of MEASURED_PEAKS.json ({pk['source']}): dense FP8 = 2x dense bf16 on B200"},
        "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": 2 * M * K,
                "d2h_bytes_per_step": 2 * M * N,
                "path": "nq_gemm C ABI, pinned host A/B in, bf16 C out; uploads, GEMMs and downloads of "
                        "consecutive steps overlap on three streams (two buffer sets)"},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    if args.cublas:
        line["library_comparison"] = cublaslt_fp8(args.steps, args.warmup,
                                                  torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda"))
    if not args.no_secondary:
        # printed on a line of its own before the result line, which it would
        # otherwise push out of the tail of the log a reader keeps
        sizes = tuple(int(v) for v in args.sweep_sizes.split(","))
        try:
            sec = {"quantize_hbm": quantize_sweep(pk["hbm_gbs"], sizes, args.sweep_reps), **c3_c4_bench(pk)}
        except Exception as e:  # reported, the headline line still prints
            sec = {"error": f"{type(e).__name__}: {e}"[:300]}
        print("secondary " + json.dumps(sec), flush=True)
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline()
    if tp_res is not None:
        line["tp_mlp"] = tp_res          # last key: the sharded workload closes the line
    print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def quantize_sweep(hbm_gbs, sizes=(1 << 20, 56 << 20, 224 << 20), reps=None):
    """HBM-bound kernels of the path at the sweep sizes (fp32 input ~N(0,1)).
    Algorithmic bytes: quantize 5 B/elem (4 read + 1 write), amax 4 B/elem,
    calibrate+quantize 5 B/elem compulsory (9 B/elem as two passes), dequant
    5 B/elem, bf16 per-token quantize 3 B/elem + 4 B/row."""
    import torch
    import nova_b200.capi as nq
    s = torch.cuda.current_stream().cuda_stream
    out = []
    for n in sizes:
        x = torch.randn(n, device="cuda")
        q = torch.empty(n, dtype=torch.uint8, device="cuda")
        y = torch.empty(n, device="cuda")
        sc = torch.empty(2, device="cuda")
        nq.amax_scale_async(x.data_ptr(), nq.F32, n, nq.E4M3, sc.data_ptr(), s)
        cols = 4096
        rows = n // cols
        xb = x[: rows * cols].view(rows, cols).to(torch.bfloat16)
        rs = torch.empty(rows, device="cuda")
        cases = [
            ("quantize_f32_to_e4m3 (device scale)", 5.0, lambda: nq.quantize_scaled(x.data_ptr(), nq.F32, q.data_ptr(), n, nq.E4M3, sc.data_ptr() + 4, s)),
            ("quantize_f32_to_int8 (reference API)", 5.0, lambda: nq.quantize_f32_to_int8(x.data_ptr(), q.data_ptr(), n, 0.02, 0.0, 1, s)),
            ("quantize_f32_to_fp8e4m3 (reference codec)", 5.0, lambda: nq.quantize_f32_to_fp8e4m3(x.data_ptr(), q.data_ptr(), n, s)),
            ("amax+scale", 4.0, lambda: nq.amax_scale_async(x.data_ptr(), nq.F32, n, nq.E4M3, sc.data_ptr(), s)),
            ("calibrate+quantize (2 launches)", 5.0, lambda: nq.calibrate_quantize(x.data_ptr(), nq.F32, q.data_ptr(), n, nq.E4M3, sc.data_ptr(), s)),
            ("dequantize_int8_to_f32", 5.0, lambda: nq.dequantize_int8_to_f32(q.data_ptr(), y.data_ptr(), n, 0.02, 0.0, 1, s)),
            ("per-token quantize bf16 -> e4m3 (4096 cols)", 3.0, lambda: nq.quantize_rows(xb.data_ptr(), nq.BF16, q.data_ptr(), rs.data_ptr(), rows, cols, nq.E4M3, s)),
        ]
        for name, bpe, fn in cases:
            spin_up(fn, 0.02)
            nrep = reps if reps else (20 if n <= (64 << 20) else 10)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            for _ in range(nrep):
                fn()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / nrep
            gbs = bpe * n / (ms * 1e-3) / 1e9
            out.append({"kernel": name, "n": n, "us": round(ms * 1e3, 2), "GB/s": round(gbs, 1),
                        "frac_hbm": round(gbs / hbm_gbs, 3)})
        del x, q, y, xb
    return out


def _time_flushed(fn, reps, flush):
    """Mean CUDA-event time (ms) of fn(); with `flush` an L2 flush (a 256 MiB
    write) precedes each launch, without it the inputs must exceed L2.  All
    launches are enqueued back to back (one synchronize at the end), so the
    GPU never idles between them."""
    import torch
    fl = (lambda: flush.zero_()) if flush is not None else (lambda: None)
    spin_up(lambda: (fl(), fn()), 0.02)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for e0, e1 in evs:
        fl()
        e0.record()
        fn()
        e1.record()
    torch.cuda.synchronize()
    return sum(e0.elapsed_time(e1) for e0, e1 in evs) / reps


def _time_batch(fn, reps):
    """Mean CUDA-event time (ms) of `reps` launches of fn() enqueued back to
    back between one pair of events (inputs larger than L2, no flush)."""
    import torch
    spin_up(fn, 0.02)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def c3_c4_bench(pk, reps=20, c3=True, c4_ms=(16, 64, 256)):
    """BASELINE configs[2] and [3] on one GPU.
    C3, W8A8 FP8 MLP up-projection: X 8192 x 4096 bf16 ~N(0,1) with 41 of
    4096 channels x20; W 4096 x 14336 ~N(0,0.02), per-output-channel E4M3
    (nq_quantize_cols); per-token E4M3 quantize of X (nq_quantize_rows) then
    the GEMM with row/col scales in the epilogue, bf16 out: 9.621e11 flop.
    C4, decode INT8 W8A8: W 28672 x 8192 (N x K) int8 per-channel, X M x 8192
    int8 per-token, int32 accumulation, bf16 out; bytes = K*N + M*K + 2*M*N +
    4*(M+N).  C3 launches follow an L2 flush (256 MiB write); C4 streams 224 MiB
    of weights, larger than the 126 MB L2, and is timed without a flush (the
    write-back of a write-flush's dirty lines would be charged to the kernel),
    as the mean of `reps` back-to-back launches between one pair of events, as a
    decode step issues them (a pair of events around every launch adds about
    2 us of idle GPU per launch, reported beside it)."""
    import torch
    import nova_b200.capi as nq
    s = torch.cuda.current_stream().cuda_stream
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    fp8_peak = 2.0 * pk["bf16_tflops"]
    res = {}
    g = torch.Generator(device="cuda").manual_seed(4)
    if c3:
        Mx, Kx, Nx = 8192, 4096, 14336
        x = torch.randn(Mx, Kx, device="cuda", generator=g)
        out_ch = torch.randperm(Kx, generator=torch.Generator().manual_seed(5))[:41].cuda()
        x[:, out_ch] *= 20.0
        x = x.to(torch.bfloat16)
        w = torch.randn(Kx, Nx, device="cuda", generator=g).mul_(0.02)
        wq = torch.empty(Kx, Nx, dtype=torch.uint8, device="cuda")
        ws = torch.empty(Nx, device="cuda")
        nq.quantize_cols(w.data_ptr(), wq.data_ptr(), ws.data_ptr(), Kx, Nx, nq.E4M3, s)
        del w
        xq = torch.empty(Mx, Kx, dtype=torch.uint8, device="cuda")
        xs = torch.empty(Mx, device="cuda")
        y = torch.empty(Mx, Nx, dtype=torch.bfloat16, device="cuda")
        d = nq.make_desc(Mx, Nx, Kx, nq.E4M3, nq.E4M3, nq.B_KN, nq.BF16, 1.0, xs.data_ptr(), ws.data_ptr(), 0)
        quant = lambda: nq.quantize_rows(x.data_ptr(), nq.BF16, xq.data_ptr(), xs.data_ptr(), Mx, Kx, nq.E4M3, s)
        gemm = lambda: nq.gemm(d, xq.data_ptr(), wq.data_ptr(), y.data_ptr(), s)
        dq = nq.make_desc(Mx, Nx, Kx, nq.E4M3, nq.E4M3, nq.B_KN, nq.BF16, 1.0, 0, ws.data_ptr(), 0)
        fused = lambda: nq.gemm_quant_a(dq, x.data_ptr(), xq.data_ptr(), xs.data_ptr(), wq.data_ptr(), y.data_ptr(), s)
        flop = 2.0 * Mx * Nx * Kx
        # the variants alternate (3 rounds, best of each), so that clock and power
        # drift over the run does not favour the one measured first
        t_q = t_g = t_all = t_f = float("inf")
        for _ in range(3):
            t_f = min(t_f, _time_flushed(fused, reps, flush))
            t_all = min(t_all, _time_flushed(lambda: (quant(), gemm()), reps, flush))
            t_q = min(t_q, _time_flushed(quant, reps, flush))
            t_g = min(t_g, _time_flushed(gemm, reps, flush))
        res["c3_w8a8_up_proj"] = {
            "m": Mx, "k": Kx, "n": Nx,
            "layer_us": round(t_f * 1e3, 1), "layer_tflops": round(flop / (t_f * 1e-3) / 1e12, 1),
            "layer_frac_fp8_peak": round(flop / (t_f * 1e-3) / 1e12 / fp8_peak, 3),
            "layer": "nq_gemm_quant_a: per-token quantize fused into the GEMM, one kernel",
            "two_launch_layer_us": round(t_all * 1e3, 1), "per_token_quant_us": round(t_q * 1e3, 1),
            "per_token_quant_GBps": round((3 * Mx * Kx + 4 * Mx) / (t_q * 1e-3) / 1e9, 1),
            "gemm_only_us": round(t_g * 1e3, 1), "gemm_only_tflops": round(flop / (t_g * 1e-3) / 1e12, 1)}
        del x, xq, y, wq
        torch.cuda.empty_cache()
    Kd, Nd = 8192, 28672
    wi = torch.randint(-127, 128, (Nd, Kd), dtype=torch.int8, device="cuda", generator=g)
    sw = torch.rand(Nd, device="cuda", generator=g).mul_(1e-3)
    c4 = []
    for Md in c4_ms:
        xi = torch.randint(-127, 128, (Md, Kd), dtype=torch.int8, device="cuda", generator=g)
        sx = torch.rand(Md, device="cuda", generator=g).mul_(1e-2)
        yo = torch.empty(Md, Nd, dtype=torch.bfloat16, device="cuda")
        dd = nq.make_desc(Md, Nd, Kd, nq.INT8, nq.INT8, nq.B_NK, nq.BF16, 1.0, sx.data_ptr(), sw.data_ptr(), 0)
        fn = lambda: nq.gemm(dd, xi.data_ptr(), wi.data_ptr(), yo.data_ptr(), s)
        t_ev = _time_flushed(fn, reps, None)
        t = min(_time_batch(fn, reps) for _ in range(3))
        byts = Kd * Nd + Md * Kd + 2 * Md * Nd + 4 * (Md + Nd)
        gbs = byts / (t * 1e-3) / 1e9
        c4.append({"m": Md, "us": round(t * 1e3, 1), "GB/s": round(gbs, 1), "frac_hbm": round(gbs / pk["hbm_gbs"], 3),
                   "tops": round(2.0 * Md * Nd * Kd / (t * 1e-3) / 1e12, 1),
                   "us_events_around_each_launch": round(t_ev * 1e3, 1)})
    res["c4_decode_int8"] = c4
    del wi, flush
    torch.cuda.empty_cache()
    assert nq.device_error_flags() == 0
    return res


def _time_mlp(mlp, x, out, T, steps, warmup, world):
    """max-over-ranks CUDA-event ms per forward of `steps` forwards."""
    import torch
    for _ in range(max(warmup, 5)):
        mlp.forward(x, out, 1, T, sync=False)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        mlp.forward(x, out, 1, T, sync=False)
    e1.record(stream)
    torch.cuda.synchronize()
    return max_over_ranks(e0.elapsed_time(e1) / steps, world)


def tp_parity(mlp, x, y, shards, rows, world, group=None):
    """Parity of sampled output rows of the TP MLP, every rank taking part.

    (a) From the GPU's own FP8 codes and scales:
      - the per-token codes and scales of x and of h, re-derived in torch from
        x and from the GPU's h (same multiply by 448 / amax, RNE E4M3), are
        bit-identical;
      - h within the FP8 bar of tests/test_tp_gpu.py (max relative error
        1e-2, |ref| floored at 1e-2 rms) of fp64 sums of the decoded codes;
      - each rank's bf16 partial (the symmetric partial buffer of the fused
        all-reduce; the output itself at tp = 1) within the same bar of an
        fp64 product of the GPU's h codes with the down shard;
      - tp > 1: the reduced output is one bf16 rounding of the exact sum of
        the ranks' partials (max error 2^-8 of |sum|, floored at 1e-2 rms);
        through NVSwitch multicast the switch converts its fp32 sum to bf16
        itself, within one bf16 ulp (2 x 2^-8) rather than half of one.
    (b) Against an fp32 computation with the UNQUANTIZED weights
        (tensor_parallel_layers.cpp:561-579 in fp32): normwise relative error
        below 0.1 (two E4M3 quantizations of activations and weights, about
        2^-4 / sqrt(3) relative noise each).
    Also: every rank's sampled output rows bit-identical (replicated) and the
    device error word clear on every rank."""
    import torch
    import torch.distributed as dist
    import nova_b200.capi as nq
    f8 = torch.float8_e4m3fn
    T = x.shape[0]
    idx = torch.tensor(rows, device="cuda")

    def token_codes(v):
        """nq_quantize_rows' arithmetic on fp32 rows: (codes, scales).  Both
        divisions are tensor / tensor: torch evaluates tensor / scalar and
        scalar / tensor with a reciprocal (two roundings), the kernel with
        one IEEE division."""
        amax = v.abs().amax(dim=1)
        q = torch.full_like(amax, 448.0)
        scale = torch.where(amax > 0, amax / q, torch.ones_like(amax))
        inv = torch.where(amax > 0, q / amax, torch.ones_like(amax))
        ok = torch.isfinite(inv)
        c = torch.where(ok[:, None], v * inv[:, None], v / scale[:, None])
        return c.to(f8), scale

    def rel(got, ref, mag=None):
        mag = ref.abs() if mag is None else mag
        floor = 1e-2 * torch.sqrt(torch.mean(mag * mag)) + 1e-30
        return float(torch.max(torch.abs(got - ref) / torch.maximum(mag, floor)))

    gu, dl = mlp.gate_up, mlp.down.lin
    xq, sx = gu._ws[T]
    hq, sh = dl._ws[T]
    xc, xs = token_codes(x[idx].float())
    hc, hs = token_codes(mlp._h[T][idx].float())
    codes_ok = (torch.equal(xc.view(torch.uint8), xq[idx]) and torch.equal(xs, sx[idx]) and
                torch.equal(hc.view(torch.uint8), hq[idx]) and torch.equal(hs, sh[idx]))
    # gate/up: packed [g_0 | u_0 | g_1 | ...] blocks of 128 columns
    acc = xq[idx].view(f8).double() @ gu.q.view(f8).double()
    gv = (acc * sx[idx].double()[:, None] * gu.s.double()[None, :]).view(len(rows), -1, 2, 128)
    g, u = gv[:, :, 0, :].reshape(len(rows), -1), gv[:, :, 1, :].reshape(len(rows), -1)
    h_err = rel(mlp._h[T][idx].double(), (g / (1.0 + torch.exp(-g))) * u)
    part_ref = (hq[idx].view(f8).double() @ dl.q.view(f8).double()) * sh[idx].double()[:, None] * dl.s.double()[None, :]
    fused = mlp.down.fused
    got = y[idx].double()
    sum_bound = 2.0 if (fused is not None and fused.multicast()) else 1.0
    if world == 1:
        part_err, sum_err = rel(got, part_ref), 0.0
    elif fused is not None:
        st = fused.state(T, mlp.H, mlp._bounds(T))
        part_gpu = st.partial[idx].double()
        part_err = rel(part_gpu, part_ref)
        total, mag = part_gpu.clone(), part_gpu.abs()
        dist.all_reduce(total, group=group)
        dist.all_reduce(mag, group=group)
        sum_err = rel(got, total, mag) / 2.0 ** -8
    else:   # NCCL all-reduce: no partial buffer; the sum of the references, two roundings apart
        part_err = 0.0
        total, mag = part_ref.to(torch.bfloat16).double(), part_ref.abs()
        dist.all_reduce(total, group=group)
        dist.all_reduce(mag, group=group)
        sum_err = rel(got, total, mag) / (2.0 ** -7 + 2.0 ** -8)
    # (b) fp32 with the unquantized weight shards
    wg, wu, wd = shards
    xf = x[idx].float()
    gf, uf = xf @ wg, xf @ wu
    p32 = ((gf / (1.0 + torch.exp(-gf))) * uf) @ wd
    if world > 1:
        dist.all_reduce(p32, group=group)
    fp32_norm = float(torch.linalg.norm(got - p32.double()) / torch.linalg.norm(p32.double()))
    # every rank: replicated rows, device errors, worst errors
    mx, mn = y[idx].float().clone(), y[idx].float().clone()
    worst = torch.tensor([float(nq.device_error_flags()), 0.0 if codes_ok else 1.0, h_err, part_err, sum_err],
                         device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
        dist.all_reduce(mn, op=dist.ReduceOp.MIN, group=group)
        dist.all_reduce(worst, op=dist.ReduceOp.MAX, group=group)
    replicated = bool(torch.equal(mx, mn))
    dev_err, codes_ok = int(worst[0].item()), worst[1].item() == 0.0
    h_err, part_err, sum_err = (float(v) for v in worst[2:].tolist())
    ok = (codes_ok and h_err <= 1e-2 and part_err <= 1e-2 and sum_err <= sum_bound and fp32_norm <= 0.1
          and replicated and dev_err == 0)
    return {"ok": ok, "rows": len(rows), "codes_bit_exact": codes_ok, "h_max_rel_err": round(h_err, 6),
            "partial_max_rel_err": round(part_err, 6), "sum_err_in_bf16_roundings": round(sum_err, 4),
            "sum_err_bound": sum_bound,
            "vs_fp32_weights_norm_err": round(fp32_norm, 5), "replicated": replicated, "device_errors": dev_err}


def tp_mlp_bench(world, rank, steps, warmup, T=16384, H=8192, I=28672, chunks=None, overlap="full", allreduce="auto",
                 parity_rows=64):
    """the FP8 SwiGLU MLP (nova_b200.tp.TensorParallelMLP)
    with tp = world size, T tokens per step (strong scaling: the same T at
    every tp).  x ~ N(0,1) bf16, weights ~ N(0,0.02) fp32 generated on the
    device from fixed seeds (identical on every rank), sharded and FP8
    quantized by set_weight.  One step = forward() (per-token quantize,
    gate/up GEMM + SwiGLU, quantize, down GEMM, all-reduce); time = max over
    ranks of the CUDA-event time of `steps` forwards.  Inputs (256 MiB) and
    weights exceed L2.  allreduce "auto" / "nvls" / "p2p": the down GEMM and
    the all-reduce are one kernel (nq_gemm_allreduce) and forward returns the
    symmetric output buffer; "nccl": chunked GEMM + torch.distributed
    all_reduce into `out`.  With tp > 1, every GPU then also runs the whole
    MLP alone (tp = 1, a one-rank group each, all GPUs at once) for the
    strong-scaling reference measured in the same run."""
    import torch
    import torch.distributed as dist
    from nova_b200.tp import TensorParallelMLP, shard_columns, shard_rows
    g = torch.Generator(device="cuda").manual_seed(11)
    mlp = TensorParallelMLP(H, I, chunks=chunks, overlap=overlap, allreduce=allreduce)
    wg = torch.randn(H, I, device="cuda", generator=g).mul_(0.02)
    wu = torch.randn(H, I, device="cuda", generator=g).mul_(0.02)
    wd = torch.randn(I, H, device="cuda", generator=g).mul_(0.02)
    mlp.set_weight(wg, wu, wd)
    shards = (shard_columns(wg, rank, world).contiguous(), shard_columns(wu, rank, world).contiguous(),
              shard_rows(wd, rank, world).contiguous())
    x = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
    fused = mlp.down.fused is not None
    out = None if fused else torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    ms = _time_mlp(mlp, x, out, T, steps, warmup, world)
    flops = 6.0 * T * H * I
    pk = peaks()
    fp8_peak = 2.0 * pk["bf16_tflops"]
    tflops = flops / (ms * 1e-3) / 1e12
    res = {"workload": "tp_fp8_swiglu_mlp (BASELINE configs[4])", "tokens": T, "hidden": H, "intermediate": I,
           "tp": world, "allreduce": (("fused-nvls" if mlp.down.fused.multicast() else "fused-p2p") if fused
                                      else ("nccl" if world > 1 else "none")),
           "chunks": mlp.chunks, "ms_per_step": round(ms, 4), "tokens_per_s": round(T / (ms * 1e-3)),
           "tflops_total": round(tflops, 1), "frac_of_tp_x_fp8_peak": round(tflops / (world * fp8_peak), 4),
           # a forward is milliseconds of back-to-back GEMMs under the 1 kW power cap:
           # its roofline is the sustained figure (2 x sustained bf16 of MEASURED_PEAKS.json)
           "frac_of_tp_x_fp8_sustained": round(tflops / (world * 2.0 * pk["bf16_tflops_sustained"]), 4),
           "allreduce_bytes": 2 * T * H if world > 1 else 0, "scaling": "strong"}
    # parity of sampled rows spread over every token chunk, from one more forward
    y = mlp.forward(x, out, 1, T, sync=True)
    rows = sorted(set(int(v) for v in torch.linspace(0, T - 1, parity_rows).round().tolist()))
    try:
        res["parity"] = tp_parity(mlp, x, y, shards, rows, world)
    except Exception as e:  # reported in the line
        res["parity"] = {"ok": False, "error": f"{type(e).__name__}: {e}"[:200]}
    del mlp, out, y, shards
    torch.cuda.empty_cache()
    if world > 1:
        # tp = 1 on every GPU at once (one-rank groups), same inputs and weights
        groups = [dist.new_group([r]) for r in range(world)]
        solo = TensorParallelMLP(H, I, group=groups[rank])
        solo.set_weight(wg, wu, wd)
        o1 = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
        ms1 = _time_mlp(solo, x, o1, T, steps, warmup, world)
        res["tp1_ms_per_step_same_run"] = round(ms1, 4)
        res["strong_scaling_vs_tp1"] = round(ms1 / (world * ms), 4)
        del solo, o1
    del wg, wu, wd, x
    torch.cuda.empty_cache()
    return res


def cublaslt_fp8(steps, warmup, flush):
    """cuBLASLt FP8 (torch._scaled_mm, e4m3 x e4m3 -> bf16, per-tensor scales)
    on the same shape, timed the same way: the library number to beat, and at
    8192^3 the practical dense FP8 ceiling of the part."""
    import torch
    res = {}
    for size in (4096, 8192):
        a = torch.randn(size, size, device="cuda").to(torch.float8_e4m3fn)
        b = torch.randn(size, size, device="cuda").to(torch.float8_e4m3fn).t()  # column-major B
        one = torch.ones((), device="cuda")
        f = lambda: torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        for _ in range(warmup):
            f()
        ts = []
        for _ in range(max(10, steps // 4)):
            flush.zero_()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            f()
            s1.record()
            torch.cuda.synchronize()
            ts.append(s0.elapsed_time(s1))
        ms = sum(ts) / len(ts)
        res[f"cublaslt_fp8_{size}_tflops"] = 2.0 * size ** 3 / (ms * 1e-3) / 1e12
        del a, b
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cublas", action="store_true", help="also time cuBLASLt FP8 on the same shape")
    ap.add_argument("--no-secondary", action="store_true", help="skip the quantize bandwidth sweep")
    ap.add_argument("--no-tp-mlp", action="store_true", help="skip the TP SwiGLU MLP (configs[4]) block")
    ap.add_argument("--tp-chunks", type=int, default=None, help="token chunks of the TP pipeline (default: by tp)")
    ap.add_argument("--tp-overlap", choices=["full", "down"], default="full")
    ap.add_argument("--tp-allreduce", choices=["auto", "nvls", "p2p", "nccl"], default="auto")
    ap.add_argument("--c4-m", default="16,64,256", help="decode token counts of the c4 workload")
    ap.add_argument("--only", choices=["all", "gemm", "sweep", "c3c4", "c4"], default="all",
                    help="gemm: the headline GEMM line alone; sweep / c3c4 / c4: one secondary workload alone")
    ap.add_argument("--sweep-sizes", default="1048576,58720256,234881024")
    ap.add_argument("--sweep-reps", type=int, default=0)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.only in ("sweep", "c3c4", "c4"):
        # one secondary workload alone (a small, self-contained command for ncu captures)
        import torch
        torch.cuda.set_device(0)
        pk = peaks()
        if args.only == "sweep":
            sizes = tuple(int(v) for v in args.sweep_sizes.split(","))
            res = quantize_sweep(pk["hbm_gbs"], sizes, args.sweep_reps)
        else:
            res = c3_c4_bench(pk, c3=args.only == "c3c4", c4_ms=tuple(int(v) for v in args.c4_m.split(",")))
        print(json.dumps({"only": args.only, "result": res}), flush=True)
        return 0
    if args.only == "gemm":
        args.no_secondary = args.no_tp_mlp = args.no_cpu_baseline = True
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
