#!/usr/bin/env python
"""Benchmark of the NVFP4 data path (prints ONE JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (metric "NVFP4 GEMM TFLOPS"): the cfg3 block-scaled GEMM M=N=K=8192 on each GPU,
operands quantized on the device from seeded synthetic bf16 (A ~ N(0,1) with 0.1 % x50
outliers, B ~ N(0, 0.02)).  One step = one GEMM launch; L2 is flushed (256 MB write) between
timed steps; steps are timed with CUDA events on the launching stream and the max over ranks
is taken.  With N > 1 every rank runs its own GEMM (replicas, weak scaling) and the line also
carries the cfg4 NVFP4 all-reduce (bf16-equivalent bus bandwidth) when the all-reduce module
is built.  Extra keys: the cfg2 quantizer (GB/s), the roofline of the GEMM kernel, the CPU
baseline, the end-to-end number through the C ABI with host buffers, and SM clocks sampled
during the timed region.

--impl reference times the reference's own CPU implementation of the GEMM
(cpu_gemm_ref_bs from random_cpu_ref/verify_random.h, compiled into oracle/_ref) on a bounded
sample with all host threads, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M_ = N_ = K_ = 8192
FLUSH_BYTES = 256 << 20          # > 126 MB L2
PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
FP4_NOMINAL_TFLOPS = 9000.0       # B200 dense FP4 (NVIDIA spec, without sparsity)
HBM_FALLBACK_GBS = 6650.0
BF16_FALLBACK_TFLOPS = 1590.0


def load_peaks():
    try:
        with open(PEAKS_PATH) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return {"hbm_gbs": HBM_FALLBACK_GBS, "bf16_tflops": BF16_FALLBACK_TFLOPS}, "fallback"


# --------------------------------------------------------------- clocks ----
REASON_BITS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clocks_setting"}


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled through NVML (read
    only) every 5 ms while the timed region runs."""

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.samples = []
        self.stop_flag = threading.Event()
        self.thread = None
        self.err = None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            entry = vis.split(",")[self.idx].strip() if vis else str(self.idx)
            if entry.startswith("GPU-") or entry.startswith("MIG-"):
                self.h = pynvml.nvmlDeviceGetHandleByUUID(entry)
            else:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(int(entry))
            self.nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as e:
            self.err = str(e)
            return
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()

    def _run(self):
        n = self.nvml
        while not self.stop_flag.is_set():
            try:
                mhz = n.nvmlDeviceGetClockInfo(self.h, n.NVML_CLOCK_SM)
                try:
                    bits = n.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                except AttributeError:
                    bits = n.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                self.samples.append((mhz, bits))
            except Exception as e:
                self.err = str(e)
            time.sleep(0.005)

    def stop(self):
        if self.thread is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [f"nvml unavailable: {self.err}"]}
        self.stop_flag.set()
        self.thread.join(timeout=2)
        sm = sorted(s[0] for s in self.samples)
        reasons = set()
        for _, bits in self.samples:
            for b, name in REASON_BITS.items():
                if bits & b and name != "gpu_idle":
                    reasons.add(name)
        med = sm[len(sm) // 2] if sm else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ distributed ----
def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("NCCL_DEBUG", "WARN")     # keep NCCL's banner off stdout (one JSON line)
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------- GEMM ----
def gemm_setup(nv, rank):
    import torch
    from tensorcore_ptx_example_b200 import workloads
    a = workloads.activations(M_, K_, seed=3 + 17 * rank)
    b = workloads.gaussian(N_, K_, seed=4 + 17 * rank, std=0.02)
    pa, sa, gsa = nv.quantize(a, None)
    pb, sb, gsb = nv.quantize(b, None)
    torch.cuda.synchronize()
    del a, b
    alpha = float(gsa.item()) * float(gsb.item())
    d = torch.empty((M_, N_), dtype=torch.bfloat16, device="cuda")
    return pa, sa, pb, sb, alpha, d


class L2Flush:
    """Between timed steps: write a 256 MB buffer (more than the 126 MB L2), then read a second
    one.  The read evicts the written (dirty) lines, so their write-back happens here, outside
    the timed region, instead of competing with the next timed kernel's own traffic."""

    def __init__(self, nbytes=FLUSH_BYTES):
        import torch
        self.w = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        self.r = torch.zeros(nbytes // 4, dtype=torch.float32, device="cuda")

    def __call__(self):
        self.w.zero_()
        self.r.sum()


HIDE_HOST_CYCLES = 400_000       # ~200 us of GPU spin before each timed step


def timed_steps(fn, steps, flush, hide_host=True):
    """Per-step CUDA-event timing on the current stream with an L2 flush between steps.
    With hide_host the GPU spins for a while before each step's start event, so the host's
    launch work for the step is done before the GPU reaches the event: the region then holds
    device time only, even for calls shorter than their launch overhead."""
    import torch
    s = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        if flush is not None:
            flush()
        if hide_host:
            torch.cuda._sleep(HIDE_HOST_CYCLES)
        evs[i][0].record(s)
        fn()
        evs[i][1].record(s)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


def quantize_bench(nv, steps, warmup, flush):
    """cfg2: 8192 x 7168 bf16 -> NVFP4 with a given global scale (2.5625 B/elt)."""
    import torch
    from tensorcore_ptx_example_b200 import workloads
    rows, cols = workloads.CFG2_SHAPE
    x = workloads.activations(rows, cols, seed=2)
    gs = float(nv.amax(x).item()) / 2688.0
    packed = torch.empty((rows, cols // 2), dtype=torch.uint8, device="cuda")
    sf = torch.empty(nv.sf_bytes(rows, cols), dtype=torch.uint8, device="cuda")
    fn = lambda: nv.quantize(x, gs, packed=packed, sf=sf)  # noqa: E731
    for _ in range(warmup):
        fn()
    ts = timed_steps(fn, steps, flush)
    amax_out = torch.empty(1, dtype=torch.float32, device="cuda")
    ts_amax = timed_steps(lambda: nv.amax(x, out=amax_out), steps, flush)
    ws = torch.empty(256, dtype=torch.uint8, device="cuda")
    gsd = torch.empty(1, dtype=torch.float32, device="cuda")
    ts_auto = timed_steps(lambda: nv.lib().nvfp4_quantize_bf16_auto(
        nv._ptr(x), rows, cols, nv._ptr(packed), nv._ptr(sf), nv._ptr(gsd), nv._ptr(ws), nv._stream()), steps, flush)
    n = rows * cols
    ms = sum(ts) / len(ts)
    byts = n * 2.5625
    peaks, peak_kind = load_peaks()
    hbm = float(peaks.get("hbm_gbs", HBM_FALLBACK_GBS))
    gbs = byts / (ms * 1e-3) / 1e9
    return {
        "workload": "cfg2 quantize 8192x7168 bf16 -> NVFP4 (tcgen05 SF layout), given global scale",
        "us": round(ms * 1e3, 2),
        "gbs": round(gbs, 1),
        "bytes_per_launch": int(byts),
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(gbs / hbm, 4), "peak_source": f"{peak_kind} HBM copy",
                     "traffic": read_profile_traffic("quantize_cfg2")},
        "amax_us": round(sum(ts_amax) / len(ts_amax) * 1e3, 2),
        "auto_scale_total_us": round(sum(ts_auto) / len(ts_auto) * 1e3, 2),
    }


def decode_bench(nv, steps, warmup, flush):
    """cfg3 decode shape M16 N7168 K8192 (HBM-bound: the kernel streams B once)."""
    import torch
    from tensorcore_ptx_example_b200 import workloads
    M, N, K = workloads.CFG3_DECODE_SHAPE
    a = workloads.activations(M, K, seed=5)
    b = workloads.gaussian(N, K, seed=6, std=0.02)
    pa, sa, gsa = nv.quantize(a, None)
    pb, sb, gsb = nv.quantize(b, None)
    torch.cuda.synchronize()
    alpha = float(gsa.item()) * float(gsb.item())
    d = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    fn = lambda: nv.gemm(pa, sa, pb, sb, M, N, K, alpha=alpha, out=d)  # noqa: E731
    for _ in range(warmup):
        fn()
    ts = timed_steps(fn, steps, flush)
    ms = sum(ts) / len(ts)
    # Decode stream: back-to-back calls over WEIGHT_SETS different B (like consecutive layers of
    # a decode step); 8 x 33 MB > L2, so every call reads its B from HBM without a flush.
    weight_sets = 8
    bs = [(pb, sb)]
    for i in range(1, weight_sets):
        bi = workloads.gaussian(N, K, seed=100 + i, std=0.02)
        pbi, sbi, _ = nv.quantize(bi, None)
        del bi
        bs.append((pbi, sbi))
    torch.cuda.synchronize()
    calls = max(steps, 2 * weight_sets)
    for i in range(weight_sets):
        nv.gemm(pa, sa, bs[i][0], bs[i][1], M, N, K, alpha=alpha, out=d)
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(HIDE_HOST_CYCLES * 4)
    e0.record(s)
    for i in range(calls):
        pbi, sbi = bs[i % weight_sets]
        nv.gemm(pa, sa, pbi, sbi, M, N, K, alpha=alpha, out=d)
    e1.record(s)
    torch.cuda.synchronize()
    ms_stream = e0.elapsed_time(e1) / calls
    # the same stream with the weights marked constant (B streams before each dependency wait)
    torch.cuda._sleep(HIDE_HOST_CYCLES * 4)
    e0.record(s)
    for i in range(calls):
        pbi, sbi = bs[i % weight_sets]
        nv.gemm(pa, sa, pbi, sbi, M, N, K, alpha=alpha, out=d, weights_const=True)
    e1.record(s)
    torch.cuda.synchronize()
    ms_stream_wc = e0.elapsed_time(e1) / calls
    del bs
    # algorithmic bytes: B and its scales, A and its scales, D
    byts = N * K // 2 + N * K // 16 + M * K // 2 + nv.sf_bytes(M, K) + M * N * 2
    peaks, peak_kind = load_peaks()
    hbm = float(peaks.get("hbm_gbs", HBM_FALLBACK_GBS))
    gbs = byts / (ms * 1e-3) / 1e9
    gbs_stream = byts / (ms_stream * 1e-3) / 1e9
    return {"workload": "cfg3 decode GEMM M16 N7168 K8192 (split-K over 128-row tiles of B)",
            "us": round(ms * 1e3, 2), "tflops": round(2.0 * M * N * K / (ms * 1e-3) / 1e12, 1),
            "bytes_per_call": int(byts),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(gbs / hbm, 4), "peak_source": f"{peak_kind} HBM copy",
                         "timing": "one call after an L2 flush (includes the launch after foreign kernels)"},
            "stream": {"us_per_call": round(ms_stream * 1e3, 2), "calls": calls, "weight_sets": weight_sets,
                       "roofline": {"bound": "hbm", "achieved": round(gbs_stream, 1), "peak": hbm, "unit": "GB/s",
                                    "frac": round(gbs_stream / hbm, 4)},
                       "timing": "back-to-back calls over 8 different B (264 MB > L2), one event pair",
                       "us_per_call_weights_const": round(ms_stream_wc * 1e3, 2),
                       "frac_weights_const": round(byts / (ms_stream_wc * 1e-3) / 1e9 / hbm, 4)},
            "launches_per_call": 2}


def gemm_quantize_bench(nv, steps, flush):
    """cfg3 GEMM whose epilogue writes NVFP4 (next layer's input) against GEMM (bf16 D) followed by
    the quantizer; both produce the same bytes."""
    import torch
    pa, sa, pb, sb, alpha, d = gemm_setup(nv, 0)
    nv.gemm(pa, sa, pb, sb, M_, N_, K_, alpha=alpha, out=d)
    torch.cuda.synchronize()
    gs = nv.global_scale_from_amax(float(d.float().abs().max()))
    qp = torch.empty((M_, N_ // 2), dtype=torch.uint8, device="cuda")
    qs = torch.empty(nv.sf_bytes(M_, N_), dtype=torch.uint8, device="cuda")
    fused = lambda: nv.gemm_quantize(pa, sa, pb, sb, M_, N_, K_, alpha, gs, packed=qp, sf=qs)  # noqa: E731

    def two_step():
        nv.gemm(pa, sa, pb, sb, M_, N_, K_, alpha=alpha, out=d)
        nv.quantize(d, gs, packed=qp, sf=qs)

    for fn in (fused, two_step):
        for _ in range(3):
            fn()
    ms_f = sum(timed_steps(fused, steps, flush)) / steps
    ms_t = sum(timed_steps(two_step, steps, flush)) / steps
    return {"workload": "cfg3 GEMM 8192^3 with NVFP4 output (given global scale)",
            "us_fused": round(ms_f * 1e3, 1), "us_gemm_then_quantize": round(ms_t * 1e3, 1),
            "tflops_fused": round(2.0 * M_ * N_ * K_ / (ms_f * 1e-3) / 1e12, 1), "launches_fused": 1,
            "launches_two_step": 2}


def cpu_baseline_gemm(target_s=8.0):
    """Reference CPU GEMM (cpu_gemm_ref_bs, random_cpu_ref/verify_random.h:154) on all host
    threads over a bounded M x N slice of the K=8192 problem; returns TFLOPS."""
    import ctypes

    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import py_oracle
    threads = os.cpu_count() or 1
    K = K_
    nseg = K // 16
    rng = np.random.default_rng(0)
    vals = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -.5, -1, -1.5, -2, -3, -4, -6], np.float32)

    def run(M, N):
        A = rng.choice(vals, size=(M, K)).astype(np.float32)
        B = rng.choice(vals, size=(N, K)).astype(np.float32)
        sfa = np.ones(nseg, np.float32)
        sfb = np.ones(nseg, np.float32)
        D = np.zeros((M, N), np.float32)
        p = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
        t0 = time.perf_counter()
        if py_oracle.ref_verify_available():
            py_oracle.ref_lib().ref_cpu_gemm_ref_bs_threads(p(A), p(B), p(D), M, N, K, p(sfa), p(sfb), nseg, threads)
            kind = "reference"
        else:
            # oracle port of the same arithmetic (packed operands)
            pa = np.zeros((M, K // 2), np.uint8)
            pb = np.zeros((N, K // 2), np.uint8)
            sa = np.full(py_oracle.sf_bytes(M, K), 0x38, np.uint8)
            sb = np.full(py_oracle.sf_bytes(N, K), 0x38, np.uint8)
            py_oracle.gemm_f32(pa, sa, pb, sb, M, N, K, nthreads=threads)
            kind = "port"
        return time.perf_counter() - t0, kind

    dt, kind = run(threads, 64)                        # calibration
    rate = 2.0 * threads * 64 * K / max(dt, 1e-6)
    M = max(threads, int(target_s * rate / (2.0 * 256 * K)) // threads * threads)
    M = min(M, 8192)
    dt, kind = run(M, 256)
    flops = 2.0 * M * 256 * K
    return {"value": flops / dt / 1e12, "unit": "TFLOPS", "cores": threads, "kind": kind,
            "sample": f"{M}x256x{K} slice of the cfg3 GEMM (cpu_gemm_ref_bs, {nseg} K segments)",
            "seconds": round(dt, 3)}


def _bf16_sample(rng, shape):
    """N(0, 1) bf16 bit patterns (float32 draws truncated to their top 16 bits); at most 4 M
    distinct draws, repeated to fill the shape."""
    import numpy as np
    n = int(np.prod(shape))
    base = (rng.standard_normal(min(n, 1 << 22), dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)
    return np.resize(base, shape)


def _sized_sample(run, unit, limit, target_s):
    """Units (a multiple of `unit`, at most `limit`) that `run` handles in about target_s seconds,
    from a calibration run of one unit; returns (units, seconds of the sized run)."""
    rate = unit / max(run(unit), 1e-6)
    n = min(limit, max(unit, int(target_s * rate) // unit * unit))
    return n, run(n)


def cpu_baseline_quantize(target_s=2.0):
    """The oracle's quantizer (its restatement of q16 / quantize_kernel,
    blackwell/allreduce_sm100_sm120/nvfp4_allreduce.cuh:272-302,427-454; the reference has no CPU
    quantizer) on all host threads over a bounded row slice of cfg2, given the global scale;
    GB/s at 2.5625 B/elt."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import py_oracle
    from tensorcore_ptx_example_b200 import workloads
    threads = py_oracle.nthreads_default()
    rows_total, cols = workloads.CFG2_SHAPE
    full = _bf16_sample(np.random.default_rng(2), (rows_total, cols))
    gs, _ = py_oracle.global_scale(py_oracle.amax_bf16(full))

    def run(rows, nthreads=threads):
        x = full[:rows]
        t0 = time.perf_counter()
        py_oracle.quantize_bf16(x, gs, nthreads=nthreads)
        return time.perf_counter() - t0

    rows, dt = _sized_sample(run, 128, rows_total, target_s)
    rows1, dt1 = _sized_sample(lambda r: run(r, 1), 128, rows_total, target_s / 2)
    return {"value": round(rows * cols * 2.5625 / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{rows}x{cols} rows of cfg2 (N(0,1)), oracle orc_quantize_bf16", "seconds": round(dt, 3),
            "single_thread_gbs": round(rows1 * cols * 2.5625 / dt1 / 1e9, 3), "single_thread_rows": rows1}


def cpu_baseline_allreduce(target_s=2.0, world=8):
    """The oracle's fixed-order NVFP4 two-shot (quantize, dequant-sum in rank order 0..n-1,
    requantize, dequantize: the data flow of twoshot_fused_kernel, nvfp4_allreduce.cuh:498-567)
    for 8 ranks on all host threads, over a bounded slice of cfg4 per rank; bf16-equivalent
    algbw 2 * numel / t in GB/s, the unit of the GPU all-reduce lines."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import py_oracle
    from tensorcore_ptx_example_b200 import workloads
    threads = py_oracle.nthreads_default()
    rows, cols = workloads.CFG4_SHAPE
    rng = np.random.default_rng(4)
    full = [_bf16_sample(rng, rows * cols) for _ in range(world)]
    gs, _ = py_oracle.global_scale(max(py_oracle.amax_bf16(x) for x in full))

    def run(numel):
        ins = [x[:numel] for x in full]
        t0 = time.perf_counter()
        py_oracle.ar_twoshot(ins, gs, nthreads=threads)
        return time.perf_counter() - t0

    numel, dt = _sized_sample(run, 32 * world * 256, rows * cols, target_s)
    return {"value": round(2.0 * numel / dt / 1e9, 3), "unit": "GB/s (bf16-equivalent algbw)", "cores": threads,
            "kind": "port", "sample": f"{numel} elements per rank x {world} ranks of cfg4 (N(0,1)), oracle "
                                      f"orc_ar_twoshot", "seconds": round(dt, 3)}


def run_ours(args):
    import torch
    import tensorcore_ptx_example_b200 as nv
    world, rank, local = dist_setup(args)
    peaks, peak_kind = load_peaks()
    flush = L2Flush()

    pa, sa, pb, sb, alpha, d = gemm_setup(nv, rank)
    fn = lambda: nv.gemm(pa, sa, pb, sb, M_, N_, K_, alpha=alpha, out=d)  # noqa: E731
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    assert nv.device_status() == 0
    barrier(world)
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    ts = timed_steps(fn, args.steps, flush)
    clocks = sampler.stop()
    barrier(world)
    total_ms = max_over_ranks(sum(ts), world)
    flops = 2.0 * M_ * N_ * K_
    value = flops * args.steps * world / (total_ms * 1e-3) / 1e12
    mean_ms = sum(ts) / len(ts)
    achieved = flops / (mean_ms * 1e-3) / 1e12
    fp4_peak = 4.0 * float(peaks.get("bf16_tflops", BF16_FALLBACK_TFLOPS))
    assert nv.device_status() == 0

    # end to end through the public API with host buffers: every step copies its operands from
    # pinned host memory, runs the GEMM and copies D back.  Steps are pipelined over two buffer
    # sets and three streams (H2D of step i+1 and D2H of step i-1 overlap the GEMM of step i; PCIe
    # carries both directions at once); the time is the whole run divided by the steps.
    host = [t.cpu().pin_memory() for t in (pa, sa, pb, sb)]
    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = M_ * N_ * 2
    dev_sets = [(pa, sa, pb, sb, d), tuple(torch.empty_like(t) for t in (pa, sa, pb, sb, d))]
    host_out = [torch.empty((M_, N_), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    s_in, s_mm, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()

    def e2e_run(n_steps):
        done_out = [None, None]                       # D2H of the step that last used a buffer set
        for i in range(n_steps):
            j = i & 1
            da, dsa, db, dsb, dd = dev_sets[j]
            ev_in = torch.cuda.Event()
            with torch.cuda.stream(s_in):
                if done_out[j] is not None:
                    s_in.wait_event(done_out[j])
                for h, dv in zip(host, (da, dsa, db, dsb)):
                    dv.copy_(h, non_blocking=True)
                ev_in.record(s_in)
            ev_mm = torch.cuda.Event()
            with torch.cuda.stream(s_mm):
                s_mm.wait_event(ev_in)
                nv.gemm(da, dsa, db, dsb, M_, N_, K_, alpha=alpha, out=dd, stream=s_mm)
                ev_mm.record(s_mm)
            ev_out = torch.cuda.Event()
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_mm)
                host_out[j].copy_(dd, non_blocking=True)
                ev_out.record(s_out)
            done_out[j] = ev_out

    e2e_run(3)
    torch.cuda.synchronize()
    e2e_steps = max(4, min(args.steps, 12))
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(HIDE_HOST_CYCLES * 8)
    e0.record()
    for st in (s_in, s_mm, s_out):
        st.wait_stream(torch.cuda.current_stream())
    e2e_run(e2e_steps)
    for st in (s_in, s_mm, s_out):
        torch.cuda.current_stream().wait_stream(st)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps, world)
    assert torch.equal(host_out[(e2e_steps - 1) & 1], d.cpu())

    extra = {}
    if rank == 0:
        try:
            extra["quantize"] = quantize_bench(nv, max(5, args.steps), 3, flush)
        except Exception as e:  # reported, not fatal
            extra["quantize"] = {"error": str(e)}
        try:
            extra["gemm_decode"] = decode_bench(nv, max(5, args.steps), 3, flush)
        except Exception as e:  # reported, not fatal
            extra["gemm_decode"] = {"error": str(e)}
        try:
            extra["gemm_quantize"] = gemm_quantize_bench(nv, min(max(5, args.steps), 20), flush)
        except Exception as e:  # reported, not fatal
            extra["gemm_quantize"] = {"error": str(e)}
    if world > 1:
        extra["allreduce"] = allreduce_bench(nv, world, rank, args, flush=flush)
        extra["gemm_allreduce"] = gemm_allreduce_bench(nv, world, rank, args, flush=flush)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_gemm()
        for key, fn in (("quantize", cpu_baseline_quantize), ("allreduce_cpu_baseline", cpu_baseline_allreduce)):
            try:
                res = fn()
            except Exception as e:  # reported, not fatal
                res = {"error": str(e)}
            if key == "quantize":
                if isinstance(extra.get("quantize"), dict):
                    extra["quantize"]["cpu_baseline"] = res
            else:
                extra[key] = res

    traffic = read_profile_traffic("gemm_cfg3")
    line = {
        "metric": "NVFP4 GEMM TFLOPS (1 GPU); NVFP4 all-reduce bf16-equiv GB/s at 2/4/8 B200",
        "value": round(value, 1),
        "unit": "TFLOPS",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "e2m1 x e2m1 (ue4m3 per-16 scales) -> fp32 accumulate -> bf16",
        "data": "synthetic (seeded N(0,1)+0.1% x50 outliers / N(0,0.02), quantized on device)",
        "config": {"workload": "cfg3 NVFP4 GEMM M=N=K=8192, bf16 out", "M": M_, "N": N_, "K": K_,
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "flushed between timed steps (256 MB write, then 256 MB read)",
                   "tile": "CTA pair (tcgen05 cta_group::2) 256x256, BK=256, 5 stages, persistent"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(fp4_peak, 1),
                     "unit": "TFLOP/s", "frac": round(achieved / fp4_peak, 4),
                     "peak_source": f"4 x {peak_kind} cuBLAS bf16 burst ({peaks.get('bf16_tflops')}) = dense FP4 rate",
                     "frac_of_nominal_fp4_9000": round(achieved / FP4_NOMINAL_TFLOPS, 4),
                     "traffic": traffic,
                     "algorithmic_flops_per_launch": flops},
        "e2e": {"value": round(flops / (e2e_ms * 1e-3) / 1e12 * world, 2), "unit": "TFLOPS",
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                "path": "pinned host A/B/SF -> device, nvfp4_gemm_bf16, device D -> pinned host; steps pipelined "
                        "over two buffer sets (copies of neighbouring steps overlap the GEMM)"},
        "gpu_launches": args.steps,
        "clocks": clocks,
        **extra,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


NVLINK_PEER_GBS = 770.0      # measured peer copy per direction per GPU on this pool (900 nominal)


def _ar_time(fn, steps, warmup, flush, world):
    """Per-call device time (ms) of an all-reduce, max over ranks of the per-rank mean."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    ts = timed_steps(fn, steps, flush)
    barrier(world)
    return max_over_ranks(sum(ts) / len(ts), world)


def _ar_time_b2b(fn, calls, warmup, world):
    """Per-call device time (ms) of `calls` back-to-back all-reduces (the reference harness's
    method, bench_ar.cu:965-972: events around a loop of calls), max over ranks.  The GPU spins
    first while the host queues every call, so no host launch gap falls inside the region.  One
    untimed call after the spin lines the ranks up (spins of equal cycle counts end at different
    times on GPUs at different clocks); the calls' own barriers keep them in step after that."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(HIDE_HOST_CYCLES * max(1, calls // 4))
    fn()
    e0.record(s)
    for _ in range(calls):
        fn()
    e1.record(s)
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(e0.elapsed_time(e1) / calls, world)


def _ar_entry(name, numel, world, ms, payload_bytes_per_elt):
    """bf16-equivalent algbw / busbw (nccl-tests convention) and wire rate of one algorithm."""
    t = ms * 1e-3
    algbw = 2.0 * numel / t / 1e9
    busbw = algbw * 2.0 * (world - 1) / world
    two = "twoshot" in name
    wire = (2.0 * (world - 1) / world if two else (world - 1)) * payload_bytes_per_elt * numel
    return {"us": round(ms * 1e3, 2), "algbw_gbs": round(algbw, 1), "busbw_gbs": round(busbw, 1),
            "wire_bytes_per_rank": int(wire), "wire_gbs_per_rank": round(wire / t / 1e9, 1),
            "frac_of_nvlink_770": round(wire / t / 1e9 / NVLINK_PEER_GBS, 4)}


def allreduce_bench(nv, world, rank, args, numel=None, steps=None, flush=None):
    """cfg4: every rank holds 4096 x 7168 bf16 N(0, 1), seed = rank.  NVFP4 two-shot / one-shot
    and the in-house bf16 P2P all-reduce, device time per call (max over ranks), L2 flushed
    between calls; plus the NVFP4 error against the exact sum and an end-to-end number through
    the public API with the input copied from pinned host memory and the result copied back."""
    import torch
    import torch.distributed as dist

    from tensorcore_ptx_example_b200 import allreduce as ar
    from tensorcore_ptx_example_b200 import workloads
    rows, cols = workloads.CFG4_SHAPE
    numel = numel or rows * cols
    steps = steps or max(5, min(args.steps, 20))
    x = workloads.gaussian(1, numel, seed=rank).view(-1)
    gs = ar.agree_global_scale(float(nv.amax(x).item()))
    ctx = ar.AllReduce.from_process_group(numel)
    out = torch.empty_like(x)
    res = {"workload": f"cfg4 all-reduce {numel} bf16 elements per rank (N(0,1), seed = rank)",
           "world": world, "global_scale": gs, "l2": "flushed between calls" if flush is not None else "not flushed"}
    try:
        runs = [("nvfp4_twoshot", lambda: ctx.allreduce(x, out, global_scale=gs, algo="twoshot"), 0.5625),
                ("nvfp4_oneshot", lambda: ctx.allreduce(x, out, global_scale=gs, algo="oneshot"), 0.5625),
                ("bf16_twoshot", lambda: ctx.bf16_allreduce(x, out, algo="twoshot"), 2.0),
                ("bf16_oneshot", lambda: ctx.bf16_allreduce(x, out, algo="oneshot"), 2.0)]
        for name, fn, bpe in runs:
            ms = _ar_time(fn, steps, 3, flush, world)
            res[name] = _ar_entry(name, numel, world, ms, bpe)
        # accuracy of both NVFP4 algorithms against the exact (fp32, NCCL) sum
        exact = x.float().clone()
        dist.all_reduce(exact)
        for algo in ("twoshot", "oneshot"):
            o = ctx.allreduce(x, out, global_scale=gs, algo=algo).float()
            res[f"nvfp4_{algo}"]["rel_rmse_vs_fp32_sum"] = round(float((o - exact).norm() / exact.norm()), 5)
        torch.cuda.synchronize()
        res["device_status"] = nv.device_status()
        # end to end: pinned host input -> device, all-reduce (two-shot), device -> pinned host
        hx = x.cpu().pin_memory()
        ho = torch.empty_like(hx).pin_memory()

        def e2e():
            x.copy_(hx, non_blocking=True)
            ctx.allreduce(x, out, global_scale=gs, algo="twoshot")
            ho.copy_(out, non_blocking=True)
        e2e_ms = _ar_time(e2e, max(3, steps // 2), 2, None, world)
        res["e2e_nvfp4_twoshot"] = {"us": round(e2e_ms * 1e3, 2),
                                    "algbw_gbs": round(2.0 * numel / (e2e_ms * 1e-3) / 1e9, 1),
                                    "h2d_bytes_per_step": numel * 2, "d2h_bytes_per_step": numel * 2}
        res["gpu_launches_per_call"] = 1
    finally:
        torch.cuda.synchronize()
        barrier(world)
        ctx.close()
    return res


def gemm_allreduce_bench(nv, world, rank, args, flush=None):
    """Row-parallel layer with the cfg4 output (M 4096 x N 7168 bf16) and K 8192 split over the
    ranks: the NVFP4 GEMM fused with the two-shot all-reduce (one GEMM kernel whose epilogue
    pushes the quantized tiles to their owners, then the all-reduce's reduce and all-gather)
    against GEMM then all-reduce; device time per call, max over ranks."""
    import torch

    from tensorcore_ptx_example_b200 import allreduce as ar
    from tensorcore_ptx_example_b200 import workloads
    M, N = workloads.CFG4_SHAPE
    K = 8192 // world
    a = workloads.activations(M, K, seed=11 + 2 * rank)
    b = workloads.gaussian(N, K, seed=12 + 2 * rank, std=0.02)
    pa, sa, gsa = nv.quantize(a, None)
    pb, sb, gsb = nv.quantize(b, None)
    torch.cuda.synchronize()
    del a, b
    alpha = float(gsa.item()) * float(gsb.item())
    d = nv.gemm(pa, sa, pb, sb, M, N, K, alpha=alpha)
    torch.cuda.synchronize()
    gs = ar.agree_global_scale(float(d.float().abs().max()))
    ctx = ar.AllReduce.from_process_group(M * N)
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    steps = max(5, min(args.steps, 20))
    res = {"workload": f"row-parallel NVFP4 GEMM M{M} N{N} K{K} per rank (K 8192 total) + two-shot all-reduce",
           "world": world}
    try:
        fused = lambda: ctx.gemm_allreduce(pa, sa, pb, sb, M, N, K, alpha, gs, out=out)  # noqa: E731

        def unfused():
            nv.gemm(pa, sa, pb, sb, M, N, K, alpha=alpha, out=d)
            ctx.allreduce(d.view(-1), out.view(-1), global_scale=gs, algo="twoshot")

        ms_f = _ar_time(fused, steps, 3, flush, world)
        ms_u = _ar_time(unfused, steps, 3, flush, world)
        o_f = ctx.gemm_allreduce(pa, sa, pb, sb, M, N, K, alpha, gs).clone()
        unfused()
        torch.cuda.synchronize()
        res.update({"us_fused": round(ms_f * 1e3, 1), "us_gemm_then_allreduce": round(ms_u * 1e3, 1),
                    "speedup": round(ms_u / ms_f, 3), "same_bytes": bool(torch.equal(o_f, out)),
                    "launches_fused": 2, "launches_unfused": 2, "device_status": nv.device_status()})
    finally:
        torch.cuda.synchronize()
        barrier(world)
        ctx.close()
    return res


def allreduce_sweep(args):
    """cfg5: 16 KB .. 256 MB of bf16 per rank (doubling), NVFP4 low-latency one-shot (up to
    1 MB) / one-shot / two-shot and bf16 one-shot / two-shot, max over ranks of the mean device
    time per call over back-to-back calls."""
    import torch

    import tensorcore_ptx_example_b200 as nv
    from tensorcore_ptx_example_b200 import allreduce as ar
    from tensorcore_ptx_example_b200 import workloads
    world, rank, local = dist_setup(args)
    sizes = [b for b in workloads.sweep_sizes_bytes() if (b // 2) % (32 * world) == 0]
    max_numel = max(sizes) // 2
    ctx = ar.AllReduce.from_process_group(max_numel)
    xfull = workloads.gaussian(1, max_numel, seed=rank).view(-1)
    gs = ar.agree_global_scale(float(nv.amax(xfull).item()))
    ofull = torch.empty_like(xfull)
    rows = []
    try:
        for b in sizes:
            n = b // 2
            x, o = xfull[:n], ofull[:n]
            calls = 50 if b <= (16 << 20) else 10
            row = {"bytes": b, "numel": n}
            algos = [
                ("nvfp4_lowlat", lambda: ctx.allreduce(x, o, global_scale=gs, algo="lowlat"), 0.75),
                ("nvfp4_oneshot", lambda: ctx.allreduce(x, o, global_scale=gs, algo="oneshot"), 0.5625),
                ("nvfp4_twoshot", lambda: ctx.allreduce(x, o, global_scale=gs, algo="twoshot"), 0.5625),
                ("bf16_oneshot", lambda: ctx.bf16_allreduce(x, o, algo="oneshot"), 2.0),
                ("bf16_twoshot", lambda: ctx.bf16_allreduce(x, o, algo="twoshot"), 2.0)]
            if b > ar.LOWLAT_CAP_BYTES:
                algos = algos[1:]
            for name, fn, bpe in algos:
                ms = _ar_time_b2b(fn, calls, 3, world)
                e = _ar_entry(name, n, world, ms, bpe)
                row[name] = {"us": e["us"], "algbw_gbs": e["algbw_gbs"], "busbw_gbs": e["busbw_gbs"]}
            rows.append(row)
        torch.cuda.synchronize()
        status = nv.device_status()
    finally:
        barrier(world)
        ctx.close()
    if rank == 0:
        print(json.dumps({"sweep": "cfg5 all-reduce message sizes", "world": world, "device_status": status,
                          "l2": "not flushed (back-to-back calls)", "rows": rows}), flush=True)
    import torch.distributed as dist
    if world > 1:
        dist.destroy_process_group()


def read_profile_traffic(name):
    """DRAM bytes per launch from a committed ncu summary (profiles/<name>*.md line
    'traffic_bytes_per_launch: N'), or None."""
    d = os.path.join(ROOT, "profiles")
    if not os.path.isdir(d):
        return None
    for f in sorted(os.listdir(d)):
        if f.startswith(name) and f.endswith((".md", ".txt")):
            for ln in open(os.path.join(d, f)):
                if ln.strip().startswith("traffic_bytes_per_launch:"):
                    try:
                        return int(float(ln.split(":", 1)[1].strip().split()[0]))
                    except ValueError:
                        return None
    return None


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    vals = []
    res = None
    for i in range(args.warmup + args.steps):
        res = cpu_baseline_gemm(target_s=2.0)
        if i >= args.warmup:
            vals.append(res["value"])
    v = sum(vals) / len(vals)
    line = {
        "impl": "reference",
        "metric": "NVFP4 GEMM TFLOPS (1 GPU); NVFP4 all-reduce bf16-equiv GB/s at 2/4/8 B200",
        "value": v, "unit": "TFLOPS", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32 (reference CPU path on decoded E2M1 values)",
        "data": "synthetic (seeded E2M1 values)",
        "config": {"workload": "cfg3 NVFP4 GEMM M=N=K=8192 (bounded CPU sample per step)",
                   "M": M_, "N": N_, "K": K_},
        "cpu_baseline": {"value": v, "unit": "TFLOPS", "cores": res["cores"], "kind": res["kind"],
                         "sample": res["sample"]},
        "e2e": {"value": v, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_only(args):
    """One workload alone (used under ncu): warmup + steps launches, timings printed."""
    import torch
    import tensorcore_ptx_example_b200 as nv
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    flush = L2Flush()
    if args.only == "quantize":
        out = quantize_bench(nv, args.steps, args.warmup, flush)
    elif args.only == "gemm-decode":
        out = decode_bench(nv, args.steps, args.warmup, flush)
    elif args.only == "gemm-quantize":
        out = gemm_quantize_bench(nv, args.steps, flush)
    elif args.only == "ar-emulated":
        # the all-reduce data path of 8 ranks on this one GPU, phase by phase (no cross-GPU
        # waits): for profiling the phase kernels' memory traffic on a single device
        from tensorcore_ptx_example_b200 import allreduce as ar
        from tensorcore_ptx_example_b200 import workloads
        world, numel = 8, args.numel
        ins = [workloads.gaussian(1, numel, seed=r).view(-1) for r in range(world)]
        gs = nv.global_scale_from_amax(max(float(nv.amax(x).item()) for x in ins))
        ctxs = [ar.AllReduce(world, r, numel) for r in range(world)]
        ar.join_in_process(ctxs)
        for algo in ("twoshot", "oneshot"):
            for _ in range(args.warmup + args.steps):
                ar.emulated_allreduce(ins, gs, algo, contexts=ctxs)
        torch.cuda.synchronize()
        for c in ctxs:
            c.close()
        out = {"workload": f"emulated 8-rank all-reduce, {numel} elements per rank", "launches_per_call":
               "twoshot 3 phases x 8 ranks, oneshot 2 phases x 8 ranks"}
    else:
        pa, sa, pb, sb, alpha, d = gemm_setup(nv, 0)
        fn = lambda: nv.gemm(pa, sa, pb, sb, M_, N_, K_, alpha=alpha, out=d)  # noqa: E731
        for _ in range(args.warmup):
            fn()
        ts = timed_steps(fn, args.steps, flush)
        ms = sum(ts) / len(ts)
        out = {"workload": "cfg3 GEMM 8192^3", "ms": round(ms, 4),
               "tflops": round(2.0 * M_ * N_ * K_ / (ms * 1e-3) / 1e12, 1)}
    torch.cuda.synchronize()
    out["device_status"] = nv.device_status()
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--numel", type=int, default=4 << 20, help="elements per rank for --only ar-emulated")
    ap.add_argument("--only", choices=["gemm", "gemm-decode", "gemm-quantize", "quantize", "ar-sweep", "ar-emulated"],
                    default=None,
                    help="profiling mode: run one workload (warmup + steps launches) and print its "
                         "timings; not the benchmark line")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.only == "ar-sweep":
        allreduce_sweep(args)
    elif args.only:
        run_only(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
