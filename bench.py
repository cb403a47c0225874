#!/usr/bin/env python
"""Benchmark of the NVFP4 data path (prints ONE JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

The metric is BASELINE's: "NVFP4 GEMM TFLOPS (1 GPU); NVFP4 all-reduce bf16-equiv GB/s at 2/4/8 B200".

N = 1: the cfg3 block-scaled GEMM M=N=K=8192 (operands quantized on the device from seeded
synthetic bf16: A ~ N(0,1) with 0.1 % x50 outliers, B ~ N(0, 0.02)).  One step = one GEMM launch;
L2 is flushed between timed steps; CUDA events on the launching stream.  Extra keys: the roofline
against the FP4 MMA issue rate measured live on the same GPU, the cfg2 quantizer (with the
reference's own quantize kernel timed beside it), the decode GEMM, the GEMM with the quantizing
epilogue, the CPU baselines, an end-to-end number through the C ABI with host buffers, and SM
clocks sampled during the timed region.

N > 1 (one process per GPU under torchrun): the cfg4 NVFP4 all-reduce (4096 x 7168 bf16 per
rank, N(0,1), seed = rank; algorithm NVFP4_AR_AUTO).  One step = one all-reduce call; the K steps
run back to back between one pair of events, each reading the next of several copies of the input
that together exceed L2; the time is the max over ranks.  `value` is the bf16-equivalent algorithm
bandwidth 2 * numel / t (nccl-tests convention; busbw = algbw * 2 (n-1) / n).  The line also
carries bit-exact parity against the CPU oracle on sampled windows of every algorithm's output,
each algorithm's time and wire rate, compact cfg5 rows (best NVFP4 against best bf16), the
reference's own fused kernels timed on the same GPUs, the fused row-parallel GEMM + all-reduce,
GEMM replicas, and the end-to-end all-reduce with host buffers.

--impl reference times the reference's CPU path on rank 0 (other ranks exit): at N = 1 its
cpu_gemm_ref_bs (random_cpu_ref/verify_random.h, compiled into oracle/_ref) on a bounded slice of
the GEMM; at N > 1 the oracle's fixed-order NVFP4 two-shot for N ranks over a bounded slice of
cfg4 (the reference has no CPU all-reduce of its own).
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
METRIC = "NVFP4 GEMM TFLOPS (1 GPU); NVFP4 all-reduce bf16-equiv GB/s at 2/4/8 B200"
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
    try:
        ref = reference_quantize_kernel(x, gs, steps, flush)
    except Exception as e:  # reported, not fatal
        ref = {"error": str(e)}
    n = rows * cols
    ms = sum(ts) / len(ts)
    byts = n * 2.5625
    peaks, peak_kind = load_peaks()
    hbm = float(peaks.get("hbm_gbs", HBM_FALLBACK_GBS))
    gbs = byts / (ms * 1e-3) / 1e9
    # Back-to-back launches over three input / output sets (3 x 150 MB > L2, so no flush is needed
    # between launches): each launch's start overlaps the previous one's tail, as in a stream of
    # layers; one event pair around all of them.
    sets = [(x, packed, sf)] + [(workloads.activations(rows, cols, seed=20 + i),
                                 torch.empty_like(packed), torch.empty_like(sf)) for i in range(2)]
    for xi, pi, si in sets:
        nv.quantize(xi, gs, packed=pi, sf=si)
    calls = max(3 * steps, 30)
    s_ = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    torch.cuda._sleep(HIDE_HOST_CYCLES * 8)
    e0.record(s_)
    for i in range(calls):
        xi, pi, si = sets[i % 3]
        nv.quantize(xi, gs, packed=pi, sf=si)
    e1.record(s_)
    torch.cuda.synchronize()
    ms_stream = e0.elapsed_time(e1) / calls
    gbs_stream = byts / (ms_stream * 1e-3) / 1e9
    del sets
    return {
        "workload": "cfg2 quantize 8192x7168 bf16 -> NVFP4 (tcgen05 SF layout), given global scale",
        "us": round(ms * 1e3, 2),
        "gbs": round(gbs, 1),
        "bytes_per_launch": int(byts),
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(gbs / hbm, 4), "peak_source": f"{peak_kind} HBM copy",
                     "timing": "one launch after an L2 flush, CUDA events around it",
                     "traffic": read_profile_traffic("quantize_cfg2")},
        "stream": {"us_per_call": round(ms_stream * 1e3, 2), "calls": calls,
                   "roofline": {"bound": "hbm", "achieved": round(gbs_stream, 1), "peak": hbm, "unit": "GB/s",
                                "frac": round(gbs_stream / hbm, 4)},
                   "timing": "back-to-back launches over 3 input/output sets (450 MB > L2), one event pair"},
        "amax_us": round(sum(ts_amax) / len(ts_amax) * 1e3, 2),
        "amax_gbs": round(n * 2 / (sum(ts_amax) / len(ts_amax) * 1e-3) / 1e9, 1),
        "auto_scale_total_us": round(sum(ts_auto) / len(ts_auto) * 1e3, 2),
        "reference_kernel": ref,
    }


def decode_bench(nv, steps, warmup, flush, shape=None):
    """cfg3 decode shape M16 N7168 K8192 (HBM-bound: the kernel streams B once), or `shape`."""
    import torch
    from tensorcore_ptx_example_b200 import workloads
    M, N, K = shape or workloads.CFG3_DECODE_SHAPE
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
    # the same weights-const stream captured once in a CUDA graph and replayed (as a decode step's
    # layers would be): no host launch work between the kernels
    ms_graph = None
    try:
        g = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream()
        cap.wait_stream(s)
        with torch.cuda.stream(cap):
            for i in range(weight_sets):           # warm-up on the capture stream
                nv.gemm(pa, sa, bs[i][0], bs[i][1], M, N, K, alpha=alpha, out=d, weights_const=True)
            cap.synchronize()
            with torch.cuda.graph(g, stream=cap):
                for i in range(calls):
                    pbi, sbi = bs[i % weight_sets]
                    nv.gemm(pa, sa, pbi, sbi, M, N, K, alpha=alpha, out=d, weights_const=True)
        s.wait_stream(cap)
        g.replay()
        torch.cuda.synchronize()
        torch.cuda._sleep(HIDE_HOST_CYCLES)
        e0.record(s)
        g.replay()
        e1.record(s)
        torch.cuda.synchronize()
        ms_graph = e0.elapsed_time(e1) / calls
        del g
    except Exception as e:  # reported, not fatal
        ms_graph = f"graph capture failed: {e}"
    del bs
    # algorithmic bytes: B and its scales, A and its scales, D
    byts = N * K // 2 + N * K // 16 + M * K // 2 + nv.sf_bytes(M, K) + M * N * 2
    peaks, peak_kind = load_peaks()
    hbm = float(peaks.get("hbm_gbs", HBM_FALLBACK_GBS))
    gbs = byts / (ms * 1e-3) / 1e9
    gbs_stream = byts / (ms_stream * 1e-3) / 1e9
    return {"workload": f"{'cfg3 ' if shape is None else ''}decode GEMM M{M} N{N} K{K} (split-K over 128-row tiles of B)",
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
                       "frac_weights_const": round(byts / (ms_stream_wc * 1e-3) / 1e9 / hbm, 4),
                       "us_per_call_graph": round(ms_graph * 1e3, 2) if isinstance(ms_graph, float) else ms_graph,
                       "frac_graph": (round(byts / (ms_graph * 1e-3) / 1e9 / hbm, 4)
                                      if isinstance(ms_graph, float) else None)},
            # the in-cluster split-K reduction needs no workspace and no second kernel
            "launches_per_call": 1 if int(nv.lib().nvfp4_gemm_workspace_bytes(M, N, K)) == 0 else 2}


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


class CpuAllReduceSample:
    """The oracle's fixed-order NVFP4 two-shot (quantize, dequant-sum in rank order 0..n-1,
    requantize, dequantize: the data flow of twoshot_fused_kernel, nvfp4_allreduce.cuh:498-567)
    for `world` ranks on all host threads, over a bounded slice of cfg4 per rank; bf16-equivalent
    algbw 2 * numel / t in GB/s, the unit of the GPU all-reduce lines.  Inputs are drawn once."""

    def __init__(self, world=8):
        import numpy as np
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import py_oracle
        from tensorcore_ptx_example_b200 import workloads
        self.po = py_oracle
        self.world = world
        self.threads = py_oracle.nthreads_default()
        rows, cols = workloads.CFG4_SHAPE
        self.limit = rows * cols
        rng = np.random.default_rng(4)
        self.full = [_bf16_sample(rng, rows * cols) for _ in range(world)]
        self.gs, _ = py_oracle.global_scale(max(py_oracle.amax_bf16(x) for x in self.full))

    def run(self, numel):
        ins = [x[:numel] for x in self.full]
        t0 = time.perf_counter()
        self.po.ar_twoshot(ins, self.gs, nthreads=self.threads)
        return time.perf_counter() - t0

    def measure(self, target_s=2.0):
        numel, dt = _sized_sample(self.run, 32 * self.world * 256, self.limit, target_s)
        return {"value": round(2.0 * numel / dt / 1e9, 3), "unit": "GB/s (bf16-equivalent algbw)",
                "cores": self.threads, "kind": "port",
                "sample": f"{numel} elements per rank x {self.world} ranks of cfg4 (N(0,1)), oracle orc_ar_twoshot",
                "seconds": round(dt, 3)}


def cpu_baseline_allreduce(target_s=2.0, world=8):
    return CpuAllReduceSample(world).measure(target_s)


def reference_quantize_kernel(x, gs, steps, flush):
    """Same-box baseline: the reference's own quantize_kernel (nvfp4_allreduce.cuh:427-454; linear
    scale layout, rcp.approx reciprocals, 4-byte loads), compiled from the reference header into
    oracle/_ref/libref_ar.so, timed on the same GPU and input as ours, with SFScaleVal = 1 / gs."""
    import ctypes

    import numpy as np
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import py_oracle
    if not py_oracle.ref_ar_available():
        return {"unavailable": "oracle/_ref/libref_ar.so not built (needs the reference tree at build time)"}
    L = py_oracle.ref_ar_lib()
    numel = x.numel()
    out = torch.empty(int(L.ref_layout_total_bytes(numel)), dtype=torch.uint8, device="cuda")
    sf_val = float(np.float32(1.0) / np.float32(gs))
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    xp, op = ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr())

    def fn():
        rc = L.ref_quantize(xp, op, numel, sf_val, st)
        if rc:
            raise RuntimeError(f"ref_quantize: cuda error {rc}")
    for _ in range(3):
        fn()
    ts = timed_steps(fn, steps, flush)
    ms = sum(ts) / len(ts)
    return {"kernel": "nvfp4_ar::quantize_kernel (reference, oracle/_ref/libref_ar.so)", "us": round(ms * 1e3, 2),
            "gbs": round(numel * 2.5625 / (ms * 1e-3) / 1e9, 1),
            "note": "same input and L2 flush; linear scale layout instead of the tcgen05 one"}


def fp4_peak_measure(local):
    """The FP4 block-scaled MMA issue rate of this GPU, measured live (diagnostics library:
    every SM pair issues M256 N256 K64 MMAs from resident shared memory on pseudo-random E2M1
    operands), with its own clock samples: the tensor roofline of the GEMM."""
    from tensorcore_ptx_example_b200 import diag
    sampler = ClockSampler(local)
    sampler.start()
    diag.mma_peak_clock()                                    # reset the in-kernel clock counters
    tf = diag.mma_peak(cta_group=2, iters=32768, repeats=5, random_operands=True)
    mhz = diag.mma_peak_clock()
    clocks = sampler.stop()
    assert diag.device_status() == 0
    return {"tflops": round(tf, 1), "clocks": clocks, "sm_mhz_in_kernel": round(mhz, 1),
            "probe": "nvfp4_diag_mma_peak cta_group 2, 32768 MMAs per SM pair, random operands, best of 5; "
                     "sm_mhz_in_kernel = SM cycles / elapsed ns inside the probe's CTAs (clock64, globaltimer)"}


def run_gemm_line(args):
    import torch
    import tensorcore_ptx_example_b200 as nv
    world, rank, local = 1, 0, int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    peaks, peak_kind = load_peaks()
    flush = L2Flush()

    pa, sa, pb, sb, alpha, d = gemm_setup(nv, rank)
    fn = lambda: nv.gemm(pa, sa, pb, sb, M_, N_, K_, alpha=alpha, out=d)  # noqa: E731
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    assert nv.device_status() == 0
    sampler = ClockSampler(local)
    sampler.start()
    # no spin before each step: a 200-us GEMM hides its own launch, and the spin's idle time
    # measurably lowers the clock the GEMM then starts at (214.0 vs 209.6 us per step on B200)
    ts = timed_steps(fn, args.steps, flush, hide_host=False)
    clocks = sampler.stop()
    total_ms = sum(ts)
    flops = 2.0 * M_ * N_ * K_
    value = flops * args.steps / (total_ms * 1e-3) / 1e12
    mean_ms = sum(ts) / len(ts)
    achieved = flops / (mean_ms * 1e-3) / 1e12
    bf16x4 = 4.0 * float(peaks.get("bf16_tflops", BF16_FALLBACK_TFLOPS))
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

    def gemm_step(dev, stream):
        da, dsa, db, dsb, dd = dev
        nv.gemm(da, dsa, db, dsb, M_, N_, K_, alpha=alpha, out=dd, stream=stream)

    e2e_steps = max(4, min(args.steps, 12))
    e2e_ms = pipelined_e2e(host, dev_sets, host_out, gemm_step, e2e_steps)
    assert torch.equal(host_out[(e2e_steps - 1) & 1], d.cpu())

    fp4 = None
    try:
        fp4 = fp4_peak_measure(local)
    except Exception as e:  # reported, not fatal
        fp4 = {"error": str(e)}
    extra = {}
    for key, fn_ in (("quantize", lambda: quantize_bench(nv, max(5, args.steps), 3, flush)),
                     ("gemm_decode", lambda: decode_bench(nv, max(5, args.steps), 3, flush)),
                     ("gemm_quantize", lambda: gemm_quantize_bench(nv, min(max(5, args.steps), 20), flush))):
        try:
            extra[key] = fn_()
        except Exception as e:  # reported, not fatal
            extra[key] = {"error": str(e)}

    cpu = None
    if not args.no_cpu_baseline:
        cpu = cpu_baseline_gemm()
        for key, fn_ in (("quantize", cpu_baseline_quantize), ("allreduce_cpu_baseline", cpu_baseline_allreduce)):
            try:
                res = fn_()
            except Exception as e:  # reported, not fatal
                res = {"error": str(e)}
            if key == "quantize":
                if isinstance(extra.get("quantize"), dict):
                    extra["quantize"]["cpu_baseline"] = res
            else:
                extra[key] = res

    fp4_tf = fp4.get("tflops") if isinstance(fp4, dict) else None
    peak = fp4_tf if fp4_tf else bf16x4
    roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4),
                "peak_source": ("FP4 MMA issue rate measured live on this GPU (peak_measured_fp4)" if fp4_tf else
                                f"4 x {peak_kind} cuBLAS bf16 burst (no live FP4 measurement)"),
                "peak_measured_fp4": fp4,
                "frac_of_measured_fp4": round(achieved / fp4_tf, 4) if fp4_tf else None,
                "peak_4x_bf16_burst": round(bf16x4, 1),
                "frac_of_4x_bf16_burst": round(achieved / bf16x4, 4),
                "frac_of_nominal_fp4_9000": round(achieved / FP4_NOMINAL_TFLOPS, 4),
                "traffic": read_profile_traffic("gemm_cfg3"),
                "algorithmic_flops_per_launch": flops}
    line = {
        "metric": METRIC,
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
                   "parallelism": "single GPU",
                   "l2": "flushed between timed steps (256 MB write, then 256 MB read)",
                   "timing": "CUDA events around each step's launch; the GPU clock is power-limited under this load "
                             "(the same kernel measures 196.5 us per launch in ncu's serialised launch list)",
                   "tile": "CTA pair (tcgen05 cta_group::2) 256x256, BK=256, 5 stages, persistent"},
        "roofline": roofline,
        "e2e": {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOPS",
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                "path": "pinned host A/B/SF -> device, nvfp4_gemm_bf16, device D -> pinned host; steps pipelined "
                        "over two buffer sets (copies of neighbouring steps overlap the GEMM)"},
        "gpu_launches": args.steps,
        "clocks": clocks,
        **extra,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def pipelined_e2e(host_in, dev_sets, host_out, step_fn, n_steps, world=1):
    """End-to-end steps through a public entry point with host buffers: per step, H2D copies of
    `host_in` into one of two device buffer sets, step_fn(dev_set, stream), and a D2H copy of the
    set's last tensor into host_out; copies of neighbouring steps overlap the step on three
    streams.  Returns ms per step (device events around the whole run, max over ranks)."""
    import torch
    s_in, s_mm, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()

    def run(n):
        done_out = [None, None]                       # D2H of the step that last used a buffer set
        for i in range(n):
            j = i & 1
            dev = dev_sets[j]
            ev_in = torch.cuda.Event()
            with torch.cuda.stream(s_in):
                if done_out[j] is not None:
                    s_in.wait_event(done_out[j])
                for h, dv in zip(host_in, dev):
                    dv.copy_(h, non_blocking=True)
                ev_in.record(s_in)
            ev_mm = torch.cuda.Event()
            with torch.cuda.stream(s_mm):
                s_mm.wait_event(ev_in)
                step_fn(dev, s_mm)
                ev_mm.record(s_mm)
            ev_out = torch.cuda.Event()
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_mm)
                host_out[j].copy_(dev[-1], non_blocking=True)
                ev_out.record(s_out)
            done_out[j] = ev_out

    run(3)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(HIDE_HOST_CYCLES * 8)
    e0.record()
    for st in (s_in, s_mm, s_out):
        st.wait_stream(torch.cuda.current_stream())
    run(n_steps)
    for st in (s_in, s_mm, s_out):
        torch.cuda.current_stream().wait_stream(st)
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(e0.elapsed_time(e1) / n_steps, world)


NVLINK_PEER_GBS = 770.0      # measured peer copy per direction per GPU on this pool
NVLINK_NOMINAL_GBS = 900.0   # NVLink 5, per direction per GPU


def _ar_time(fn, steps, warmup, flush, world):
    """Per-call device time (ms) of an all-reduce, max over ranks of the per-rank mean."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    fn()                      # untimed: its own barrier lines up the GPUs' timelines
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


ROT_BYTES = 192 << 20     # inputs rotated through by back-to-back timed calls: more than the 126 MB L2


def rotating_inputs(x, min_bytes=ROT_BYTES):
    """Copies of x at distinct places of one buffer of at least min_bytes (more than L2): calls
    that take them in turn read their input from HBM, as after an L2 flush, with neither a flush
    nor a host gap between calls.  Every copy holds x, so every call computes the same result."""
    n = x.numel()
    sets = max(2, -(-min_bytes // (x.element_size() * n)))
    buf = x.reshape(1, -1).expand(sets, -1).contiguous()
    return [buf[i] for i in range(sets)]


def _ar_time_rot(fn, xs, steps, warmup, world, sampler=None):
    """Per-call device time (ms) of `steps` back-to-back calls fn(xs[i % len(xs)]) between one
    pair of events, max over ranks: the reference harness's method (bench_ar.cu:965-972) with
    the input rotating through more than L2.  Barrier and synchronize on both sides; the GPU
    spins while the host queues the calls, and one untimed call lines the ranks up (every call
    meets its peers, whose clocks and queues differ), so the region holds device time only.
    With a sampler, it runs from before the first barrier to after the region."""
    import torch
    for i in range(warmup):
        fn(xs[i % len(xs)])
    if sampler is not None:
        sampler.start()
    torch.cuda.synchronize()
    barrier(world)
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(HIDE_HOST_CYCLES * max(1, steps // 4))
    fn(xs[-1])
    e0.record(s)
    for i in range(steps):
        fn(xs[i % len(xs)])
    e1.record(s)
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler is not None else None
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    return (ms, clocks) if sampler is not None else ms


def _wire_bytes(name, numel, world, payload_bytes_per_elt):
    """Bytes one rank sends over NVLink per call: two-shot 2 (n-1)/n of the payload, one-shot
    (n-1) times the payload."""
    two = "twoshot" in name or "nvls" in name          # NVLS: each shard's sum leaves and returns once
    return (2.0 * (world - 1) / world if two else (world - 1)) * payload_bytes_per_elt * numel


def _ar_entry(name, numel, world, ms, payload_bytes_per_elt):
    """bf16-equivalent algbw / busbw (nccl-tests convention) and wire rate of one algorithm."""
    t = ms * 1e-3
    algbw = 2.0 * numel / t / 1e9
    busbw = algbw * 2.0 * (world - 1) / world
    wire = _wire_bytes(name, numel, world, payload_bytes_per_elt)
    return {"us": round(ms * 1e3, 2), "algbw_gbs": round(algbw, 1), "busbw_gbs": round(busbw, 1),
            "wire_bytes_per_rank": int(wire), "wire_gbs_per_rank": round(wire / t / 1e9, 1),
            "frac_of_nvlink_770": round(wire / t / 1e9 / NVLINK_PEER_GBS, 4),
            "frac_of_nvlink_900": round(wire / t / 1e9 / NVLINK_NOMINAL_GBS, 4)}


ORACLE_AR = {"nvfp4_twoshot": "ar_twoshot", "nvfp4_oneshot": "ar_oneshot", "nvfp4_lowlat": "ar_oneshot",
             "bf16_twoshot": "ar_bf16", "bf16_oneshot": "ar_bf16"}


def ar_parity(ctx, x, out, gs, world, rank, windows=12, win=8192, nvls=False):
    """Bit-exact check of every algorithm against the CPU oracle (its fixed-order restatement of
    the two-shot / one-shot data flow) on sampled windows of the output.  A window of aligned
    16-element blocks depends only on the same window of every rank's input (quantization blocks,
    shard boundaries and requantization blocks are all aligned), so rank 0 gathers the ranks'
    input and output windows and runs the oracle on them.  The low-latency one-shot is checked on
    a prefix within its size cap."""
    import numpy as np
    import torch
    import torch.distributed as dist
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import py_oracle
    from tensorcore_ptx_example_b200 import allreduce as ar
    numel = x.numel()
    res = {"windows": windows, "window_elems": win}
    ok_all = True
    cases = [("nvfp4_twoshot", numel), ("nvfp4_oneshot", numel), ("bf16_twoshot", numel),
             ("bf16_oneshot", numel), ("nvfp4_lowlat", min(numel, ar.LOWLAT_CAP_BYTES // 2))]
    if nvls:
        cases.append(("bf16_nvls", numel))
    for name, n in cases:
        nw = min(windows, n // win)
        rng = np.random.default_rng(1234 + n)
        starts = np.sort(rng.choice(n // win, size=nw, replace=False)) * win
        idx = torch.from_numpy(np.concatenate([np.arange(s0, s0 + win) for s0 in starts])).cuda()
        xs, os_ = x[:n], out[:n]
        algo = name.split("_", 1)[1]
        if name.startswith("bf16"):
            ctx.bf16_allreduce(xs, os_, algo=algo)
        else:
            ctx.allreduce(xs, os_, global_scale=gs, algo=algo)
        xin = x[idx].contiguous()
        xout = out[idx].contiguous()
        ins = [torch.empty_like(xin) for _ in range(world)]
        outs = [torch.empty_like(xout) for _ in range(world)]
        dist.all_gather(ins, xin)
        dist.all_gather(outs, xout)
        ok = True
        if rank == 0 and name == "bf16_nvls":
            # the switch orders the fp32 additions: within 1 bf16 ulp of the exact sum, and the
            # same on every rank
            u16 = [t.view(torch.int16).cpu().numpy().view(np.uint16) for t in ins]
            exact = py_oracle.sum_f64(u16)
            got0 = outs[0].view(torch.int16).cpu().numpy().view(np.uint16)
            g = py_oracle.bf16_to_f32(got0).astype(np.float64)
            ulp = np.abs(py_oracle.bf16_to_f32(py_oracle.f32_to_bf16(exact.astype(np.float32)))) * 2.0 ** -7
            ok = bool(np.all(np.abs(g - exact) <= np.maximum(ulp, 2.0 ** -133)))
            for r in range(world):
                ok = ok and bool(np.array_equal(outs[r].view(torch.int16).cpu().numpy().view(np.uint16), got0))
        elif rank == 0:
            u16 = [t.view(torch.int16).cpu().numpy().view(np.uint16) for t in ins]
            fn = getattr(py_oracle, ORACLE_AR[name])
            want = fn(u16) if name.startswith("bf16") else fn(u16, gs)
            for r in range(world):
                got = outs[r].view(torch.int16).cpu().numpy().view(np.uint16)
                ok = ok and bool(np.array_equal(got, want))
        res[name] = ok
        ok_all = ok_all and ok
    torch.cuda.synchronize()
    flag = torch.tensor([1 if ok_all else 0], dtype=torch.int32, device="cuda")
    dist.broadcast(flag, 0)
    res["all"] = bool(flag.item())
    return res


def allreduce_algos(ctx, xs, out, gs, world, steps, nvls=False):
    """cfg4, every algorithm: device time per call of back-to-back calls over rotating inputs (max
    over ranks), and the NVFP4 error against the exact fp32 sum."""
    import torch
    import torch.distributed as dist
    x = xs[0]
    numel = x.numel()
    res = {}
    runs = [("nvfp4_twoshot", lambda xi: ctx.allreduce(xi, out, global_scale=gs, algo="twoshot"), 0.5625),
            ("nvfp4_oneshot", lambda xi: ctx.allreduce(xi, out, global_scale=gs, algo="oneshot"), 0.5625),
            ("bf16_twoshot", lambda xi: ctx.bf16_allreduce(xi, out, algo="twoshot"), 2.0),
            ("bf16_oneshot", lambda xi: ctx.bf16_allreduce(xi, out, algo="oneshot"), 2.0)]
    if nvls:
        runs.append(("bf16_nvls", lambda xi: ctx.bf16_allreduce(xi, out, algo="nvls"), 2.0))
    for name, fn, bpe in runs:
        res[name] = _ar_entry(name, numel, world, _ar_time_rot(fn, xs, steps, 3, world), bpe)
    exact = x.float().clone()
    dist.all_reduce(exact)
    for algo in ("twoshot", "oneshot"):
        o = ctx.allreduce(x, out, global_scale=gs, algo=algo).float()
        res[f"nvfp4_{algo}"]["rel_rmse_vs_fp32_sum"] = round(float((o - exact).norm() / exact.norm()), 5)
        res[f"nvfp4_{algo}"]["max_abs_err_vs_fp32_sum"] = round(float((o - exact).abs().max()), 4)
    torch.cuda.synchronize()
    return res, exact


SWEEP_ROWS_BYTES = [64 << 10, 1 << 20, 4 << 20, 16 << 20, 64 << 20, 256 << 20]


def ar_sweep_rows(ctx, xfull, ofull, gs, world, sizes=SWEEP_ROWS_BYTES, nvls=False):
    """cfg5 rows: every algorithm at each size, back-to-back calls (max over ranks); best NVFP4
    against best bf16."""
    from tensorcore_ptx_example_b200 import allreduce as ar
    rows = []
    for b in sizes:
        n = b // 2
        if n % (32 * world) or n > xfull.numel():
            continue
        x, o = xfull[:n], ofull[:n]
        calls = 50 if b <= (16 << 20) else 10
        algos = [("nvfp4_lowlat", lambda: ctx.allreduce(x, o, global_scale=gs, algo="lowlat")),
                 ("nvfp4_oneshot", lambda: ctx.allreduce(x, o, global_scale=gs, algo="oneshot")),
                 ("nvfp4_twoshot", lambda: ctx.allreduce(x, o, global_scale=gs, algo="twoshot")),
                 ("bf16_oneshot", lambda: ctx.bf16_allreduce(x, o, algo="oneshot")),
                 ("bf16_twoshot", lambda: ctx.bf16_allreduce(x, o, algo="twoshot"))]
        if nvls:
            algos.append(("bf16_nvls", lambda: ctx.bf16_allreduce(x, o, algo="nvls")))
        if b > ar.LOWLAT_CAP_BYTES:
            algos = algos[1:]
        row = {"bytes": b}
        for name, fn in algos:
            row[name + "_us"] = round(_ar_time_b2b(fn, calls, 3, world) * 1e3, 2)
        best_fp4 = min((k for k in row if k.startswith("nvfp4")), key=lambda k: row[k])
        best_bf16 = min((k for k in row if k.startswith("bf16")), key=lambda k: row[k])
        row["best_nvfp4"] = best_fp4[:-3]
        row["best_bf16"] = best_bf16[:-3]
        row["best_nvfp4_algbw_gbs"] = round(2.0 * n / (row[best_fp4] * 1e-6) / 1e9, 1)
        row["best_bf16_algbw_gbs"] = round(2.0 * n / (row[best_bf16] * 1e-6) / 1e9, 1)
        row["nvfp4_speedup_vs_bf16"] = round(row[best_bf16] / row[best_fp4], 3)
        rows.append(row)
    return rows


def reference_ar_kernels(world, rank, xs, gs, steps, exact):
    """Same-box baseline: the reference's own fused two-shot and one-shot kernels
    (launch_fused_rank / launch_oneshot_fused_rank, nvfp4_allreduce.cuh:650-682), compiled from
    the reference header into oracle/_ref/libref_ar.so, on the same GPUs and inputs (SFScaleVal =
    1 / gs), their buffers shared through CUDA IPC: device time per call (max over ranks) and
    error against the exact fp32 sum.  Each grid is the launcher's NVLink default capped at the
    blocks that are resident at once (the fused kernels' block barriers wait for the same block
    index on every rank).  Timed like this repository's kernels: back-to-back calls over the same
    rotating inputs.  Every rank takes the same steps; the kernels launch only after every
    rank has confirmed its buffers and peer mappings."""
    import ctypes

    import numpy as np
    import torch
    import torch.distributed as dist
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import py_oracle

    def all_ok(flag):
        t = torch.tensor([1 if flag else 0], dtype=torch.int32, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        return bool(t.item())

    def all_min(v):
        t = torch.tensor([int(v)], dtype=torch.int64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        return int(t.item())

    if not all_ok(py_oracle.ref_ar_available() and world in (2, 4, 8)):
        return {"unavailable": "oracle/_ref/libref_ar.so not built, or world not in {2, 4, 8}"}
    L = py_oracle.ref_ar_lib()
    x = xs[0]
    numel = x.numel()
    shard = numel // world
    sizes = {"comm2": L.ref_fused_comm_bytes(shard, world), "bin": 4 * L.ref_fused_barrier_words(world),
             "bout": 4 * L.ref_fused_barrier_words(world), "comm1": L.ref_oneshot_comm_bytes(numel, world),
             "bar1": 4 * L.ref_fused_barrier_words(world)}
    own, opened, arrays = {}, [], {}
    res = {}
    try:
        ok = True
        for k, nbytes in sizes.items():
            p = ctypes.c_void_p()
            ok = ok and L.ref_dev_alloc_zero(nbytes, ctypes.byref(p)) == 0
            own[k] = p
        if not all_ok(ok):
            return {"unavailable": "allocation failed"}
        hb = int(L.ref_ipc_handle_bytes())
        mine = {}
        for k, p in own.items():
            buf = ctypes.create_string_buffer(hb)
            ok = ok and L.ref_ipc_get(p, buf) == 0
            mine[k] = buf.raw
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        for k in sizes:
            ptrs = []
            for r in range(world):
                if r == rank:
                    ptrs.append(own[k].value)
                    continue
                q = ctypes.c_void_p()
                ok = ok and L.ref_ipc_open(gathered[r][k], ctypes.byref(q)) == 0
                opened.append(q)
                ptrs.append(q.value)
            arr = ctypes.c_void_p()
            host = (ctypes.c_void_p * world)(*ptrs)
            ok = ok and L.ref_dev_ptr_array(host, world, ctypes.byref(arr)) == 0
            arrays[k] = arr
        grid2 = min(int(L.ref_default_fused_grid(shard, 256)), int(L.ref_fused_resident_blocks(world, 0)))
        grid1 = min(int(L.ref_default_fused_grid(numel, 256)), int(L.ref_fused_resident_blocks(world, 1)))
        grid2, grid1 = all_min(grid2), all_min(grid1)
        if not all_ok(ok and grid2 > 0 and grid1 > 0):
            return {"unavailable": "IPC mapping or occupancy query failed"}
        torch.cuda.synchronize()
        out = torch.empty_like(x)
        sf_val = float(np.float32(1.0) / np.float32(gs))
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        op = ctypes.c_void_p(out.data_ptr())
        flags = {"two": 0, "one": 0}

        def twoshot(xi):
            flags["two"] += 1
            rc = L.ref_launch_twoshot(world, ctypes.c_void_p(xi.data_ptr()), op, arrays["comm2"], arrays["bin"], arrays["bout"], rank, numel,
                                      sf_val, flags["two"], st, grid2)
            if rc:
                raise RuntimeError(f"ref_launch_twoshot: cuda error {rc}")

        def oneshot(xi):
            flags["one"] += 1
            rc = L.ref_launch_oneshot(world, ctypes.c_void_p(xi.data_ptr()), op, arrays["comm1"], arrays["bar1"], rank, numel, sf_val,
                                      flags["one"], st, grid1)
            if rc:
                raise RuntimeError(f"ref_launch_oneshot: cuda error {rc}")

        for name, fn in (("reference_twoshot", twoshot), ("reference_oneshot", oneshot)):
            ms = _ar_time_rot(fn, xs, steps, 3, world)
            e = _ar_entry(name, numel, world, ms, 0.5625)
            fn(x)
            o = out.float()
            e["rel_rmse_vs_fp32_sum"] = round(float((o - exact).norm() / exact.norm()), 5)
            e["grid"] = grid2 if "two" in name else grid1
            res[name] = e
        torch.cuda.synchronize()
        res["kernels"] = "nvfp4_ar::twoshot_fused_kernel / oneshot_fused_kernel (reference, oracle/_ref/libref_ar.so)"
        return res
    finally:
        torch.cuda.synchronize()
        barrier(world)
        for q in opened:
            L.ref_ipc_close(q)
        for arr in arrays.values():
            L.ref_dev_free(arr)
        for p in own.values():
            if p.value:
                L.ref_dev_free(p)
        torch.cuda.synchronize()
        barrier(world)


def gemm_replicas(nv, world, rank, steps, flush):
    """Every rank runs its own cfg3 GEMM (independent replicas, no exchange): aggregate TFLOPS."""
    import torch
    pa, sa, pb, sb, alpha, d = gemm_setup(nv, rank)
    fn = lambda: nv.gemm(pa, sa, pb, sb, M_, N_, K_, alpha=alpha, out=d)  # noqa: E731
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    ts = timed_steps(fn, steps, flush)
    barrier(world)
    total = max_over_ranks(sum(ts), world)
    return {"workload": "cfg3 GEMM 8192^3 on every rank (replicas)", "steps": steps,
            "aggregate_tflops": round(2.0 * M_ * N_ * K_ * steps * world / (total * 1e-3) / 1e12, 1)}


def run_allreduce_line(args):
    """N > 1: the cfg4 NVFP4 all-reduce as the headline (see the module docstring)."""
    import torch

    import tensorcore_ptx_example_b200 as nv
    from tensorcore_ptx_example_b200 import allreduce as ar
    from tensorcore_ptx_example_b200 import workloads
    world, rank, local = dist_setup(args)
    flush = L2Flush()
    rows, cols = workloads.CFG4_SHAPE
    numel = rows * cols
    sweep_max = max(SWEEP_ROWS_BYTES) // 2
    x = workloads.gaussian(1, numel, seed=rank).view(-1)
    gs = ar.agree_global_scale(float(nv.amax(x).item()))
    ctx = ar.AllReduce.from_process_group(max(numel, sweep_max))
    nvls_error = None
    try:
        nvls = ctx.enable_nvls()          # in-switch bf16 baseline, where the GPUs offer multicast
    except Exception as e:  # reported, not fatal
        nvls, nvls_error = False, str(e)
    out = torch.empty_like(x)
    algo = {ar.ONESHOT: "oneshot", ar.TWOSHOT: "twoshot", ar.LOWLAT: "lowlat"}[ar.choose_algo(world, numel)]
    extra = {}
    try:
        # K back-to-back steps over copies of the input that together exceed L2 (each step
        # reads its input from HBM); the sampler starts before the barrier (its NVML set-up takes
        # a varying while on each rank)
        xs = rotating_inputs(x)
        nsets = len(xs)
        fn = lambda xi: ctx.allreduce(xi, out, global_scale=gs, algo="auto")  # noqa: E731
        mean_ms, clocks = _ar_time_rot(fn, xs, args.steps, args.warmup, world, sampler=ClockSampler(local))
        total_ms = mean_ms * args.steps
        status = nv.device_status()
        value = 2.0 * numel * args.steps / (total_ms * 1e-3) / 1e9
        wire = _wire_bytes(algo, numel, world, 0.5625)
        achieved = wire / (mean_ms * 1e-3) / 1e9

        parity = ar_parity(ctx, x, out, gs, world, rank, nvls=nvls)
        algos, exact = allreduce_algos(ctx, xs, out, gs, world, max(5, min(args.steps, 20)), nvls=nvls)

        # end to end through the public API with host buffers: the input copied from pinned
        # host memory and the result copied back every step (pipelined like the GEMM's)
        hx = x.cpu().pin_memory()
        dev_sets = [(x, out), (torch.empty_like(x), torch.empty_like(x))]
        host_out = [torch.empty_like(hx).pin_memory() for _ in range(2)]
        e2e_steps = max(4, min(args.steps, 12))
        e2e_ms = pipelined_e2e([hx], dev_sets, host_out,
                               lambda dev, s: ctx.allreduce(dev[0], dev[1], global_scale=gs, algo="auto", stream=s),
                               e2e_steps, world)
        ok_e2e = bool(torch.equal(host_out[(e2e_steps - 1) & 1], out.cpu()))

        xfull = workloads.gaussian(1, sweep_max, seed=100 + rank).view(-1)
        gs_sweep = ar.agree_global_scale(float(nv.amax(xfull).item()))
        ofull = torch.empty_like(xfull)
        sweep = ar_sweep_rows(ctx, xfull, ofull, gs_sweep, world, nvls=nvls)
        del xfull, ofull
        status = status or nv.device_status()
    finally:
        torch.cuda.synchronize()
        barrier(world)
        ctx.close()
    for key, fn_ in (("gemm_allreduce", lambda: gemm_allreduce_bench(nv, world, rank, args, flush=flush)),
                     ("gemm_replicas", lambda: gemm_replicas(nv, world, rank, 10, flush))):
        extra[key] = fn_()
    # the reference's kernels last: they wait without a time limit, so they run only after every
    # measurement of ours is in
    extra["reference_kernels"] = reference_ar_kernels(world, rank, xs, gs, max(5, min(args.steps, 20)), exact)
    del xs

    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16 in/out; NVFP4 (e2m1 + ue4m3 per 16) on the wire; fp32 sums in rank order",
        "data": "synthetic (seeded N(0,1) bf16 per rank, seed = rank)",
        "config": {"workload": f"cfg4 NVFP4 all-reduce, {rows}x{cols} bf16 per rank", "numel_per_rank": numel,
                   "algorithm": f"NVFP4_AR_AUTO -> {algo}", "parallelism": f"all-reduce over {world} GPUs (NVLink P2P)",
                   "value_convention": "bf16-equivalent algbw = 2 * numel_per_rank / t (nccl-tests)",
                   "l2": f"inputs larger than L2: back-to-back steps rotate through {nsets} copies of the "
                         f"58.7 MB input ({nsets * numel * 2 / 1e6:.0f} MB per rank), one event pair around K steps"},
        "busbw_gbs": round(value * 2.0 * (world - 1) / world, 1),
        "roofline": {"bound": "nvlink", "achieved": round(achieved, 1), "peak": NVLINK_PEER_GBS, "unit": "GB/s",
                     "frac": round(achieved / NVLINK_PEER_GBS, 4),
                     "frac_of_900": round(achieved / NVLINK_NOMINAL_GBS, 4),
                     "peak_source": "measured peer copy per direction per GPU on this pool (900 nominal)",
                     "achieved_is": "wire bytes one rank sends per call / mean call time",
                     "wire_bytes_per_launch": int(wire), "traffic": None},
        "parity_ok": parity["all"],
        "parity": parity,
        "nvls": nvls if nvls_error is None else {"error": nvls_error},
        "device_status": status,
        "algorithms": algos,
        "sweep_rows": sweep,
        "e2e": {"value": round(2.0 * numel / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": numel * 2, "d2h_bytes_per_step": numel * 2, "result_matches": ok_e2e,
                "path": "pinned host bf16 -> device, nvfp4_ar_allreduce (AUTO), device -> pinned host; steps "
                        "pipelined over two buffer sets"},
        "gpu_launches": args.steps,
        "clocks": clocks,
        **extra,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    import torch.distributed as dist
    dist.destroy_process_group()


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
    """cfg5: 16 KB .. 256 MB of bf16 per rank (doubling): NVFP4 low-latency one-shot (up to 1 MB),
    one-shot and two-shot against the bf16 one-shot, two-shot and (where the GPUs offer NVLink
    multicast) in-switch NVLS all-reduce; max over ranks of the mean device time per call over
    back-to-back calls."""
    import torch

    import tensorcore_ptx_example_b200 as nv
    from tensorcore_ptx_example_b200 import allreduce as ar
    from tensorcore_ptx_example_b200 import workloads
    world, rank, local = dist_setup(args)
    sizes = [b for b in workloads.sweep_sizes_bytes() if (b // 2) % (32 * world) == 0]
    max_numel = max(sizes) // 2
    ctx = ar.AllReduce.from_process_group(max_numel)
    try:
        nvls = ctx.enable_nvls()
        xfull = workloads.gaussian(1, max_numel, seed=rank).view(-1)
        gs = ar.agree_global_scale(float(nv.amax(xfull).item()))
        ofull = torch.empty_like(xfull)
        rows = ar_sweep_rows(ctx, xfull, ofull, gs, world, sizes=sizes, nvls=nvls)
        torch.cuda.synchronize()
        status = nv.device_status()
    finally:
        barrier(world)
        ctx.close()
    if rank == 0:
        print(json.dumps({"sweep": "cfg5 all-reduce message sizes", "world": world, "device_status": status,
                          "nvls": nvls, "l2": "not flushed (back-to-back calls)", "rows": rows}), flush=True)
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
    """The reference arm: the reference's CPU path on rank 0 (the other ranks exit without work),
    on this line's metric and config, each step a bounded sample."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    vals = []
    res = None
    if world > 1:
        sample = CpuAllReduceSample(world)
        for i in range(args.warmup + args.steps):
            res = sample.measure(target_s=0.5)
            if i >= args.warmup:
                vals.append(res["value"])
        unit = "GB/s"
        config = {"workload": "cfg4 NVFP4 all-reduce, 4096x7168 bf16 per rank (bounded CPU sample per step)",
                  "numel_per_rank": 4096 * 7168, "ranks": world,
                  "value_convention": "bf16-equivalent algbw = 2 * numel_per_rank / t (nccl-tests)"}
        dtype = "fp32 sums in rank order (CPU restatement of the NVFP4 two-shot; the reference has no CPU all-reduce)"
        data = "synthetic (seeded N(0,1) bf16 per rank)"
    else:
        for i in range(args.warmup + args.steps):
            res = cpu_baseline_gemm(target_s=2.0)
            if i >= args.warmup:
                vals.append(res["value"])
        unit = "TFLOPS"
        config = {"workload": "cfg3 NVFP4 GEMM M=N=K=8192 (bounded CPU sample per step)", "M": M_, "N": N_, "K": K_}
        dtype = "fp32 (reference CPU path on decoded E2M1 values)"
        data = "synthetic (seeded E2M1 values)"
    v = sum(vals) / len(vals)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": v, "unit": unit, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": dtype, "data": data, "config": config,
        "cpu_baseline": {"value": v, "unit": unit, "cores": res["cores"], "kind": res["kind"],
                         "sample": res["sample"]},
        "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
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
        # and the dequantizer over the same shape (cfg2 round trip)
        from tensorcore_ptx_example_b200 import workloads
        rows, cols = workloads.CFG2_SHAPE
        x = workloads.activations(rows, cols, seed=2)
        gs = float(nv.amax(x).item()) / 2688.0
        packed, sf, _ = nv.quantize(x, gs)
        y = torch.empty_like(x)
        for _ in range(args.warmup):
            nv.dequantize(packed, sf, rows, cols, gs, out=y)
        ts = timed_steps(lambda: nv.dequantize(packed, sf, rows, cols, gs, out=y), args.steps, flush)
        ms = sum(ts) / len(ts)
        out["dequantize_us"] = round(ms * 1e3, 2)
        out["dequantize_gbs"] = round(rows * cols * 2.5625 / (ms * 1e-3) / 1e9, 1)
    elif args.only == "gemm-decode":
        shape = tuple(int(v) for v in args.shape.split("x")) if args.shape else None
        out = decode_bench(nv, args.steps, args.warmup, flush, shape=shape)
    elif args.only == "mma-peak":
        # the FP4 MMA issue-rate probe alone (the GEMM's roofline), with its in-kernel SM clock
        from tensorcore_ptx_example_b200 import diag
        diag.mma_peak_clock()
        tf = diag.mma_peak(cta_group=2, iters=32768, repeats=max(1, args.steps), random_operands=True)
        out = {"workload": "FP4 MMA issue-rate probe (nvfp4_diag_mma_peak, cta_group 2, 32768 MMAs per pair)",
               "tflops": round(tf, 1), "sm_mhz_in_kernel": round(diag.mma_peak_clock(), 1)}
    elif args.only == "gemm-quantize":
        out = gemm_quantize_bench(nv, args.steps, flush)
    elif args.only == "ar-emulated":
        # the all-reduce data path of 8 ranks on this one GPU, phase by phase (no cross-GPU
        # waits): for profiling the phase kernels' memory traffic on a single device.  NVFP4
        # two-shot and one-shot, the low-latency one-shot (on its 1 MB cap), bf16 two-shot and
        # one-shot, in that order.
        from tensorcore_ptx_example_b200 import allreduce as ar
        from tensorcore_ptx_example_b200 import workloads
        world, numel = 8, args.numel
        ins = [workloads.gaussian(1, numel, seed=r).view(-1) for r in range(world)]
        gs = nv.global_scale_from_amax(max(float(nv.amax(x).item()) for x in ins))
        ctxs = [ar.AllReduce(world, r, numel) for r in range(world)]
        ar.join_in_process(ctxs)
        ll = min(numel, ar.LOWLAT_CAP_BYTES // 2)
        for algo, bf16, n in (("twoshot", False, numel), ("oneshot", False, numel), ("lowlat", False, ll),
                              ("twoshot", True, numel), ("oneshot", True, numel)):
            for _ in range(args.warmup + args.steps):
                ar.emulated_allreduce([x[:n] for x in ins], gs, algo, bf16=bf16, contexts=ctxs)
        torch.cuda.synchronize()
        for c in ctxs:
            c.close()
        out = {"workload": f"emulated 8-rank all-reduce, {numel} elements per rank", "launches_per_call":
               "nvfp4 twoshot 3 phases x 8 ranks, oneshot 2 x 8, lowlat 2 x 8, then bf16 twoshot / oneshot"}
    elif args.only == "gemm-ar-emulated":
        # the row-parallel GEMM + two-shot of 2 ranks on this one GPU (cfg4 output, K 4096 per
        # rank): gemm2_kernel with the payload epilogue, then the all-reduce phases
        from tensorcore_ptx_example_b200 import allreduce as ar
        from tensorcore_ptx_example_b200 import workloads
        world = 2
        M, N = workloads.CFG4_SHAPE
        K = 8192 // world
        ops, alphas, ds = [], [], []
        for r in range(world):
            pa, sa, gsa = nv.quantize(workloads.activations(M, K, seed=11 + 2 * r), None)
            pb, sb, gsb = nv.quantize(workloads.gaussian(N, K, seed=12 + 2 * r, std=0.02), None)
            ops.append((pa, sa, pb, sb))
            alphas.append(float(gsa.item()) * float(gsb.item()))
            ds.append(nv.gemm(pa, sa, pb, sb, M, N, K, alpha=alphas[-1]))
        gs = nv.global_scale_from_amax(max(float(d.float().abs().max()) for d in ds))
        ctxs = [ar.AllReduce(world, r, M * N) for r in range(world)]
        ar.join_in_process(ctxs)
        for _ in range(args.warmup + args.steps):
            ar.emulated_gemm_allreduce(ops, M, N, K, alphas, gs, ctxs)
        torch.cuda.synchronize()
        for c in ctxs:
            c.close()
        out = {"workload": f"emulated 2-rank row-parallel GEMM M{M} N{N} K{K} per rank + two-shot"}
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
    ap.add_argument("--only", choices=["gemm", "gemm-decode", "gemm-quantize", "quantize", "ar-sweep", "ar-emulated",
                                       "gemm-ar-emulated", "mma-peak"],
                    default=None,
                    help="profiling mode: run one workload (warmup + steps launches) and print its "
                         "timings; not the benchmark line")
    ap.add_argument("--shape", default=None,
                    help="with --only gemm-decode: MxNxK instead of cfg3's decode shape (e.g. 16x1024x16384, "
                         "which takes the workspace split-K path)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.only == "ar-sweep":
        allreduce_sweep(args)
    elif args.only:
        run_only(args)
    elif args.impl == "reference":
        run_reference(args)
    elif int(os.environ.get("WORLD_SIZE", "1")) > 1:
        run_allreduce_line(args)
    else:
        run_gemm_line(args)


if __name__ == "__main__":
    main()
