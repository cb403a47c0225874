"""NVFP4-compressed all-reduce across the GPUs of one node (host side).

Python mirror of the all-reduce part of include/nvfp4.h.  One `AllReduce` context per rank,
created on that rank's GPU.  Two ways to join the ranks:

* one process per GPU (torchrun): `AllReduce.from_process_group(max_numel)` exchanges the CUDA
  IPC handles of every rank's buffer through `torch.distributed.all_gather_object` (any
  backend; gloo is enough) and opens the peers' buffers;
* one process driving all GPUs (the reference harness, bench_ar.cu:763-850): create one context
  per device and call `join_in_process(contexts)`.

The reduction itself runs in the library's kernels over NVLink / NVSwitch peer memory; torch
only provides device memory, streams and the handle exchange.  Every rank must issue the same
sequence of calls (same numel, algo and order).

Reference: nvfp4_ar::launch_fused_rank / launch_oneshot_fused_rank
(blackwell/allreduce_sm100_sm120/nvfp4_allreduce.cuh:650-682).
"""
from __future__ import annotations

import ctypes

from . import _empty, _ptr, _stream, check, lib

AUTO, ONESHOT, TWOSHOT, LOWLAT, NVLS = 0, 1, 2, 3, 4
LOWLAT_CAP_BYTES = 1 << 20          # NVFP4_AR_LOWLAT_CAP_BYTES: largest low-latency call (bf16 bytes)
_ALGOS = {"auto": AUTO, "oneshot": ONESHOT, "twoshot": TWOSHOT, "lowlat": LOWLAT, "nvls": NVLS,
          AUTO: AUTO, ONESHOT: ONESHOT, TWOSHOT: TWOSHOT, LOWLAT: LOWLAT, NVLS: NVLS}


def buffer_bytes(world: int, max_numel: int) -> int:
    """Device bytes one context allocates."""
    return int(lib().nvfp4_ar_buffer_bytes(world, max_numel))


def choose_algo(world: int, numel: int) -> int:
    return int(lib().nvfp4_ar_choose_algo(world, numel))


def _algo(a) -> int:
    if a not in _ALGOS:
        raise ValueError(f"algo must be one of auto/oneshot/twoshot/lowlat/nvls, got {a!r}")
    return _ALGOS[a]


class AllReduce:
    """One rank's all-reduce context (owns its communication buffers on the current GPU)."""

    def __init__(self, world: int, rank: int, max_numel: int):
        import torch
        self.world, self.rank, self.max_numel = int(world), int(rank), int(max_numel)
        self.device = torch.cuda.current_device()
        h = ctypes.c_void_p()
        check(lib().nvfp4_ar_create(self.world, self.rank, self.max_numel, ctypes.byref(h)))
        self._h = h
        self._nvls = None

    # ------------------------------------------------------------ set-up ----
    @property
    def handle(self) -> ctypes.c_void_p:
        if self._h is None:
            raise RuntimeError("all-reduce context is closed")
        return self._h

    def export_handle(self) -> bytes:
        n = int(lib().nvfp4_ar_handle_bytes())
        buf = ctypes.create_string_buffer(n)
        check(lib().nvfp4_ar_export_handle(self.handle, buf))
        return buf.raw

    def open_peers(self, handles) -> None:
        """handles: every rank's export_handle() bytes, in rank order."""
        n = int(lib().nvfp4_ar_handle_bytes())
        if len(handles) != self.world or any(len(x) != n for x in handles):
            raise ValueError(f"need {self.world} handles of {n} bytes")
        blob = ctypes.create_string_buffer(b"".join(handles), n * self.world)
        check(lib().nvfp4_ar_open_peers(self.handle, blob))

    def local_base(self) -> int:
        p = ctypes.c_void_p()
        check(lib().nvfp4_ar_local_base(self.handle, ctypes.byref(p)))
        return int(p.value)

    def set_peers(self, bases) -> None:
        arr = (ctypes.c_void_p * self.world)(*[ctypes.c_void_p(int(b)) for b in bases])
        check(lib().nvfp4_ar_set_peers(self.handle, arr))

    def enable_nvls(self, group=None) -> bool:
        """Give this context a buffer bound to an NVLink multicast object, for the in-switch bf16
        all-reduce (bf16_allreduce(..., algo="nvls")).  Collective over `group` (every rank calls
        it): torch symmetric memory allocates the buffer and binds every rank's to one multicast
        object; this library only receives the two addresses.  Returns False on every rank (and
        leaves NVLS off) when any rank's GPU or driver offers no multicast."""
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm
        group = group or dist.group.WORLD
        nbytes = 2 * ((self.max_numel * 2 + 15) // 16 * 16)
        buf = symm.empty(nbytes, dtype=torch.uint8, device=torch.device("cuda", self.device))
        hdl = symm.rendezvous(buf, group)
        mc = int(hdl.multicast_ptr or 0)         # 0 when the device offers no NVLink multicast
        backend = dist.get_backend(group)
        dev = torch.device("cuda", self.device) if backend == "nccl" else torch.device("cpu")
        ok = torch.tensor([1 if mc else 0], dtype=torch.int32, device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if not int(ok.item()):
            return False
        check(lib().nvfp4_ar_set_multicast(self.handle, ctypes.c_void_p(mc), ctypes.c_void_p(buf.data_ptr()),
                                           nbytes))
        self._nvls = (buf, hdl)          # keep the buffer and its mapping alive with the context
        return True

    def set_timeout(self, seconds: float) -> None:
        check(lib().nvfp4_ar_set_timeout(self.handle, int(seconds * 1e9)))

    def reset(self) -> None:
        """After a timed-out call: clear this rank's barrier words and epoch.  Every rank must
        reset, with no all-reduce in flight anywhere, before the next call."""
        check(lib().nvfp4_ar_reset(self.handle))

    @classmethod
    def from_process_group(cls, max_numel: int, group=None) -> "AllReduce":
        """Context for this process's rank of `group`, joined with the other ranks through
        CUDA IPC handles gathered over torch.distributed."""
        import torch.distributed as dist
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        ctx = cls(world, rank, max_numel)
        handles = exchange(ctx.export_handle(), world, group)
        ctx.open_peers(handles)
        dist.barrier(group)
        return ctx

    # ------------------------------------------------------------- calls ----
    def allreduce(self, x, out=None, global_scale: float = None, algo="auto", stream=None):
        """NVFP4 all-reduce of a contiguous bf16 CUDA tensor (numel % (32 * world) == 0).
        global_scale: gs = amax / (6 * 448), the same on every rank (see agree_global_scale).
        algo: "oneshot", "twoshot", "lowlat" (one-shot with flags carried in the data, no
        barrier; same results as "oneshot"; at most LOWLAT_CAP_BYTES of bf16) or "auto"."""
        import torch
        if global_scale is None:
            raise ValueError("global_scale is required (the same on every rank)")
        assert x.dtype == torch.bfloat16 and x.is_cuda and x.is_contiguous()
        if out is None:
            out = _empty(x.shape, x.dtype, x.device, stream)
        check(lib().nvfp4_ar_allreduce(self.handle, _ptr(x), _ptr(out), x.numel(), ctypes.c_float(global_scale),
                                       _algo(algo), _stream(stream)))
        return out

    def gemm_allreduce(self, a_packed, sfa, b_packed, sfb, M: int, N: int, K: int, alpha: float,
                       global_scale: float, out=None, stream=None):
        """Row-parallel NVFP4 GEMM fused with the two-shot all-reduce: every rank passes its K
        shard (A_r [M, K], B_r [N, K] packed, scales in the tcgen05 layout) and gets
        sum_r bf16(alpha_r A_r B_r^T) reduced through NVFP4, the bytes of gemm() followed by
        allreduce(algo="twoshot").  global_scale: the same on every rank."""
        import torch
        if out is None:
            out = _empty((M, N), torch.bfloat16, a_packed.device, stream)
        check(lib().nvfp4_gemm_allreduce(self.handle, _ptr(a_packed), _ptr(sfa), _ptr(b_packed), _ptr(sfb),
                                         ctypes.c_float(alpha), ctypes.c_float(global_scale), _ptr(out), M, N, K,
                                         _stream(stream)))
        return out

    def bf16_allreduce(self, x, out=None, algo="auto", stream=None):
        """In-house bf16 all-reduce (numel % (8 * world) == 0): peer-to-peer ("oneshot",
        "twoshot", "auto") or summed in the NVSwitch ("nvls", after enable_nvls)."""
        import torch
        assert x.dtype == torch.bfloat16 and x.is_cuda and x.is_contiguous()
        if out is None:
            out = _empty(x.shape, x.dtype, x.device, stream)
        check(lib().nvfp4_ar_bf16_allreduce(self.handle, _ptr(x), _ptr(out), x.numel(), _algo(algo),
                                            _stream(stream)))
        return out

    def close(self) -> None:
        if self._h is not None:
            check(lib().nvfp4_ar_destroy(self._h))
            self._h = None
        self._nvls = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def exchange(blob: bytes, world: int, group=None) -> list:
    """Every rank's `blob`, in rank order (host-side all-gather over torch.distributed)."""
    import torch.distributed as dist
    out = [None] * world
    dist.all_gather_object(out, blob, group=group)
    return list(out)


def agree_global_scale(local_amax: float, group=None) -> float:
    """The global scale every rank uses: gs = max over ranks of amax / (6 * 448), computed on the
    host from the ranks' amax values (a max all-reduce of one float over torch.distributed)."""
    import torch
    import torch.distributed as dist

    from . import global_scale_from_amax
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.tensor([float(local_amax)], dtype=torch.float32, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return global_scale_from_amax(float(t.item()))


def join_in_process(contexts) -> None:
    """Join contexts that one process created on different GPUs (or, for emulation, on one GPU)."""
    import torch
    bases = []
    for c in contexts:
        with torch.cuda.device(c.device):
            bases.append(c.local_base())
    for c in contexts:
        with torch.cuda.device(c.device):
            c.set_peers(bases)


def emulated_allreduce(inputs, global_scale: float = 1.0, algo="auto", bf16: bool = False, contexts=None,
                       stream=None):
    """Run the all-reduce data path for len(inputs) ranks that all live on the current GPU
    (phase by phase, rank by rank; no kernel waits for another).  Returns the per-rank outputs.
    For checking the arithmetic on one GPU."""
    import torch
    world = len(inputs)
    numel = inputs[0].numel()
    own = contexts is None
    if own:
        contexts = [AllReduce(world, r, numel) for r in range(world)]
        join_in_process(contexts)
    try:
        outs = [_empty(x.shape, x.dtype, x.device, stream) for x in inputs]
        hs = (ctypes.c_void_p * world)(*[c.handle for c in contexts])
        ins = (ctypes.c_void_p * world)(*[ctypes.c_void_p(x.data_ptr()) for x in inputs])
        os_ = (ctypes.c_void_p * world)(*[ctypes.c_void_p(o.data_ptr()) for o in outs])
        check(lib().nvfp4_ar_allreduce_emulated(hs, world, ins, os_, numel, ctypes.c_float(global_scale),
                                                _algo(algo), 1 if bf16 else 0, _stream(stream)))
        return outs
    finally:
        if own:
            torch.cuda.synchronize()
            for c in contexts:
                c.close()


def emulated_gemm_allreduce(operands, M: int, N: int, K: int, alphas, global_scale: float, contexts, stream=None):
    """nvfp4_gemm_allreduce for len(operands) ranks on the current GPU: operands[r] =
    (a_packed, sfa, b_packed, sfb) of rank r.  Returns the per-rank outputs."""
    import torch
    world = len(operands)
    outs = [_empty((M, N), torch.bfloat16, operands[0][0].device, stream) for _ in range(world)]

    def arr(i):
        return (ctypes.c_void_p * world)(*[ctypes.c_void_p(op[i].data_ptr()) for op in operands])

    hs = (ctypes.c_void_p * world)(*[c.handle for c in contexts])
    al = (ctypes.c_float * world)(*[float(a) for a in alphas])
    os_ = (ctypes.c_void_p * world)(*[ctypes.c_void_p(o.data_ptr()) for o in outs])
    check(lib().nvfp4_gemm_allreduce_emulated(hs, world, arr(0), arr(1), arr(2), arr(3), al,
                                              ctypes.c_float(global_scale), os_, M, N, K, _stream(stream)))
    return outs
