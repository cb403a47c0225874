"""All-reduce: oracle pins and host-side logic (CPU only).

* The oracle's NVFP4 one-shot / two-shot sums reproduce the accuracy the reference publishes for
  its own kernels (blackwell/allreduce_sm100_sm120/README.md, "Results": rel_rmse vs the fp32
  sum, 8 ranks, U[-1, 1] inputs, global scale from rank 0's amax -- one-shot 0.102, two-shot
  0.1398; harness bench_ar.cu:776-778, :878).  A statistical pin: the reference's rand() stream
  is libc-specific, so the inputs are drawn from another generator with the same distribution.
* Buffer sizing, algorithm choice and argument checks of the C ABI (no GPU work).
* The multi-process set-up (handle exchange, global-scale agreement) on world_size-2 gloo ranks.
"""
import ctypes
import os
import socket

import numpy as np
import pytest


def _bf16(a):
    u = a.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _f32(u):
    return (u.astype(np.uint32) << 16).view(np.float32)


def _rel_rmse(out_u16, ref):
    e = _f32(out_u16).astype(np.float64) - ref.astype(np.float64)
    return float(np.sqrt((e * e).sum() / ((ref.astype(np.float64) ** 2).sum() + 1e-12)))


def test_oracle_allreduce_matches_published_accuracy(oracle):
    world, numel = 8, 1 << 20
    rng = np.random.default_rng(1234)
    hin = [(rng.random(numel, dtype=np.float32) * 2 - 1).astype(np.float32) for _ in range(world)]
    ref = np.zeros(numel, np.float32)
    for h in hin:
        ref += h
    ins = [_bf16(h) for h in hin]
    gs = float(np.float32(np.abs(hin[0]).max()) / np.float32(2688.0))    # SFScaleVal = 1 / gs
    one = _rel_rmse(oracle.ar_oneshot(ins, gs), ref)
    two = _rel_rmse(oracle.ar_twoshot(ins, gs), ref)
    assert abs(one - 0.102) < 0.002, one
    assert abs(two - 0.1398) < 0.002, two
    # fixed-order fp32 sum then one bf16 rounding: far below the NVFP4 error
    assert _rel_rmse(oracle.ar_bf16(ins), ref) < 0.004


def test_oracle_allreduce_order_and_determinism(oracle):
    """Rank order matters (fp32 sums are not associative) and the oracle follows 0..n-1."""
    rng = np.random.default_rng(7)
    ins = [_bf16(rng.standard_normal(4096).astype(np.float32) * (10.0 ** (r % 3))) for r in range(4)]
    gs = 100.0 / 2688.0
    a = oracle.ar_oneshot(ins, gs)
    assert np.array_equal(a, oracle.ar_oneshot(ins, gs))
    # the fp32 sum in the oracle's order, recomputed here from decoded values
    acc = np.zeros(4096, np.float32)
    for x in ins:
        acc = (acc + _f32(x)).astype(np.float32)
    assert np.array_equal(oracle.ar_bf16(ins), _bf16(acc))


def test_buffer_bytes_and_algo_choice(nv):
    L = nv.lib()
    # flags (1024 blocks x 8 ranks x 4 B) + 2 parities x (world IN slots + world GATHER slots)
    # + 2 parities x world low-latency slots (3 u64 words per 32 elements, up to 512 K elements)
    numel, world = 1 << 20, 8
    in_slot = max(numel // 2 + numel // 16, numel * 2)
    gather = max((numel // world) // 2 + (numel // world) // 16, (numel // world) * 2)
    ll_slot = min(numel, 1 << 19) // 32 * 24
    assert L.nvfp4_ar_buffer_bytes(world, numel) == (1024 * 8 * 4 + 2 * (world * in_slot + world * gather)
                                                     + 2 * world * ll_slot)
    assert L.nvfp4_ar_buffer_bytes(0, numel) == -1 and L.nvfp4_ar_buffer_bytes(9, numel) == -1
    assert L.nvfp4_ar_choose_algo(1, 1 << 30) == 1
    assert L.nvfp4_ar_choose_algo(8, 1024) == 3                      # small: low-latency one-shot
    assert L.nvfp4_ar_choose_algo(8, (1 << 20) // 2) == 3
    assert L.nvfp4_ar_choose_algo(8, (1 << 20) // 2 + 256) == 1
    assert L.nvfp4_ar_choose_algo(8, (2 << 20) // 2) == 1          # 2 MB of bf16: one-shot
    assert L.nvfp4_ar_choose_algo(8, (2 << 20) // 2 + 256) == 2    # above: two-shot
    assert L.nvfp4_ar_choose_algo(8, (4 << 20) // 2) == 2
    assert L.nvfp4_ar_choose_algo(2, 1024) == 3
    assert L.nvfp4_ar_choose_algo(2, 1 << 30) == 1                  # two ranks: one-shot at any size


def test_create_rejects_bad_arguments(nv):
    L = nv.lib()
    h = ctypes.c_void_p()
    for world, rank, n in [(0, 0, 64), (9, 0, 64), (2, 2, 64), (2, -1, 64), (2, 0, -5)]:
        assert L.nvfp4_ar_create(world, rank, n, ctypes.byref(h)) == nv.NVFP4_ERR_INVALID_ARG
        assert h.value is None
    assert L.nvfp4_ar_destroy(None) == 0
    # calls on a null context are rejected before any CUDA work
    assert L.nvfp4_ar_allreduce(None, None, None, 64, ctypes.c_float(1.0), 0, None) == nv.NVFP4_ERR_INVALID_ARG
    assert L.nvfp4_ar_set_timeout(None, 10 ** 9) == nv.NVFP4_ERR_INVALID_ARG
    fake = ctypes.c_void_p(1 << 20)
    f1 = ctypes.c_float(1.0)
    assert L.nvfp4_gemm_allreduce(None, fake, fake, fake, fake, f1, f1, fake, 256, 256, 256,
                                  None) == nv.NVFP4_ERR_INVALID_ARG
    assert L.nvfp4_gemm_allreduce(None, fake, fake, fake, fake, f1, f1, fake, 128, 256, 256,
                                  None) == nv.NVFP4_ERR_INVALID_ARG
    assert L.nvfp4_gemm_allreduce_emulated(None, 2, None, None, None, None, None, f1, None, 256, 256, 256,
                                           None) == nv.NVFP4_ERR_INVALID_ARG
    assert L.nvfp4_ar_set_multicast(None, fake, fake, 1 << 20) == nv.NVFP4_ERR_INVALID_ARG
    assert L.nvfp4_ar_bf16_allreduce(None, fake, fake, 64, 4, None) == nv.NVFP4_ERR_INVALID_ARG


# ------------------------------------------------------------ gloo ranks ----
def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _gloo_worker(rank, world, port, results):
    import torch
    import torch.distributed as dist

    from tensorcore_ptx_example_b200 import allreduce as ar
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        blob = bytes([rank]) * 64                     # stands in for a CUDA IPC handle
        got = ar.exchange(blob, world)
        gs = ar.agree_global_scale(10.0 * (rank + 1))  # max amax = 10 * world
        results[rank] = (got, gs)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_handle_exchange_and_scale_agreement_on_gloo_ranks():
    import torch.multiprocessing as mp
    world = 2
    port = _free_port()
    with mp.get_context("spawn").Manager() as m:
        results = m.dict()
        mp.spawn(_gloo_worker, args=(world, port, results), nprocs=world, join=True)
        res = dict(results)
    want_gs = float(np.float32(np.float32(10.0 * world) / np.float32(2688.0)))
    for r in range(world):
        got, gs = res[r]
        assert got == [bytes([q]) * 64 for q in range(world)]
        assert gs == want_gs


def test_oracle_nonfinite_blocks(oracle):
    """Oracle side of the non-finite contract: a block with NaN or Inf gets scale 0x7F and zero
    codes; amax skips non-finite values."""
    x = np.zeros((1, 64), np.uint16)
    x[0, :] = 0x3F80                       # 1.0
    x[0, 3] = 0x7FC0                       # NaN in block 0
    x[0, 40] = 0xFF80                      # -Inf in block 2
    assert oracle.amax_bf16(x) == 1.0
    packed, sf = oracle.quantize_bf16(x, 1.0 / 2688)
    offs = oracle.sf_offsets(1, 64)[0]
    assert sf[offs[0]] == 0x7F and sf[offs[2]] == 0x7F
    assert sf[offs[1]] != 0x7F and sf[offs[3]] != 0x7F
    assert np.all(packed[0, 0:8] == 0) and np.all(packed[0, 16:24] == 0)
    assert np.any(packed[0, 8:16] != 0)
