"""Row-parallel NVFP4 GEMM fused with the two-shot all-reduce (nvfp4_gemm_allreduce), on ONE GPU:
every rank's buffers on the same device, every rank's GEMM then each all-reduce phase launched for
every rank in turn (nvfp4_gemm_allreduce_emulated), so no kernel waits for another.

The fused path must give the bytes of the unfused one -- nvfp4_gemm_bf16 per rank, then the
two-shot all-reduce of the bf16 partial products -- and of the oracle (oracle/nvfp4_oracle.c:
the tcgen05 GEMM model, the bf16 epilogue, orc_ar_twoshot).  The cross-GPU path is covered by
tests/test_allreduce_multigpu.py.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tensorcore_ptx_example_b200 import allreduce as ar  # noqa: E402
from tensorcore_ptx_example_b200 import workloads  # noqa: E402

pytestmark = pytest.mark.gpu

MODEL = 4   # ORC_ACC_TCGEN05


def u16(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)


def rank_operands(nv, world, M, N, K, seed):
    ops, alphas = [], []
    for r in range(world):
        a = workloads.activations(M, K, seed=seed + 2 * r)
        b = workloads.gaussian(N, K, seed=seed + 2 * r + 1, std=0.02)
        pa, sa, gsa = nv.quantize(a, None)
        pb, sb, gsb = nv.quantize(b, None)
        ops.append((pa, sa, pb, sb))
        alphas.append(float(np.float32(float(gsa.item())) * np.float32(float(gsb.item()))))
    torch.cuda.synchronize()
    return ops, alphas


def partials(nv, ops, alphas, M, N, K):
    return [nv.gemm(pa, sa, pb, sb, M, N, K, alpha=al) for (pa, sa, pb, sb), al in zip(ops, alphas)]


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_gemm_allreduce_matches_unfused_and_oracle(nv, oracle, world):
    M, N, K = 256, 768 if world == 3 else 512, 512
    ops, alphas = rank_operands(nv, world, M, N, K, seed=40 * world)
    ds = partials(nv, ops, alphas, M, N, K)
    torch.cuda.synchronize()
    gs = nv.global_scale_from_amax(max(float(d.float().abs().max()) for d in ds))
    ctxs = [ar.AllReduce(world, r, M * N) for r in range(world)]
    ar.join_in_process(ctxs)
    try:
        fused = ar.emulated_gemm_allreduce(ops, M, N, K, alphas, gs, ctxs)
        unfused = ar.emulated_allreduce([d.view(-1) for d in ds], gs, "twoshot", contexts=ctxs)
        torch.cuda.synchronize()
        assert nv.device_status() == 0
        want = u16(unfused[0])
        for r in range(world):
            assert np.array_equal(u16(fused[r]), want), r
            assert np.array_equal(u16(unfused[r]), want), r
        # oracle: per-rank GEMM model + bf16 epilogue, then the two-shot all-reduce
        d16 = []
        for (pa, sa, pb, sb), al, d in zip(ops, alphas, ds):
            acc = oracle.gemm_f32(pa.cpu().numpy(), sa.cpu().numpy(), pb.cpu().numpy(), sb.cpu().numpy(), M, N, K,
                                  model=MODEL)
            e = oracle.gemm_epilogue_bf16(acc, al).reshape(-1)
            assert np.array_equal(e, u16(d))
            d16.append(e)
        assert np.array_equal(oracle.ar_twoshot(d16, gs), want)
    finally:
        for c in ctxs:
            c.close()


def test_gemm_allreduce_repeated_and_mixed_calls(nv, oracle):
    """Back-to-back fused calls and plain all-reduce calls on the same contexts (parity regions
    and epochs advance together)."""
    world, M, N, K = 4, 256, 256, 256
    ctxs = [ar.AllReduce(world, r, M * N) for r in range(world)]
    ar.join_in_process(ctxs)
    try:
        for i in range(3):
            ops, alphas = rank_operands(nv, world, M, N, K, seed=700 + 10 * i)
            ds = partials(nv, ops, alphas, M, N, K)
            torch.cuda.synchronize()
            gs = nv.global_scale_from_amax(max(float(d.float().abs().max()) for d in ds))
            fused = ar.emulated_gemm_allreduce(ops, M, N, K, alphas, gs, ctxs)
            torch.cuda.synchronize()
            want = oracle.ar_twoshot([u16(d) for d in ds], gs)
            for r in range(world):
                assert np.array_equal(u16(fused[r]), want), (i, r)
            plain = ar.emulated_allreduce([d.view(-1) for d in ds], gs, "oneshot", contexts=ctxs)
            torch.cuda.synchronize()
            assert np.array_equal(u16(plain[0]), oracle.ar_oneshot([u16(d) for d in ds], gs))
        assert nv.device_status() == 0
    finally:
        for c in ctxs:
            c.close()


def test_gemm_allreduce_cfg_size(nv, oracle):
    """8 ranks, M 4096 x N 7168 output, K 1024 per rank (a row-parallel split of K 8192): the fused
    path against the unfused one, byte for byte."""
    world, M, N, K = 8, 4096, 7168, 1024
    ops, alphas = rank_operands(nv, world, M, N, K, seed=91)
    ds = partials(nv, ops, alphas, M, N, K)
    torch.cuda.synchronize()
    gs = nv.global_scale_from_amax(max(float(d.float().abs().max()) for d in ds))
    ctxs = [ar.AllReduce(world, r, M * N) for r in range(world)]
    ar.join_in_process(ctxs)
    try:
        fused = ar.emulated_gemm_allreduce(ops, M, N, K, alphas, gs, ctxs)
        unfused = ar.emulated_allreduce([d.view(-1) for d in ds], gs, "twoshot", contexts=ctxs)
        torch.cuda.synchronize()
        assert nv.device_status() == 0
        for r in (0, 3, 7):
            assert torch.equal(fused[r], unfused[r].view(M, N)), r
    finally:
        for c in ctxs:
            c.close()
