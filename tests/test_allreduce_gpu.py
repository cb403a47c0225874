"""NVFP4 all-reduce data path on ONE GPU: every rank's buffers on the same device, each phase
launched for every rank in turn (nvfp4_ar_allreduce_emulated), so no kernel waits for another.
Bit-exact against the oracle (oracle/nvfp4_oracle.c orc_ar_*), which sums in rank order 0..n-1
and requantizes two-shot shards with global scale gs * n, following the data flow of the
reference's fused kernels (blackwell/allreduce_sm100_sm120/nvfp4_allreduce.cuh:498-619).
The cross-GPU barriers are covered by tests/test_allreduce_multigpu.py.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tensorcore_ptx_example_b200 import allreduce as ar  # noqa: E402
from tensorcore_ptx_example_b200 import workloads  # noqa: E402

pytestmark = pytest.mark.gpu


def u16(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)


def rank_inputs(world, numel, seed0=0, std=1.0):
    return [workloads.gaussian(1, numel, seed=seed0 + r, std=std).view(-1) for r in range(world)]


def global_scale(nv, inputs):
    a = max(float(nv.amax(x).item()) for x in inputs)
    return nv.global_scale_from_amax(a)


@pytest.mark.parametrize("world", [2, 3, 4, 6, 8])
@pytest.mark.parametrize("algo", ["oneshot", "twoshot", "lowlat"])
def test_nvfp4_allreduce_bitexact(nv, oracle, world, algo):
    numel = 32 * world * 37                       # several blocks, not a power of two
    ins = rank_inputs(world, numel, seed0=100 * world)
    gs = global_scale(nv, ins)
    outs = ar.emulated_allreduce(ins, gs, algo)
    torch.cuda.synchronize()
    assert nv.device_status() == 0
    want = (oracle.ar_twoshot if algo == "twoshot" else oracle.ar_oneshot)([u16(x) for x in ins], gs)
    for r in range(world):                        # every rank holds the same result
        got = u16(outs[r])
        assert np.array_equal(got, want), f"rank {r}: {np.count_nonzero(got != want)} mismatches"


@pytest.mark.parametrize("world", [2, 8])
@pytest.mark.parametrize("algo", ["oneshot", "twoshot"])
def test_bf16_allreduce_bitexact(nv, oracle, world, algo):
    numel = 8 * world * 301
    ins = rank_inputs(world, numel, seed0=7)
    outs = ar.emulated_allreduce(ins, algo=algo, bf16=True)
    torch.cuda.synchronize()
    want = oracle.ar_bf16([u16(x) for x in ins])
    for r in range(world):
        assert np.array_equal(u16(outs[r]), want)


def test_repeated_calls_alternate_buffers(nv, oracle):
    """Back-to-back calls on the same contexts (parity alternation, growing epochs), with
    different inputs, algorithms and payload kinds."""
    world, numel = 4, 32 * 4 * 64
    ctxs = [ar.AllReduce(world, r, numel) for r in range(world)]
    ar.join_in_process(ctxs)
    try:
        for i, (algo, bf16) in enumerate([("oneshot", False), ("twoshot", False), ("twoshot", True),
                                          ("lowlat", False), ("lowlat", False), ("lowlat", False),
                                          ("oneshot", True), ("twoshot", False), ("oneshot", False),
                                          ("lowlat", False)]):
            ins = rank_inputs(world, numel, seed0=1000 + 10 * i, std=1.0 + i)
            gs = global_scale(nv, ins)
            outs = ar.emulated_allreduce(ins, gs, algo, bf16=bf16, contexts=ctxs)
            torch.cuda.synchronize()
            x16 = [u16(x) for x in ins]
            if bf16:
                want = oracle.ar_bf16(x16)
            else:
                want = (oracle.ar_twoshot if algo == "twoshot" else oracle.ar_oneshot)(x16, gs)
            for r in range(world):
                assert np.array_equal(u16(outs[r]), want), (i, algo, bf16, r)
    finally:
        for c in ctxs:
            c.close()


def test_lowlat_sizes_change_between_calls(nv, oracle):
    """The low-latency area is laid out per call (word-major over this call's chunks) and zeroed
    by its readers: calls of changing sizes on the same contexts stay exact."""
    world = 4
    ctxs = [ar.AllReduce(world, r, 32 * world * 96) for r in range(world)]
    ar.join_in_process(ctxs)
    try:
        for i, m in enumerate([96, 5, 96, 1, 40, 40, 96]):
            ins = rank_inputs(world, 32 * world * m, seed0=3000 + i, std=0.5 + i)
            gs = global_scale(nv, ins)
            outs = ar.emulated_allreduce(ins, gs, "lowlat", contexts=ctxs)
            torch.cuda.synchronize()
            assert nv.device_status() == 0
            want = oracle.ar_oneshot([u16(x) for x in ins], gs)
            for r in range(world):
                assert np.array_equal(u16(outs[r]), want), (i, m, r)
    finally:
        for c in ctxs:
            c.close()


def test_lowlat_limits(nv):
    """NVFP4 only and at most LOWLAT_CAP_BYTES of bf16; "auto" picks it for small messages."""
    world = 2
    cap = ar.LOWLAT_CAP_BYTES // 2
    numel = 2 * cap
    ctxs = [ar.AllReduce(world, r, numel) for r in range(world)]
    ar.join_in_process(ctxs)
    try:
        big = [torch.zeros(numel, dtype=torch.bfloat16, device="cuda") for _ in range(world)]
        with pytest.raises(nv.NVFP4Error) as e:
            ar.emulated_allreduce(big, 1.0, "lowlat", contexts=ctxs)
        assert e.value.code == nv.NVFP4_ERR_INVALID_ARG
        with pytest.raises(nv.NVFP4Error) as e:
            ctxs[0].bf16_allreduce(big[0][:64], algo="lowlat")
        assert e.value.code == nv.NVFP4_ERR_INVALID_ARG
        ok = [x[:cap] for x in big]
        outs = ar.emulated_allreduce(ok, 1.0, "lowlat", contexts=ctxs)
        torch.cuda.synchronize()
        assert nv.device_status() == 0 and all(int(torch.count_nonzero(o)) == 0 for o in outs)
        assert ar.choose_algo(world, 1024) == ar.LOWLAT
    finally:
        for c in ctxs:
            c.close()


def test_edge_cases(nv):
    world, numel = 2, 32 * 2 * 8
    ctxs = [ar.AllReduce(world, r, numel) for r in range(world)]
    ar.join_in_process(ctxs)
    try:
        x = torch.zeros(numel, dtype=torch.bfloat16, device="cuda")
        # empty: a no-op
        ar.emulated_allreduce([x[:0], x[:0]], 1.0, contexts=ctxs)
        # ragged (not a multiple of 32 * world), too large, bad scale, bad algo: rejected
        for bad in [lambda: ar.emulated_allreduce([x[:48], x[:48]], 1.0, contexts=ctxs),
                    lambda: ar.emulated_allreduce([torch.zeros(2 * numel, dtype=torch.bfloat16, device="cuda")] * 2,
                                                  1.0, contexts=ctxs),
                    lambda: ar.emulated_allreduce([x, x], 0.0, contexts=ctxs),
                    lambda: ar.emulated_allreduce([x, x], float("inf"), contexts=ctxs)]:
            with pytest.raises(nv.NVFP4Error) as e:
                bad()
            assert e.value.code == nv.NVFP4_ERR_INVALID_ARG
        with pytest.raises(ValueError):
            ar.emulated_allreduce([x, x], 1.0, algo="ring", contexts=ctxs)
        # a context whose peers were never set refuses to run
        lone = ar.AllReduce(2, 0, numel)
        with pytest.raises(nv.NVFP4Error) as e:
            lone.allreduce(x, global_scale=1.0)
        assert e.value.code == nv.NVFP4_ERR_NOT_READY
        lone.close()
        # all-zero input: scales 0, codes 0, output exactly zero
        out = ar.emulated_allreduce([x, x], 1.0, "twoshot", contexts=ctxs)
        torch.cuda.synchronize()
        assert all(int(torch.count_nonzero(o)) == 0 for o in out)
    finally:
        for c in ctxs:
            c.close()


def test_cfg4_full_size_sampled(nv, oracle):
    """cfg4 at full size: 8 ranks x 4096 x 7168 bf16 N(0, 1), seed = rank.  The GPU result is
    checked bit for bit on sampled windows (the sum is independent per 16-element block), and
    the error against the exact sum is reported."""
    world = 8
    rows, cols = workloads.CFG4_SHAPE
    numel = rows * cols
    ins = [workloads.gaussian(rows, cols, seed=r).view(-1) for r in range(world)]
    gs = global_scale(nv, ins)
    rng = np.random.default_rng(5)
    starts = sorted(set(int(s) * 32 for s in rng.integers(0, numel // 32 - 256, size=12)))
    x16 = [u16(x) for x in ins]
    for algo in ("oneshot", "twoshot"):
        outs = ar.emulated_allreduce(ins, gs, algo)
        torch.cuda.synchronize()
        assert nv.device_status() == 0
        got = u16(outs[3])
        fn = oracle.ar_oneshot if algo == "oneshot" else oracle.ar_twoshot
        for s in starts:
            w = slice(s, s + 32 * 256)
            want = fn([x[w] for x in x16], gs)
            assert np.array_equal(got[w], want), (algo, s)
        assert np.array_equal(u16(outs[0]), got) and np.array_equal(u16(outs[7]), got)
        exact = sum(x.double() for x in ins)
        rel = float(((outs[0].double() - exact).norm() / exact.norm()).item())
        assert rel < (0.12 if algo == "oneshot" else 0.16), (algo, rel)
        del outs


def test_nvls_argument_checks(nv):
    """NVFP4_AR_NVLS: bf16 only, only after a multicast buffer is registered, not emulated on one
    GPU; the registration checks its addresses.  (The in-switch sum itself needs NVLink multicast
    across GPUs: tests/test_allreduce_multigpu.py.)"""
    import ctypes

    from tensorcore_ptx_example_b200 import allreduce as ar
    L = nv.lib()
    numel = 1024
    x = torch.zeros(numel, dtype=torch.bfloat16, device="cuda")
    o = torch.empty_like(x)
    ctx = ar.AllReduce(1, 0, numel)
    try:
        h = ctx.handle
        p = ctypes.c_void_p
        assert L.nvfp4_ar_bf16_allreduce(h, p(x.data_ptr()), p(o.data_ptr()), numel, ar.NVLS, None) == \
            nv.NVFP4_ERR_NOT_READY
        assert L.nvfp4_ar_allreduce(h, p(x.data_ptr()), p(o.data_ptr()), numel, ctypes.c_float(1.0), ar.NVLS,
                                    None) == nv.NVFP4_ERR_UNSUPPORTED
        assert L.nvfp4_ar_set_multicast(h, p(x.data_ptr() + 4), p(x.data_ptr()), 4096) == nv.NVFP4_ERR_INVALID_ARG
        assert L.nvfp4_ar_set_multicast(h, None, p(x.data_ptr()), 4096) == nv.NVFP4_ERR_INVALID_ARG
        hs = (ctypes.c_void_p * 1)(h)
        ins = (ctypes.c_void_p * 1)(p(x.data_ptr()))
        outs = (ctypes.c_void_p * 1)(p(o.data_ptr()))
        assert L.nvfp4_ar_allreduce_emulated(hs, 1, ins, outs, numel, ctypes.c_float(1.0), ar.NVLS, 1, None) == \
            nv.NVFP4_ERR_UNSUPPORTED
    finally:
        ctx.close()
