"""Host-side pieces of bench.py (CPU only): the rotating inputs that keep back-to-back timed
all-reduce calls reading from HBM, and the per-algorithm wire-byte accounting."""
import torch

import bench


def test_rotating_inputs_exceed_l2_and_repeat_the_input():
    x = torch.arange(4096, dtype=torch.float32).to(torch.bfloat16)
    xs = bench.rotating_inputs(x, min_bytes=1 << 20)
    assert len(xs) * x.numel() * x.element_size() >= 1 << 20
    assert len(xs) >= 2
    starts = {t.data_ptr() for t in xs}
    assert len(starts) == len(xs)                      # distinct places of one buffer
    for t in xs:
        assert t.shape == x.shape and torch.equal(t, x)
    # the default covers more than the 126 MB L2 with a 58.7 MB cfg4 input
    n = 4096 * 7168
    sets = max(2, -(-bench.ROT_BYTES // (2 * n)))
    assert sets * n * 2 > 126 * 10 ** 6


def test_wire_bytes_per_algorithm():
    numel, world = 1 << 20, 8
    # one-shot: the whole payload to each of the n-1 peers; two-shot and NVLS: 2 (n-1)/n of it
    assert bench._wire_bytes("nvfp4_oneshot", numel, world, 0.5625) == 7 * 0.5625 * numel
    assert bench._wire_bytes("nvfp4_twoshot", numel, world, 0.5625) == 2 * 7 / 8 * 0.5625 * numel
    assert bench._wire_bytes("bf16_nvls", numel, world, 2.0) == 2 * 7 / 8 * 2.0 * numel
