"""Seeded synthetic workloads with the shapes and value distributions of the benchmark
configurations (no dataset is involved; everything is generated from a seed).

  cfg1  tile        M128 N256 K256, E2M1 codes uniform over all 16, scales 2^u, u in [-4, 4]
  cfg2  quantize    8192 x 7168 bf16, N(0, 1), 0.1 % of positions (seeded) multiplied by 50
  cfg3  GEMM        M = N = K = 8192, A ~ N(0, 1), B ~ N(0, 0.02), both quantized as cfg2;
                    decode variant M16 N7168 K8192
  cfg4  all-reduce  per rank 4096 x 7168 bf16 N(0, 1), seed = rank
  cfg5  sweep       16 KB .. 256 MB of bf16 per rank, doubling
"""
from __future__ import annotations

CFG2_SHAPE = (8192, 7168)
CFG3_SHAPE = (8192, 8192, 8192)
CFG3_DECODE_SHAPE = (16, 7168, 8192)
CFG4_SHAPE = (4096, 7168)


def activations(rows: int, cols: int, seed: int, std: float = 1.0, outlier_frac: float = 0.001,
                outlier_mul: float = 50.0, device="cuda"):
    """bf16 [rows, cols]: N(0, std^2) with round(outlier_frac * n) seeded positions scaled by
    outlier_mul (positions drawn with replacement; a repeated position is scaled once)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    x = torch.randn(rows, cols, generator=g, device=device, dtype=torch.float32)
    if std != 1.0:
        x.mul_(std)
    n = rows * cols
    k = int(round(n * outlier_frac))
    if k:
        idx = torch.randint(0, n, (k,), generator=g, device=device)
        flat = x.view(-1)
        flat[idx] = flat[idx] * outlier_mul
    return x.to(torch.bfloat16)


def gaussian(rows: int, cols: int, seed: int, std: float = 1.0, device="cuda"):
    return activations(rows, cols, seed, std=std, outlier_frac=0.0, device=device)


def sweep_sizes_bytes():
    """cfg5: 16 KB .. 256 MB of bf16 payload, doubling."""
    s, out = 16 * 1024, []
    while s <= 256 * 1024 * 1024:
        out.append(s)
        s *= 2
    return out
