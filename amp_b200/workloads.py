"""Seeded synthetic inputs with the shapes and value distributions of the
hot-path workloads (no dataset is involved anywhere in AMP).

Each generator exists in a numpy form (host, reproducible across machines,
used by the parity tests) and, where sizes are large, a torch device form
(used by the benchmark, which needs no host copy of the data).
"""
from __future__ import annotations

import numpy as np

# FP8 quantise workload: 2^26 bf16 values ~ N(0,1) with 0.1% outliers ~ N(0,50).
QUANT_N = 1 << 26
QUANT_OUTLIER_FRAC = 0.001
QUANT_OUTLIER_STD = 50.0


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def quant_input_numpy(n: int = QUANT_N, seed: int = 0) -> np.ndarray:
    """bf16 bit patterns: N(0,1), with round(0.1% * n) seeded positions ~ N(0,50)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(n, dtype=np.float32)
    k = int(round(QUANT_OUTLIER_FRAC * n))
    if k:
        pos = rng.choice(n, size=k, replace=False)
        x[pos] = rng.standard_normal(k, dtype=np.float32) * np.float32(QUANT_OUTLIER_STD)
    return f32_to_bf16_bits(x)


def quant_input_torch(n: int = QUANT_N, seed: int = 0, device="cuda"):
    """Same distribution drawn on the device (values differ from the numpy form)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.randn(n, generator=g, device=device, dtype=torch.float32)
    k = int(round(QUANT_OUTLIER_FRAC * n))
    if k:
        pos = torch.randperm(n, generator=g, device=device)[:k]
        x[pos] = torch.randn(k, generator=g, device=device) * QUANT_OUTLIER_STD
    return x.to(torch.bfloat16)


# fp32 GEMM workload (AMP's amp_verify_matmul shape class): A, B ~ U[-1, 1], seed 0.
def gemm_fp32_inputs(M: int, N: int, K: int, seed: int = 0):
    rng = np.random.default_rng(seed)
    A = rng.uniform(-1.0, 1.0, (M, K)).astype(np.float32)
    B = rng.uniform(-1.0, 1.0, (K, N)).astype(np.float32)
    return A, B
