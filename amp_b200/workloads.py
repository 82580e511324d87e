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


# Paged-KV GQA workload: batch 8, 32 query heads, 8 kv heads, head_dim 128,
# context lengths ~ U[512, 16384], 16-token pages scattered by a seeded
# random-permutation block table; prefill queries are the last 512 tokens.
PAGED_B, PAGED_HQ, PAGED_HKV, PAGED_D, PAGE = 8, 32, 8, 128, 16
PAGED_CTX_LO, PAGED_CTX_HI, PAGED_LQ = 512, 16384, 512


def paged_layout(ctx_lens, seed: int = 0, extra_pages: int = 0):
    """Block table for the given context lengths: pages of the pool handed out in
    a seeded random permutation (the pool holds exactly the pages needed, plus
    `extra_pages`).  Returns (block_table int32 [B, max_pages], num_pages)."""
    ctx = np.asarray(ctx_lens, np.int64)
    need = (ctx + PAGE - 1) // PAGE
    num_pages = int(need.sum()) + extra_pages
    perm = np.random.default_rng(seed).permutation(num_pages).astype(np.int32)
    max_pages = int(max(1, need.max()))
    bt = np.zeros((len(ctx), max_pages), np.int32)
    pos = 0
    for b, n in enumerate(need):
        bt[b, :n] = perm[pos:pos + n]
        pos += n
    return bt, num_pages


def paged_inputs(seed: int = 0, B: int = PAGED_B, Hq: int = PAGED_HQ, Hkv: int = PAGED_HKV,
                 D: int = PAGED_D, ctx_lo: int = PAGED_CTX_LO, ctx_hi: int = PAGED_CTX_HI,
                 ctx_lens=None):
    """Host-side (numpy) paged workload: context lengths, block table and pools
    of bf16 N(0,1) values (float32 arrays holding bf16-representable values)."""
    rng = np.random.default_rng(seed)
    if ctx_lens is None:
        ctx_lens = rng.integers(ctx_lo, ctx_hi + 1, size=B)
    ctx_lens = np.asarray(ctx_lens, np.int32)
    bt, num_pages = paged_layout(ctx_lens, seed + 1)
    def bf16(a):
        return (f32_to_bf16_bits(a).astype(np.uint32) << 16).view(np.float32)
    k_pool = bf16(rng.standard_normal((num_pages, Hkv, PAGE, D), dtype=np.float32))
    v_pool = bf16(rng.standard_normal((num_pages, Hkv, PAGE, D), dtype=np.float32))
    return ctx_lens, bt, num_pages, k_pool, v_pool
