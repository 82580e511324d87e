"""The algorithmic work behind every roofline figure (bench.py units_per_step)
against brute-force counts on small shapes: visible (query, key) pairs for
causal and bottom-right-aligned attention, bytes a paged decode must move, and
the GEMM / quantiser totals."""
import numpy as np
import pytest
import torch

import bench


def visible_pairs(S_q, S_kv, offset):
    i = np.arange(S_q)[:, None]
    j = np.arange(S_kv)[None, :]
    return int((j <= i + offset).sum())


@pytest.mark.parametrize("bh,S,D", [(1, 1, 128), (3, 17, 128), (2, 256, 64)])
def test_attention_flops_are_4D_per_visible_pair(bh, S, D):
    W = object.__new__(bench.AttentionWorkload)
    W.bh, W.S, W.D = bh, S, D
    assert W.units_per_step() == 4.0 * D * bh * visible_pairs(S, S, 0)
    Wb = object.__new__(bench.AttentionBwdWorkload)
    Wb.bh, Wb.S, Wb.D = bh, S, D
    assert Wb.units_per_step() == 2.5 * W.units_per_step()


def test_prefill_flops_count_bottom_right_visible_pairs():
    ctx = np.array([512, 700, 4096], np.int32)
    W = object.__new__(bench.PagedPrefillWorkload)
    W.ctx, W.Lq, W.Hq, W.D = ctx, 512, 32, 128
    pairs = sum(visible_pairs(512, int(c), int(c) - 512) for c in ctx)
    assert W.units_per_step() == 4.0 * 32 * 128 * pairs


def test_decode_bytes_are_kv_of_every_context_token_plus_io():
    ctx = np.array([17, 512, 1000], np.int32)
    B, Hq, Hkv, D, pages = 3, 32, 8, 128, 63
    W = object.__new__(bench.PagedDecodeWorkload)
    W.ctx, W.Hkv, W.D = ctx, Hkv, D
    W.q = torch.zeros(B, Hq, D, dtype=torch.bfloat16)
    W.lse = torch.zeros(B, Hq)
    W.bt = torch.zeros(B, pages, dtype=torch.int32)
    kv = sum(int(c) * Hkv * D * 2 for c in ctx) * 2        # K and V, bf16
    io = 2 * (B * Hq * D * 2) + B * Hq * 4 + B * pages * 4   # q in, out, lse, table
    assert W.units_per_step() == kv + io


def test_gemm_and_quantiser_totals():
    G = object.__new__(bench.GemmWorkload)
    G.S, G.Np = 1024, 1024
    assert G.units_per_step() == 2.0 * 1024 ** 3
    G.Np = 256                                               # one rank's N slab
    assert G.units_per_step() == 2.0 * 1024 * 1024 * 256
    Q = object.__new__(bench.QuantWorkload)
    Q.n = 1 << 20
    # quantise 5 B (amax read 2, read 2, write 1) + dequantise 3 B (read 1, write 2)
    assert Q.units_per_step() == 8 * (1 << 20)
