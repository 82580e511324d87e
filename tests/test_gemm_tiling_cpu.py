"""Index arithmetic of the tcgen05 GEMMs, checked on the CPU against the
constants in gemm_tc.cu: the grouped tile raster, the SM-pair split of a
256 x 256 tile, TMA coordinates (x * element size a multiple of 16 bytes),
the full barrier's byte count and the TMEM columns the epilogue reads."""
import math
import re
from pathlib import Path

import numpy as np
import pytest

SRC = (Path(__file__).resolve().parents[1] / "amp_b200" / "csrc" / "gemm_tc.cu").read_text()


def const(name):
    m = re.search(rf"constexpr (?:int|uint32_t) {name} = ([^;]+);", SRC)
    assert m, name
    return m.group(1)


BM, BN, SLAB, GROUP_M = (int(const(n)) for n in ("BM", "BN", "SLAB", "kGroupM"))
STAGES2, TMEM_COLS = int(const("STAGES2")), int(const("TMEM_COLS"))
A_STAGE_BYTES = BM * SLAB
STAGE2_BYTES = A_STAGE_BYTES + (BN // 2) * SLAB
assert const("STAGE2_BYTES").replace(" ", "").startswith("A_STAGE_BYTES+(BN/2)*SLAB")


def tile_coords(t, num_m, num_n):
    """tile_coords() of gemm_tc.cu: groups of kGroupM M-tiles, column-major inside."""
    per_group = GROUP_M * num_n
    g = t // per_group
    first_m = g * GROUP_M
    gm = min(GROUP_M, num_m - first_m)
    local = t - g * per_group
    return first_m + local % gm, local // gm


@pytest.mark.parametrize("num_m,num_n", [(1, 1), (3, 5), (16, 16), (17, 3), (40, 33), (64, 32)])
def test_raster_visits_every_tile_once(num_m, num_n):
    seen = np.zeros((num_m, num_n), np.int32)
    for t in range(num_m * num_n):
        tm, tn = tile_coords(t, num_m, num_n)
        seen[tm, tn] += 1
    assert (seen == 1).all()


@pytest.mark.parametrize("es", [1, 2])
@pytest.mark.parametrize("M,N,K,pairs", [(2488, 2000, 1008, 74), (4232, 4048, 512, 74),
                                         (8192, 8192, 8192, 74), (300, 272, 128, 1),
                                         (1000, 1008, 96, 37)])
def test_pair_split_covers_c_once_with_aligned_copies(es, M, N, K, pairs):
    """k_gemm_tc2: pair p takes tiles p, p + n_pairs, ...; CTA rank r of the pair
    loads A rows tm*256 + r*128 .. +128 and B columns tn*256 + r*128 .. +128, and
    its epilogue owns rows tm*256 + r*128 + lane-row of all 256 columns."""
    BK = SLAB // es
    b_box_cols = SLAB // es
    b_boxes = (BN // 2) // b_box_cols
    num_m, num_n = math.ceil(M / (2 * BM)), math.ceil(N / BN)
    num_kb = math.ceil(K * es / SLAB)
    total = num_m * num_n
    n_pairs = min(total, pairs)
    owner = np.zeros((num_m * 2 * BM, num_n * BN), np.int32)
    for pair in range(n_pairs):
        for t in range(pair, total, n_pairs):
            tm, tn = tile_coords(t, num_m, num_n)
            a_rows, b_cols = [], []
            for rank in (0, 1):
                r0 = tm * 2 * BM + rank * BM
                a_rows.append((r0, r0 + BM))
                for kb in range(num_kb):
                    assert (kb * BK * es) % 16 == 0          # A's x coordinate
                    for j in range(b_boxes):
                        x = tn * BN + rank * (BN // 2) + j * b_box_cols
                        assert (x * es) % 16 == 0            # B's x coordinate
                        b_cols.append((x, x + b_box_cols))
                owner[r0:r0 + BM, tn * BN:(tn + 1) * BN] += 1
            # the two CTAs' A rows are the tile's 256 rows; their B boxes its 256 columns
            assert a_rows == [(tm * 2 * BM, tm * 2 * BM + BM), (tm * 2 * BM + BM, (tm + 1) * 2 * BM)]
            cols = sorted(set(b_cols))
            assert cols[0][0] == tn * BN and cols[-1][1] == (tn + 1) * BN
            assert all(a[1] == b[0] for a, b in zip(cols, cols[1:]))
    assert (owner[:M, :N] == 1).all()


@pytest.mark.parametrize("es", [1, 2])
def test_full_barrier_counts_both_ctas_bytes(es):
    BK = SLAB // es
    b_boxes = (BN // 2) // (SLAB // es)
    per_cta = BM * SLAB + b_boxes * BK * SLAB       # one A box + this CTA's B boxes
    assert per_cta == STAGE2_BYTES
    assert "mbar_arrive_expect_tx(&full[s], 2 * STAGE2_BYTES)" in SRC


def test_accumulators_fit_tmem_and_smem_fits_a_cta():
    # two 256-column fp32 accumulators; the epilogue reads acc * BN + c * 32 for c < BN / 32
    assert 2 * BN <= TMEM_COLS <= 512 and max(a * BN + c * 32 + 32 for a in (0, 1)
                                              for c in range(BN // 32)) <= TMEM_COLS
    assert STAGES2 * STAGE2_BYTES + 1024 + 256 <= 227 * 1024
