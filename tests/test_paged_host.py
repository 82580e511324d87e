"""Host-side paged-KV logic (no GPU): block-table layout and validation."""
import numpy as np
import pytest

from amp_b200 import paged, workloads
from amp_b200._lib import AmpError


def test_layout_is_a_permutation_covering_every_needed_page():
    ctx = np.array([512, 16384, 1, 17, 9000])
    bt, npg = workloads.paged_layout(ctx, seed=3)
    need = (ctx + 15) // 16
    used = np.concatenate([bt[b, :n] for b, n in enumerate(need)])
    assert npg == need.sum() and sorted(used.tolist()) == list(range(npg))


def test_validation_accepts_generated_tables(amp_lib):
    ctx = np.array([512, 16384, 1, 17])
    bt, npg = workloads.paged_layout(ctx, seed=1)
    paged.validate_block_table(bt, ctx, npg)


@pytest.mark.parametrize("fault", ["range", "negative", "duplicate", "short"])
def test_validation_rejects_malformed_tables(fault, amp_lib):
    ctx = np.array([40, 40], np.int32)
    bt, npg = workloads.paged_layout(ctx, seed=2)
    bt = bt.copy()
    if fault == "range":
        bt[0, 1] = npg
    elif fault == "negative":
        bt[1, 0] = -3
    elif fault == "duplicate":
        bt[1, 2] = bt[0, 0]
    else:
        ctx = np.array([40, 80], np.int32)   # needs 5 pages, rows hold 3
    with pytest.raises(AmpError):
        paged.validate_block_table(bt, ctx, npg)
