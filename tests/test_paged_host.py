"""Host-side paged-KV logic (no GPU): block-table layout and validation."""
import numpy as np
import pytest

import oracle
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


def test_pack_block_table_pads_and_checks():
    bt = paged.pack_block_table([[5, 6], [7], []], np.array([17, 3, 0], np.int32), 4)
    assert bt.tolist() == [[5, 6, -1, -1], [7, -1, -1, -1], [-1, -1, -1, -1]]
    with pytest.raises(AmpError, match="needs 2 pages"):
        paged.pack_block_table([[5]], np.array([17], np.int32), 4)
    with pytest.raises(AmpError, match="table rows hold"):
        paged.pack_block_table([[1, 2, 3]], np.array([3], np.int32), 2)
    assert paged.pool_bytes(10, 8, 128) == 10 * 8 * 16 * 128 * 2


def test_amp_scheduler_batches_pack_into_valid_tables():
    """AMP's own Scheduler + PagePoolFast (compiled from the reference tree): every
    batch it schedules packs into a block table that passes the validator."""
    r = oracle.ref_sched_lib()
    if r is None:
        pytest.skip("AMP's scheduler driver is not built (make -C oracle ref)")
    s = oracle.RefScheduler(r, max_pages=512, max_batch_tokens=2048, max_prefill=256)
    rng = np.random.default_rng(0)
    for _ in range(12):
        s.add(int(rng.integers(1, 700)), int(rng.integers(1, 40)))
    n_pre = n_dec = 0
    try:
        for _ in range(80):
            ent, lists = s.step()
            if len(ent) == 0:
                break
            ctx = ent[:, 4].astype(np.int32)
            bt = paged.pack_block_table(lists, ctx)
            paged.validate_block_table(bt, ctx, 512)
            n_pre += int(ent[:, 1].sum())
            n_dec += int((ent[:, 1] == 0).sum())
    finally:
        s.close()
    assert n_pre > 0 and n_dec > 0
