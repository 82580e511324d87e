"""Paged-KV GQA decode and prefill on the B200 vs the fp64 oracle.

The oracle gathers each sequence's pages through the block table into a
contiguous K/V (oracle.attention.paged_gather) and runs the fp64 attention
restatement: decode = the query at position ctx-1 sees every key; prefill =
the last Lq positions, causal with bottom-right alignment.
"""
import numpy as np
import pytest
import torch

import oracle
from oracle import attention as ref
from amp_b200 import paged, workloads
from amp_b200._lib import lib

pytestmark = pytest.mark.gpu
TOL_O = 2e-2
TOL_LSE = 2e-3


def bf16_np(a):
    return (oracle.f32_to_bf16_bits(a).astype(np.uint32) << 16).view(np.float32)


def to_dev(ctx, bt, kp, vp):
    return (torch.from_numpy(kp).to(torch.bfloat16).cuda(),
            torch.from_numpy(vp).to(torch.bfloat16).cuda(),
            torch.from_numpy(bt).cuda(), torch.from_numpy(ctx).cuda())


def decode_ref(q, ctx, bt, kp, vp, heads=None):
    B, Hq, D = q.shape
    O = np.full((B, Hq, D), np.nan)
    L = np.full((B, Hq), np.nan)
    for b in range(B):
        if ctx[b] == 0:                 # no keys: O = 0, lse = -inf
            O[b], L[b] = 0.0, -np.inf
            continue
        k = ref.paged_gather(kp, bt[b], int(ctx[b]))[None]     # [1, Hkv, ctx, D]
        v = ref.paged_gather(vp, bt[b], int(ctx[b]))[None]
        o, lse = ref.flash_attn_fwd(q[b][None, :, None, :], k, v, causal=False)
        O[b], L[b] = o[0, :, 0], lse[0, :, 0]
    return O, L


def run_decode(q, ctx, bt, kp, vp):
    k_pool, v_pool, btd, ctxd = to_dev(ctx, bt, kp, vp)
    out, lse = paged.paged_attn_decode(torch.from_numpy(q).to(torch.bfloat16).cuda(), k_pool,
                                       v_pool, btd, ctxd, int(ctx.max()))
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), lse.cpu().numpy()


@pytest.mark.parametrize("Hq,Hkv", [(8, 2), (4, 4), (16, 8), (32, 4)])
def test_decode_small(Hq, Hkv, cuda, amp_lib):
    ctx = np.array([1, 17, 1000, 513, 16], np.int32)
    ctx, bt, npg, kp, vp = workloads.paged_inputs(seed=Hq, B=5, Hq=Hq, Hkv=Hkv, ctx_lens=ctx)
    q = bf16_np(np.random.default_rng(Hq).standard_normal((5, Hq, 128), dtype=np.float32))
    out, lse = run_decode(q, ctx, bt, kp, vp)
    assert lib().amp_device_status(1) == 0
    O, L = decode_ref(q, ctx, bt, kp, vp)
    assert oracle.max_rel_err(out, O) < TOL_O
    assert np.abs(lse - L).max() < TOL_LSE


def test_decode_full_workload(cuda, amp_lib):
    ctx, bt, npg, kp, vp = workloads.paged_inputs(seed=11)
    q = bf16_np(np.random.default_rng(12).standard_normal((8, 32, 128), dtype=np.float32))
    out, lse = run_decode(q, ctx, bt, kp, vp)
    assert lib().amp_device_status(1) == 0
    O, L = decode_ref(q, ctx, bt, kp, vp)
    assert oracle.max_rel_err(out, O) < TOL_O
    assert np.abs(lse - L).max() < TOL_LSE


def test_decode_many_short_sequences(cuda, amp_lib):
    # slices of the page list cross many sequence boundaries; some contexts are empty
    rng = np.random.default_rng(21)
    ctx = rng.integers(0, 70, size=96).astype(np.int32)
    ctx[[3, 40, 41]] = 0
    ctx, bt, npg, kp, vp = workloads.paged_inputs(seed=22, B=96, Hq=8, Hkv=2, ctx_lens=ctx)
    q = bf16_np(rng.standard_normal((96, 8, 128), dtype=np.float32))
    out, lse = run_decode(q, ctx, bt, kp, vp)
    assert lib().amp_device_status(1) == 0
    O, L = decode_ref(q, ctx, bt, kp, vp)
    assert oracle.max_rel_err(out, O) < TOL_O
    fin = np.isfinite(L)
    assert (np.isinf(lse) == ~fin).all() and np.abs(lse[fin] - L[fin]).max() < TOL_LSE


def test_decode_large_batch_uses_prefix_kernel(cuda, amp_lib):
    # above 1024 sequences the page prefix sums come from a separate kernel
    rng = np.random.default_rng(23)
    ctx = rng.integers(1, 40, size=1100).astype(np.int32)
    ctx, bt, npg, kp, vp = workloads.paged_inputs(seed=24, B=1100, Hq=4, Hkv=1, ctx_lens=ctx)
    q = bf16_np(rng.standard_normal((1100, 4, 128), dtype=np.float32))
    out, lse = run_decode(q, ctx, bt, kp, vp)
    assert lib().amp_device_status(1) == 0
    O, L = decode_ref(q, ctx, bt, kp, vp)
    assert oracle.max_rel_err(out, O) < TOL_O
    assert np.abs(lse - L).max() < TOL_LSE


def test_decode_context_past_max_context_len_is_flagged(cuda, amp_lib):
    ctx = np.array([100, 50], np.int32)
    ctx, bt, npg, kp, vp = workloads.paged_inputs(seed=25, B=2, Hq=8, Hkv=2, ctx_lens=ctx)
    q = bf16_np(np.random.default_rng(26).standard_normal((2, 8, 128), dtype=np.float32))
    k_pool, v_pool, btd, ctxd = to_dev(ctx, bt, kp, vp)
    out, _ = paged.paged_attn_decode(torch.from_numpy(q).to(torch.bfloat16).cuda(), k_pool,
                                     v_pool, btd, ctxd, 64)
    torch.cuda.synchronize()
    assert lib().amp_device_status(1) == -1   # sequence 0 is longer than the declared 64
    assert lib().amp_device_status(1) == 0
    O, _ = decode_ref(q[1:], ctx[1:], bt[1:], kp, vp)
    assert oracle.max_rel_err(out.float().cpu().numpy()[1:], O) < TOL_O


def test_decode_garbage_past_context_is_ignored(cuda, amp_lib):
    ctx = np.array([20, 33], np.int32)
    ctx, bt, npg, kp, vp = workloads.paged_inputs(seed=3, B=2, Hq=8, Hkv=2, ctx_lens=ctx)
    kp2, vp2 = kp.copy(), vp.copy()
    for b in range(2):   # NaN/inf in the unused slots of each last page
        last = bt[b, (ctx[b] - 1) // 16]
        kp2[last, :, ctx[b] % 16:] = np.nan
        vp2[last, :, ctx[b] % 16:] = np.inf
    q = bf16_np(np.random.default_rng(4).standard_normal((2, 8, 128), dtype=np.float32))
    out, lse = run_decode(q, ctx, bt, kp2, vp2)
    O, L = decode_ref(q, ctx, bt, kp, vp)
    assert np.isfinite(out).all() and oracle.max_rel_err(out, O) < TOL_O


def test_decode_bad_page_id_is_flagged_not_dereferenced(cuda, amp_lib):
    ctx = np.array([40, 40], np.int32)
    ctx, bt, npg, kp, vp = workloads.paged_inputs(seed=5, B=2, Hq=8, Hkv=2, ctx_lens=ctx)
    bt = bt.copy()
    bt[1, 1] = npg + 1000          # far outside the pool
    q = bf16_np(np.random.default_rng(6).standard_normal((2, 8, 128), dtype=np.float32))
    out, lse = run_decode(q, ctx, bt, kp, vp)
    assert lib().amp_device_status(1) == -1   # AMP_ERR_INVALID, then cleared
    assert lib().amp_device_status(1) == 0
    O, L = decode_ref(q[:1], ctx[:1], bt[:1], kp, vp)
    assert oracle.max_rel_err(out[:1], O) < TOL_O   # the other sequence is unaffected


def prefill_ref(q, ctx, bt, kp, vp, heads):
    B, Hq, Lq, D = q.shape
    O = np.full(q.shape, np.nan)
    L = np.full((B, Hq, Lq), np.nan)
    for b in sorted({b for b, _ in heads}):
        k = ref.paged_gather(kp, bt[b], int(ctx[b]))[None]
        v = ref.paged_gather(vp, bt[b], int(ctx[b]))[None]
        hs = [(0, h) for bb, h in heads if bb == b]
        o, lse = ref.flash_attn_fwd(q[b][None], k, v, causal=True,
                                    causal_offset=int(ctx[b]) - Lq, heads=hs)
        for _, h in hs:
            O[b, h], L[b, h] = o[0, h], lse[0, h]
    return O, L


def run_prefill(q, ctx, bt, kp, vp):
    k_pool, v_pool, btd, ctxd = to_dev(ctx, bt, kp, vp)
    out, lse = paged.paged_attn_prefill(torch.from_numpy(q).to(torch.bfloat16).cuda(), k_pool,
                                        v_pool, btd, ctxd)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), lse.cpu().numpy()


@pytest.mark.parametrize("Lq,ctx", [(128, [128, 300, 700]), (100, [100, 257, 1000]),
                                    (1, [1, 16, 17]), (256, [4096, 260, 1024])])
def test_prefill_small(Lq, ctx, cuda, amp_lib):
    ctx = np.array(ctx, np.int32)
    ctx, bt, npg, kp, vp = workloads.paged_inputs(seed=Lq, B=3, Hq=8, Hkv=2, ctx_lens=ctx)
    q = bf16_np(np.random.default_rng(Lq).standard_normal((3, 8, Lq, 128), dtype=np.float32))
    out, lse = run_prefill(q, ctx, bt, kp, vp)
    assert lib().amp_device_status(1) == 0
    heads = [(b, h) for b in range(3) for h in range(8)]
    O, L = prefill_ref(q, ctx, bt, kp, vp, heads)
    assert oracle.max_rel_err(out, O) < TOL_O
    assert np.abs(lse - L).max() < TOL_LSE


def test_prefill_full_workload_sampled_heads(cuda, amp_lib):
    ctx, bt, npg, kp, vp = workloads.paged_inputs(seed=21)
    q = bf16_np(np.random.default_rng(22).standard_normal((8, 32, 512, 128), dtype=np.float32))
    out, lse = run_prefill(q, ctx, bt, kp, vp)
    assert lib().amp_device_status(1) == 0
    assert np.isfinite(out).all()
    heads = [(0, 0), (3, 13), (7, 31), (int(np.argmax(ctx)), 5)]
    O, L = prefill_ref(q, ctx, bt, kp, vp, heads)
    for b, h in heads:
        assert oracle.max_rel_err(out[b, h], O[b, h]) < TOL_O
        assert np.abs(lse[b, h] - L[b, h]).max() < TOL_LSE


def test_paged_kernels_on_amp_scheduler_batches(cuda, amp_lib):
    """Batches from AMP's own Scheduler::schedule() (page ids from its PagePoolFast)
    drive the decode and prefill kernels over one contiguous pool per K and V."""
    r = oracle.ref_sched_lib()
    if r is None:
        pytest.skip("AMP's scheduler driver is not built (make -C oracle ref)")
    Hq, Hkv, D, NP = 8, 2, 128, 512
    rng = np.random.default_rng(7)
    kp = bf16_np(rng.standard_normal((NP, Hkv, 16, D), dtype=np.float32))
    vp = bf16_np(rng.standard_normal((NP, Hkv, 16, D), dtype=np.float32))
    s = oracle.RefScheduler(r, max_pages=NP, max_batch_tokens=1024, max_prefill=128)
    for _ in range(6):
        s.add(int(rng.integers(20, 300)), int(rng.integers(2, 12)))
    n_pre = n_dec = 0
    try:
        for _ in range(60):
            ent, lists = s.step()
            if len(ent) == 0:
                break
            ctx = ent[:, 4].astype(np.int32)
            bt = paged.pack_block_table(lists, ctx)
            dec = ent[:, 1] == 0
            if dec.any():
                idx = np.nonzero(dec)[0]
                q = bf16_np(rng.standard_normal((len(idx), Hq, D), dtype=np.float32))
                out, lse = run_decode(q, ctx[idx], bt[idx], kp, vp)
                assert lib().amp_device_status(1) == 0
                O, L = decode_ref(q, ctx[idx], bt[idx], kp, vp)
                assert oracle.max_rel_err(out, O) < TOL_O
                assert np.abs(lse - L).max() < TOL_LSE
                n_dec += len(idx)
            for i in np.nonzero(~dec)[0]:   # chunk lengths differ: one sequence per call
                Lq = int(ent[i, 2])
                q = bf16_np(rng.standard_normal((1, Hq, Lq, D), dtype=np.float32))
                out, lse = run_prefill(q, ctx[i:i + 1], bt[i:i + 1], kp, vp)
                assert lib().amp_device_status(1) == 0
                O, L = prefill_ref(q, ctx[i:i + 1], bt[i:i + 1], kp, vp,
                                   [(0, h) for h in range(Hq)])
                assert oracle.max_rel_err(out, O) < TOL_O
                n_pre += 1
    finally:
        s.close()
    assert n_pre > 0 and n_dec > 0


def test_query_and_output_buffers_are_checked_before_launch(cuda, amp_lib):
    ctx = np.array([40, 17], np.int32)
    ctx, bt, npg, kp, vp = workloads.paged_inputs(seed=3, B=2, Hq=8, Hkv=2, ctx_lens=ctx)
    k_pool, v_pool, btd, ctxd = to_dev(ctx, bt, kp, vp)
    q = torch.zeros(2, 8, 128, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError, match="q: expected"):
        paged.paged_attn_decode(q.float(), k_pool, v_pool, btd, ctxd, 64)
    with pytest.raises(ValueError, match="q: expected"):
        paged.paged_attn_decode(q[..., :64].contiguous(), k_pool, v_pool, btd, ctxd, 64)
    with pytest.raises(ValueError, match="block_table"):
        paged.paged_attn_decode(torch.zeros(3, 8, 128, dtype=torch.bfloat16, device=cuda),
                                k_pool, v_pool, btd, ctxd, 64)
    with pytest.raises(ValueError, match="lse must"):
        paged.paged_attn_decode(q, k_pool, v_pool, btd, ctxd, 64,
                                lse=torch.empty(2, 8, 1, device=cuda))
    with pytest.raises(ValueError, match="out must"):
        paged.paged_attn_decode(q, k_pool, v_pool, btd, ctxd, 64, out=torch.empty_like(q).float())
    with pytest.raises(ValueError, match="workspace"):
        paged.paged_attn_decode(q, k_pool, v_pool, btd, ctxd, 64,
                                workspace=torch.empty(8, dtype=torch.uint8, device=cuda))
    with pytest.raises(ValueError, match="q: expected"):
        paged.paged_attn_prefill(q, k_pool, v_pool, btd, ctxd)   # prefill q is [B, Hq, Lq, D]
    torch.cuda.synchronize()
