"""FlashAttention-2 forward on the B200 vs the fp64 oracle (oracle/attention.py).

Bars: O within AMP's bf16 bar (max|x-ref|/max(1,|ref|) < 2e-2); lse within
2e-3 absolute (it is fp32 in the reference and here).
"""
import numpy as np
import pytest
import torch

from amp_b200 import attention
from amp_b200._lib import AmpError, lib
from oracle import attention as ref
import oracle

pytestmark = pytest.mark.gpu
TOL_O = 2e-2
TOL_LSE = 2e-3


def make_qkv(B, Hq, Hkv, Sq, Skv, D, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, Sq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, Skv, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, Skv, D, generator=g).to(torch.bfloat16)
    return q, k, v


def run(q, k, v, causal, scale=0.0):
    o, lse = attention.flash_attn_fwd(q.cuda(), k.cuda(), v.cuda(), causal, scale)
    torch.cuda.synchronize()
    assert lib().amp_device_status(1) == 0
    return o.float().cpu().numpy(), lse.cpu().numpy()


def check(q, k, v, causal, scale=0.0, heads=None):
    o, lse = run(q, k, v, causal, scale)
    O, L = ref.flash_attn_fwd(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal,
                              scale, heads=heads)
    sel = ~np.isnan(L)
    assert oracle.max_rel_err(o[sel], O[sel]) < TOL_O
    assert np.abs(lse[sel] - L[sel]).max() < TOL_LSE


@pytest.mark.parametrize("S", [128, 256, 300, 1, 17, 640])
@pytest.mark.parametrize("causal", [True, False])
def test_small_shapes(S, causal, cuda, amp_lib):
    check(*make_qkv(1, 2, 2, S, S, 128, seed=S), causal)


@pytest.mark.parametrize("Hq,Hkv", [(8, 2), (4, 1), (32, 8)])
def test_gqa_head_mapping(Hq, Hkv, cuda, amp_lib):
    check(*make_qkv(2, Hq, Hkv, 384, 384, 128, seed=Hq), True)


def test_head_dim_64(cuda, amp_lib):
    check(*make_qkv(2, 4, 2, 513, 513, 64, seed=64), True)
    check(*make_qkv(1, 2, 2, 200, 200, 64, seed=65), False)


def test_cross_attention_lengths(cuda, amp_lib):
    check(*make_qkv(1, 2, 1, 200, 1000, 128, seed=7), False)


def test_explicit_scale_and_large_logits(cuda, amp_lib):
    q, k, v = make_qkv(1, 2, 2, 256, 256, 128, seed=8)
    check(q * 4, k * 4, v, True, scale=0.3)  # row maxima jump between tiles: O rescales


def test_config_b4_h32_s4096_causal(cuda, amp_lib):
    """Full-size FA2 configuration; every output row is produced, sampled heads
    are checked against the fp64 oracle at full sequence length."""
    q, k, v = make_qkv(4, 32, 32, 4096, 4096, 128, seed=2024)
    o, lse = run(q, k, v, True)
    assert np.isfinite(o).all() and np.isfinite(lse).all()
    heads = [(0, 0), (1, 17), (3, 31)]
    O, L = ref.flash_attn_fwd(q.float().numpy(), k.float().numpy(), v.float().numpy(), True,
                              heads=heads)
    for b, h in heads:
        assert oracle.max_rel_err(o[b, h], O[b, h]) < TOL_O
        assert np.abs(lse[b, h] - L[b, h]).max() < TOL_LSE


def test_rejects_bad_gqa(cuda, amp_lib):
    q, k, v = make_qkv(1, 3, 2, 128, 128, 128, seed=1)
    with pytest.raises(AmpError, match="multiple"):
        run(q, k, v, True)


def test_rejects_head_dim_96(cuda, amp_lib):
    q, k, v = make_qkv(1, 2, 2, 128, 128, 96, seed=1)
    with pytest.raises(AmpError, match="head_dim"):
        run(q, k, v, True)


@pytest.mark.parametrize("S,D", [(512, 128), (200, 128), (300, 64)])
def test_allgather_attention_single_rank(S, D, cuda):
    """The fused all-gather attention on a group of one: the epilogue's staged rows
    land in the rank's own O / lse exactly as the plain kernel writes them."""
    from amp_b200 import sharded
    from amp_b200._lib import lib
    from amp_b200.collective import CommGroup, PeerBuffer
    B, H = 2, 3
    g = torch.Generator(device="cuda").manual_seed(S + D)
    q, k, v = (torch.randn(B, H, S, D, generator=g, device="cuda").to(torch.bfloat16)
               for _ in range(3))
    o_ref, l_ref = attention.flash_attn_fwd(q, k, v, True)
    po = PeerBuffer(CommGroup(), B * H * S, D, torch.bfloat16)
    pl = PeerBuffer(CommGroup(), B * H, S, torch.float32, mailboxes=po.mailboxes)
    try:
        for _ in range(2):
            o, l = sharded.flash_attn_allgather(q, k, v, True, po, pl)
            torch.cuda.synchronize()
            assert torch.equal(o, o_ref) and torch.equal(l, l_ref)
        assert lib().amp_device_status(1) == 0
    finally:
        pl.close()
        po.close()


@pytest.mark.parametrize("causal", [True, False])
def test_persistent_schedule_bit_identical(causal, cuda):
    """The dense forward runs one CTA per SM over units of two query-tile pairs of one head.
    B=6 H=32 S=640 has three pairs a head, so each head's second unit holds one item and an
    empty slot, and its 6*32*2 = 384 units make a CTA walk up to three of them.  An item's
    arithmetic does not depend on the CTA that runs it, so O and lse must equal, bit for bit,
    those of per-sequence launches (64 units, one a CTA)."""
    B, Hq, Hkv, S, D = 6, 32, 8, 640, 128
    q, k, v = make_qkv(B, Hq, Hkv, S, S, D, seed=41)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    o, lse = attention.flash_attn_fwd(qd, kd, vd, causal)
    for b in range(B):
        ob, lb = attention.flash_attn_fwd(qd[b:b + 1].contiguous(), kd[b:b + 1].contiguous(),
                                          vd[b:b + 1].contiguous(), causal)
        assert torch.equal(o[b:b + 1], ob)
        assert torch.equal(lse[b:b + 1], lb)
    torch.cuda.synchronize()
    assert lib().amp_device_status(1) == 0
