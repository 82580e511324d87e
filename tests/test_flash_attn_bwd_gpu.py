"""FlashAttention-2 backward on the B200 vs the fp64 chain rule (oracle.attention.flash_attn_bwd).

Bar: max|x-ref|/max(1,|ref|) < 2e-2 for dQ, dK, dV (AMP's metric and bf16 bar; P
and dS are rounded to bf16 before the tensor-core products, as in the forward).
The forward's own O and lse feed the backward, as in training.
"""
import pytest
import torch

import oracle
from oracle import attention as ref
from amp_b200 import attention
from amp_b200._lib import AmpError, lib

pytestmark = pytest.mark.gpu
TOL = 2e-2


def run(B, Hq, Hkv, S, D, causal, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, S, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
    do = torch.randn(B, Hq, S, D, generator=g).to(torch.bfloat16)
    qd, kd, vd, dod = q.cuda(), k.cuda(), v.cuda(), do.cuda()
    o, lse = attention.flash_attn_fwd(qd, kd, vd, causal)
    dq, dk, dv = attention.flash_attn_bwd(qd, kd, vd, o, dod, lse, causal)
    torch.cuda.synchronize()
    assert lib().amp_device_status(1) == 0
    rq, rk, rv = ref.flash_attn_bwd(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                    do.float().numpy(), causal)
    return ((dq.float().cpu().numpy(), rq), (dk.float().cpu().numpy(), rk),
            (dv.float().cpu().numpy(), rv))


@pytest.mark.parametrize("S", [128, 256, 384, 100, 1, 300])
@pytest.mark.parametrize("causal", [True, False])
def test_bwd_shapes(S, causal, cuda, amp_lib):
    for name, (got, want) in zip("qkv", run(1, 2, 2, S, 128, causal, seed=S)):
        err = oracle.max_rel_err(got, want)
        assert err < TOL, (name, err)


@pytest.mark.parametrize("Hq,Hkv", [(4, 1), (8, 2), (4, 4)])
def test_bwd_gqa(Hq, Hkv, cuda, amp_lib):
    for name, (got, want) in zip("qkv", run(2, Hq, Hkv, 256, 128, True, seed=Hq * 7 + Hkv)):
        err = oracle.max_rel_err(got, want)
        assert err < TOL, (name, err)


def test_bwd_head_dim_64(cuda, amp_lib):
    for name, (got, want) in zip("qkv", run(1, 4, 2, 256, 64, True, seed=64)):
        err = oracle.max_rel_err(got, want)
        assert err < TOL, (name, err)


def test_bwd_longer_sequence(cuda, amp_lib):
    for name, (got, want) in zip("qkv", run(1, 2, 1, 1024, 128, True, seed=5)):
        err = oracle.max_rel_err(got, want)
        assert err < TOL, (name, err)


def test_bwd_rejects_causal_cross_lengths(cuda, amp_lib):
    q = torch.zeros(1, 1, 128, 128, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(1, 1, 256, 128, dtype=torch.bfloat16, device="cuda")
    lse = torch.zeros(1, 1, 128, device="cuda")
    with pytest.raises(AmpError, match="S_q == S_kv"):
        attention.flash_attn_bwd(q, k, k, q, q, lse, True)


@pytest.mark.parametrize("causal", [True, False])
def test_persistent_passes_bit_identical(causal, cuda):
    """Both backward passes run one CTA per SM over units of two tiles of one head.  B=6 S=384
    has three tiles a head, so each head's second unit holds one tile and an empty slot; with
    32 query and 16 kv heads the dQ pass has 6*32*2 = 384 units and the dK/dV pass 6*16*2 = 192,
    so CTAs walk several.  dQ, dK and dV must equal, bit for bit, those of per-sequence
    launches on the same O and lse (64 and 32 units, at most one a CTA)."""
    B, Hq, Hkv, S, D = 6, 32, 16, 384, 128
    g = torch.Generator().manual_seed(43)
    q, do = (torch.randn(B, Hq, S, D, generator=g).to(torch.bfloat16).cuda() for _ in range(2))
    k, v = (torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16).cuda() for _ in range(2))
    o, lse = attention.flash_attn_fwd(q, k, v, causal)
    dq, dk, dv = attention.flash_attn_bwd(q, k, v, o, do, lse, causal)
    for b in range(B):
        s = slice(b, b + 1)
        dqb, dkb, dvb = attention.flash_attn_bwd(
            q[s].contiguous(), k[s].contiguous(), v[s].contiguous(), o[s].contiguous(),
            do[s].contiguous(), lse[s].contiguous(), causal)
        assert torch.equal(dq[s], dqb)
        assert torch.equal(dk[s], dkb)
        assert torch.equal(dv[s], dvb)
    torch.cuda.synchronize()
    assert lib().amp_device_status(1) == 0
