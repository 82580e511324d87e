"""The fp64 attention oracle against torch in fp64 (an independent
implementation): O against scaled_dot_product_attention and lse against
logsumexp of the masked scores, with GQA, an explicit scale and the
bottom-right causal alignment of the paged path; and the block-table gather
against a token-by-token lookup."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import attention as ref


@pytest.mark.parametrize("B,Hq,Hkv,Sq,Skv,D,causal,offset,scale", [
    (2, 4, 2, 37, 37, 16, True, 0, 0.0),      # causal self-attention, GQA group 2
    (1, 4, 1, 20, 50, 32, True, 30, 0.3),     # paged prefill: last 20 of 50 tokens
    (1, 2, 2, 33, 33, 8, False, 0, 0.0),      # full attention
    (1, 8, 2, 1, 77, 16, True, 76, 0.0),      # decode: one query at the end
])
def test_forward_matches_torch(B, Hq, Hkv, Sq, Skv, D, causal, offset, scale):
    rng = np.random.default_rng(Sq * 7 + Skv)
    q = rng.standard_normal((B, Hq, Sq, D))
    k = rng.standard_normal((B, Hkv, Skv, D))
    v = rng.standard_normal((B, Hkv, Skv, D))
    O, lse = ref.flash_attn_fwd(q, k, v, causal, scale, causal_offset=offset)
    tq, tk, tv = (torch.from_numpy(x) for x in (q, k, v))
    tk, tv = (t.repeat_interleave(Hq // Hkv, dim=1) for t in (tk, tv))
    sc = scale if scale > 0 else 1.0 / np.sqrt(D)
    keep = torch.ones(Sq, Skv, dtype=torch.bool)
    if causal:
        keep = torch.arange(Skv)[None, :] <= torch.arange(Sq)[:, None] + offset
    want_o = F.scaled_dot_product_attention(tq, tk, tv, attn_mask=keep, scale=sc)
    s = (tq @ tk.transpose(-1, -2)) * sc
    want_lse = torch.logsumexp(s.masked_fill(~keep, float("-inf")), dim=-1)
    assert np.abs(O - want_o.numpy()).max() < 1e-12
    assert np.abs(lse - want_lse.numpy()).max() < 1e-12


def test_paged_gather_follows_the_block_table():
    rng = np.random.default_rng(3)
    num_pages, Hkv, P, D = 40, 2, 16, 8
    pool = rng.standard_normal((num_pages, Hkv, P, D))
    for ctx in (1, 16, 17, 100, 16 * 12):
        n = (ctx + P - 1) // P
        table = rng.permutation(num_pages)[:n]
        got = ref.paged_gather(pool, table, ctx)
        want = np.stack([pool[table[t // P], :, t % P] for t in range(ctx)], axis=1)
        assert got.shape == (Hkv, ctx, D)
        assert np.array_equal(got, want)
