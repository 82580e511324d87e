"""fp64 attention oracle -- TEST INFRASTRUCTURE ONLY (the checker).

Restates the semantics of the reference's FlashAttention-2 forward
(kernels/flash_attn.cu:73-197; AttnCfg kernels/flash_attn.cuh:26-36):
  * Q [B,Hq,S_q,D], K/V [B,Hkv,S_kv,D]; kv head = hq / (Hq/Hkv)  (flash_attn.cu:90)
  * s = scale * q.k, scale = cfg.scale if > 0 else 1/sqrt(D)  (flash_attn.cu:208)
  * causal: key j masked for query i when j > i  (flash_attn.cu:134,152); the
    paged path uses bottom-right alignment, i.e. masked when j > i + offset
    with offset = S_kv - S_q, which the `causal_offset` argument expresses
  * O = softmax(s) V; lse = m + ln(l) = ln sum_j exp(s_ij)  (flash_attn.cu:195)
The reference has no CPU attention path of its own; this is the oracle the
GPU kernels are checked against, computed exactly in fp64 (forward, and the
backward that consumes its lse).
"""
from __future__ import annotations

import numpy as np


def flash_attn_fwd(q, k, v, causal: bool = True, scale: float = 0.0, causal_offset: int = 0,
                   heads=None):
    """Returns (O, lse) in float64.  `heads` optionally restricts to a list of
    (b, hq) pairs (others are left as NaN) so that full-size cases stay cheap."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    group = Hq // Hkv
    sc = scale if scale > 0 else 1.0 / np.sqrt(D)
    O = np.full((B, Hq, Sq, D), np.nan)
    lse = np.full((B, Hq, Sq), np.nan)
    if causal:
        i = np.arange(Sq)[:, None]
        j = np.arange(Skv)[None, :]
        masked = j > i + causal_offset
    for b in range(B):
        for h in range(Hq):
            if heads is not None and (b, h) not in heads:
                continue
            hk = h // group
            s = (q[b, h] @ k[b, hk].T) * sc
            if causal:
                s = np.where(masked, -np.inf, s)
            m = s.max(axis=1, keepdims=True)
            m_safe = np.where(np.isfinite(m), m, 0.0)
            p = np.exp(s - m_safe)
            l = p.sum(axis=1, keepdims=True)
            with np.errstate(invalid="ignore", divide="ignore"):
                O[b, h] = np.where(l > 0, (p @ v[b, hk]) / l, 0.0)
                lse[b, h] = np.where(l[:, 0] > 0, m_safe[:, 0] + np.log(l[:, 0]), -np.inf)
    return O, lse


def flash_attn_bwd(q, k, v, do, causal: bool = True, scale: float = 0.0, causal_offset: int = 0):
    """Gradients of O = softmax(scale * Q K^T) V, in float64: returns (dQ, dK, dV).

    The reference has no backward (its lse output is documented as "required for
    the backward pass", kernels/flash_attn.cuh:48); this is the standard chain
    rule the GPU backward is checked against: P = softmax(S); dV = P^T dO;
    dP = dO V^T; dS = P * (dP - rowsum(dO * O)); dQ = scale dS K; dK = scale dS^T Q.
    GQA: a kv head's dK / dV sum over the query heads that share it."""
    q, k, v, do = (np.asarray(x, np.float64) for x in (q, k, v, do))
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    group = Hq // Hkv
    sc = scale if scale > 0 else 1.0 / np.sqrt(D)
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    if causal:
        masked = np.arange(Skv)[None, :] > np.arange(Sq)[:, None] + causal_offset
    for b in range(B):
        for h in range(Hq):
            hk = h // group
            s = (q[b, h] @ k[b, hk].T) * sc
            if causal:
                s = np.where(masked, -np.inf, s)
            m = s.max(axis=1, keepdims=True)
            m = np.where(np.isfinite(m), m, 0.0)
            e = np.exp(s - m)
            l = e.sum(axis=1, keepdims=True)
            p = np.where(l > 0, e / np.where(l > 0, l, 1.0), 0.0)
            o = p @ v[b, hk]
            dv[b, hk] += p.T @ do[b, h]
            dp = do[b, h] @ v[b, hk].T
            delta = (do[b, h] * o).sum(axis=1, keepdims=True)
            ds = p * (dp - delta)
            dq[b, h] = sc * (ds @ k[b, hk])
            dk[b, hk] += sc * (ds.T @ q[b, h])
    return dq, dk, dv


def paged_gather(pool, block_table, ctx_len, page_size: int = 16):
    """Contiguous [Hkv, ctx, D] view of one sequence's paged K or V: token t of
    the sequence lives in page block_table[t // page_size], slot t % page_size
    (Sequence::kv_page_ids, include/scheduler.hpp:61; 16-token pages,
    include/scheduler.hpp:88).  pool: [num_pages, Hkv, page_size, D]."""
    pool = np.asarray(pool)
    n_pages = (ctx_len + page_size - 1) // page_size
    pages = pool[np.asarray(block_table[:n_pages])]          # [n, Hkv, P, D]
    full = np.concatenate(list(pages), axis=1) if n_pages else pool[:0].sum(0)
    return full[:, :ctx_len]
