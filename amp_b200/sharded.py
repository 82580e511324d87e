"""Sharded hot-path operations over the GPUs of one node.

  quantize_e4m3_sharded  each rank quantises its shard with the GLOBAL amax
                         (local amax kernel -> 1-float all-reduce MAX -> encode)
  matmul_bf16_sharded    N-split GEMM: rank r computes C[:, r*N/p:(r+1)*N/p]
                         from all of A and its B column slab, then C is
                         all-gathered and laid out row-major (optional)
  flash_attn_sharded     (batch*head)-split attention; O / lse gathered (optional)
"""
from __future__ import annotations

import torch

from . import attention, fp8, gemm
from .collective import CommGroup, gather_columns, gather_heads, global_amax, head_range


def quantize_e4m3_sharded(x_shard: torch.Tensor, g: CommGroup | None = None, mailboxes=None):
    """Per-tensor FP8 quantisation of a tensor sharded over ranks: the global amax
    comes from the peer mailboxes when given (NVLink stores), else from a 1-float
    NCCL/gloo all-reduce."""
    g = g or CommGroup.current()
    if mailboxes is not None:
        amax = fp8.amax_allreduce_peer(x_shard, mailboxes)
    else:
        amax = fp8.amax_bf16(x_shard)
        global_amax(g, amax)
    return fp8.quantize_e4m3_from_amax(x_shard, amax)


def matmul_bf16_sharded(A: torch.Tensor, B_slab: torch.Tensor, g: CommGroup | None = None,
                        gather: bool = True, out_dtype=torch.bfloat16):
    """A [M, K] (replicated), B_slab [K, N/p] (this rank's columns)."""
    g = g or CommGroup.current()
    M, K = A.shape
    Np = B_slab.shape[1]
    C = torch.empty(M, Np, dtype=out_dtype, device=A.device)
    gemm.launch_matmul_bf16(A, B_slab, C, M, Np, K)
    return gather_columns(g, C) if gather else C


def flash_attn_sharded(q, k, v, causal: bool = True, g: CommGroup | None = None,
                       gather: bool = True):
    """q/k/v [B, H, S, D] on every rank; this rank computes its batch*head slice."""
    g = g or CommGroup.current()
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    if Hq != Hkv:
        raise ValueError("the batch*head split keeps kv heads with their query group: "
                         "use Hq == Hkv or shard along batch")
    lo, hi = head_range(B * Hq, g)
    qs = q.reshape(B * Hq, S, D)[lo:hi].unsqueeze(0).contiguous()
    ks = k.reshape(B * Hkv, S, D)[lo:hi].unsqueeze(0).contiguous()
    vs = v.reshape(B * Hkv, S, D)[lo:hi].unsqueeze(0).contiguous()
    o, lse = attention.flash_attn_fwd(qs, ks, vs, causal)
    if not gather:
        return o, lse
    return (gather_heads(g, o[0]).reshape(B, Hq, S, D),
            gather_heads(g, lse[0]).reshape(B, Hq, S))
