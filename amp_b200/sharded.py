"""Sharded hot-path operations over the GPUs of one node.

  quantize_e4m3_sharded  each rank quantises its shard with the GLOBAL amax
                         (local amax kernel -> 1-float all-reduce MAX -> encode)
  matmul_bf16_sharded    N-split GEMM: rank r computes C[:, r*N/p:(r+1)*N/p]
                         from all of A and its B column slab, then C is
                         all-gathered and laid out row-major (optional)
  matmul_allgather       the same with the all-gather fused into the GEMM
                         epilogue: every rank's block is stored straight into
                         every rank's C over NVLink (bf16 or FP8 operands)
  flash_attn_sharded     (batch*head)-split attention; O / lse gathered (optional)
  flash_attn_allgather   the same with the all-gather of O / lse fused into the
                         attention epilogue (stores into every rank's O over NVLink)
"""
from __future__ import annotations

import torch

from . import attention, fp8, gemm
from ._lib import call
from .collective import (CommGroup, PeerBuffer, gather_columns, gather_heads, global_amax,
                         head_range)


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


def matmul_allgather(A: torch.Tensor, B_slab: torch.Tensor, out: PeerBuffer,
                     scale_a=None, scale_b=None) -> torch.Tensor:
    """C = A @ B on the node with the all-gather fused into the GEMM: A [M, K] on
    every rank, B_slab [K, N/p] this rank's column block, `out` a [M, N] PeerBuffer
    (bf16 or fp32).  bf16 operands, or E4M3 codes (uint8 / float8_e4m3fn) with
    per-row scale_a [M] and per-column scale_b [N/p] (or 1-element tensors).
    Returns out.tensor, complete on every rank once the stream reaches it."""
    g = out.g
    M, K = A.shape
    Np = B_slab.shape[1]
    if tuple(out.shape) != (M, Np * g.world):
        raise ValueError(f"out is {tuple(out.shape)}, expected {(M, Np * g.world)}")
    if out.dtype not in gemm.AMP_DTYPE:
        raise ValueError("out must be bfloat16 or float32")
    for t, shape, nm in ((A, (M, K), "A"), (B_slab, (K, Np), "B_slab")):
        if not t.is_cuda or not t.is_contiguous() or tuple(t.shape) != shape:
            raise ValueError(f"{nm}: expected a contiguous CUDA tensor of shape {shape}")
    stream = torch.cuda.current_stream(A.device).cuda_stream
    with out.mailboxes.sequence() as seq:
        if A.dtype == torch.bfloat16:
            if B_slab.dtype != torch.bfloat16:
                raise ValueError("A and B_slab must have the same type")
            call("amp_gemm_bf16_allgather_dev", A.data_ptr(), B_slab.data_ptr(),
                 out.table.data_ptr(), gemm.AMP_DTYPE[out.dtype], g.rank, g.world,
                 out.mailboxes.table.data_ptr(), seq, M, Np, K, stream)
        elif A.dtype in (torch.uint8, torch.float8_e4m3fn):
            if B_slab.dtype not in (torch.uint8, torch.float8_e4m3fn):
                raise ValueError("A and B_slab must both hold E4M3 codes")
            rowcol = scale_a.numel() == M and M != 1 or scale_b.numel() == Np and Np != 1
            n_a, n_b, mode = (M, Np, 2) if rowcol else (1, 1, 1)
            sa = gemm._scale_tensor(scale_a, n_a, A.device, "scale_a")
            sb = gemm._scale_tensor(scale_b, n_b, A.device, "scale_b")
            call("amp_gemm_fp8e4m3_allgather_dev", A.data_ptr(), B_slab.data_ptr(),
                 sa.data_ptr(), sb.data_ptr(), mode, out.table.data_ptr(),
                 gemm.AMP_DTYPE[out.dtype], g.rank, g.world, out.mailboxes.table.data_ptr(), seq,
                 M, Np, K, stream)
        else:
            raise ValueError(f"unsupported operand type {A.dtype}")
    return out.tensor


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


def flash_attn_allgather(q, k, v, causal: bool, o_out: PeerBuffer, lse_out: PeerBuffer | None = None,
                         scale: float = 0.0):
    """(batch*head)-split attention with the all-gather fused into the epilogue.
    q/k/v [B, H, S, D] on every rank (Hq == Hkv); o_out a [B*H*S, D] bf16 PeerBuffer,
    lse_out an optional [B*H, S] fp32 PeerBuffer sharing o_out's mailboxes.  Returns
    (O [B, H, S, D], lse [B, H, S] or None), complete on every rank once the stream
    reaches them."""
    g = o_out.g
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    if Hq != Hkv:
        raise ValueError("the batch*head split keeps kv heads with their query group: "
                         "use Hq == Hkv or shard along batch")
    if tuple(o_out.shape) != (B * Hq * S, D) or o_out.dtype != torch.bfloat16:
        raise ValueError(f"o_out must be a ({B * Hq * S}, {D}) bfloat16 PeerBuffer")
    if lse_out is not None:
        if tuple(lse_out.shape) != (B * Hq, S) or lse_out.dtype != torch.float32:
            raise ValueError(f"lse_out must be a ({B * Hq}, {S}) float32 PeerBuffer")
        if lse_out.mailboxes is not o_out.mailboxes:
            raise ValueError("lse_out must share o_out's mailboxes")
    lo, hi = head_range(B * Hq, g)
    qs = q.reshape(B * Hq, S, D)[lo:hi].contiguous()
    ks = k.reshape(B * Hkv, S, D)[lo:hi].contiguous()
    vs = v.reshape(B * Hkv, S, D)[lo:hi].contiguous()
    stream = torch.cuda.current_stream(q.device).cuda_stream
    with o_out.mailboxes.sequence() as seq:
        call("amp_flash_attn_fwd_allgather_dev", qs.data_ptr(), ks.data_ptr(), vs.data_ptr(),
             o_out.table.data_ptr(), lse_out.table.data_ptr() if lse_out is not None else None,
             g.rank, g.world, lo, o_out.mailboxes.table.data_ptr(), seq,
             1, hi - lo, hi - lo, S, S, D, int(causal), float(scale), stream)
    o = o_out.tensor.view(B, Hq, S, D)
    return o, (lse_out.tensor.view(B, Hq, S) if lse_out is not None else None)
