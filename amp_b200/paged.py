"""Attention over a paged KV cache (16-token pages addressed by block tables).

Mirrors the block-table format of the reference's scheduler
(``Sequence::kv_page_ids``, include/scheduler.hpp:61; 16-token pages,
include/scheduler.hpp:88) with device tensors:

  k_pool, v_pool  [num_pages, Hkv, 16, D] bf16
  block_table     int32 [B, max_pages_per_seq]
  ctx_lens        int32 [B]
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._lib import call, lib

PAGE_TOKENS = 16


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _check_pools(k_pool, v_pool, block_table, ctx_lens):
    for t, nm in ((k_pool, "k_pool"), (v_pool, "v_pool")):
        if not t.is_cuda or t.dtype != torch.bfloat16 or not t.is_contiguous() or t.dim() != 4 \
                or t.shape[2] != PAGE_TOKENS:
            raise ValueError(f"{nm}: expected contiguous bf16 CUDA [pages, Hkv, 16, D]")
    if k_pool.shape != v_pool.shape:
        raise ValueError("k_pool and v_pool shapes differ")
    for t, nm in ((block_table, "block_table"), (ctx_lens, "ctx_lens")):
        if not t.is_cuda or t.dtype != torch.int32 or not t.is_contiguous():
            raise ValueError(f"{nm}: expected a contiguous int32 CUDA tensor")


def _check_q(q, out, lse, k_pool, block_table, ctx_lens, rank: int):
    """q (and a caller-supplied out) [B, Hq, (Lq,) D] bf16 with D the pools' head
    dimension and B rows of block table and context lengths; lse [B, Hq, (Lq)] fp32."""
    if not q.is_cuda or q.dtype != torch.bfloat16 or not q.is_contiguous() or q.dim() != rank \
            or q.device != k_pool.device or q.shape[-1] != k_pool.shape[3]:
        raise ValueError(f"q: expected a contiguous bf16 CUDA tensor of rank {rank} on "
                         f"{k_pool.device} with head dimension {k_pool.shape[3]}")
    B = q.shape[0]
    if block_table.dim() != 2 or block_table.shape[0] < B or ctx_lens.numel() < B:
        raise ValueError(f"block_table [>= {B}, pages] and ctx_lens [>= {B}] expected")
    if out is not None and (out.dtype != q.dtype or out.shape != q.shape or out.device != q.device
                            or not out.is_contiguous()):
        raise ValueError("out must be a contiguous tensor shaped like q")
    if lse is not None and (lse.dtype != torch.float32 or tuple(lse.shape) != tuple(q.shape[:-1])
                            or lse.device != q.device or not lse.is_contiguous()):
        raise ValueError(f"lse must be a contiguous float32 tensor of shape {tuple(q.shape[:-1])}")


def decode_workspace_bytes(B: int, Hq: int, D: int, max_context_len: int) -> int:
    return int(lib().amp_paged_decode_workspace_bytes(B, Hq, D, max_context_len))


def paged_attn_decode(q, k_pool, v_pool, block_table, ctx_lens, max_context_len: int,
                      scale: float = 0.0, out=None, lse=None, workspace=None):
    """One query token per sequence: q [B, Hq, D] -> (out [B, Hq, D], lse [B, Hq])."""
    _check_pools(k_pool, v_pool, block_table, ctx_lens)
    _check_q(q, out, lse, k_pool, block_table, ctx_lens, 3)
    B, Hq, D = q.shape
    num_pages, Hkv = k_pool.shape[0], k_pool.shape[1]
    ws_b = decode_workspace_bytes(B, Hq, D, max_context_len)
    if workspace is not None and (not workspace.is_cuda or workspace.device != q.device
                                  or workspace.dtype != torch.uint8
                                  or not workspace.is_contiguous() or workspace.numel() < ws_b):
        raise ValueError(f"workspace: expected a contiguous uint8 tensor of >= {ws_b} bytes "
                         f"on {q.device}")
    out = out if out is not None else torch.empty_like(q)
    lse = lse if lse is not None else torch.empty(B, Hq, dtype=torch.float32, device=q.device)
    ws = workspace if workspace is not None else torch.empty(ws_b, dtype=torch.uint8,
                                                             device=q.device)
    call("amp_paged_attn_decode_bf16_dev", q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(),
         block_table.data_ptr(), ctx_lens.data_ptr(), out.data_ptr(), lse.data_ptr(), B, Hq, Hkv,
         D, num_pages, block_table.shape[1], max_context_len, float(scale), ws.data_ptr(),
         ws.numel(), _stream(q))
    return out, lse


def paged_attn_prefill(q, k_pool, v_pool, block_table, ctx_lens, scale: float = 0.0,
                       out=None, lse=None):
    """q [B, Hq, Lq, D]: the last Lq tokens of each context, bottom-right causal."""
    _check_pools(k_pool, v_pool, block_table, ctx_lens)
    _check_q(q, out, lse, k_pool, block_table, ctx_lens, 4)
    B, Hq, Lq, D = q.shape
    num_pages, Hkv = k_pool.shape[0], k_pool.shape[1]
    out = out if out is not None else torch.empty_like(q)
    lse = lse if lse is not None else torch.empty(B, Hq, Lq, dtype=torch.float32,
                                                  device=q.device)
    call("amp_paged_attn_prefill_bf16_dev", q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(),
         block_table.data_ptr(), ctx_lens.data_ptr(), out.data_ptr(), lse.data_ptr(), B, Hq, Hkv,
         Lq, D, num_pages, block_table.shape[1], float(scale), _stream(q))
    return out, lse


def validate_block_table(block_table: np.ndarray, ctx_lens: np.ndarray, num_pages: int) -> None:
    """Host-side check before upload (raises AmpError on the first fault)."""
    bt = np.ascontiguousarray(block_table, np.int32)
    cl = np.ascontiguousarray(ctx_lens, np.int32)
    call("amp_paged_validate_block_table", bt.ctypes.data, cl.ctypes.data, bt.shape[0],
         bt.shape[1], num_pages)


def pack_block_table(page_lists, ctx_lens, max_pages_per_seq: int | None = None) -> np.ndarray:
    """Padded int32 block table [B, max_pages] from per-sequence page-id lists (the
    shape of AMP's Sequence::kv_page_ids), -1 past each list.  Raises AmpError if a
    list cannot hold its sequence's context."""
    lists = [np.asarray(p, np.int32).ravel() for p in page_lists]
    B = len(lists)
    starts = np.zeros(B + 1, np.int32)
    starts[1:] = np.cumsum([len(p) for p in lists])
    flat = np.concatenate(lists) if B and starts[-1] else np.zeros(1, np.int32)
    width = max_pages_per_seq or max(1, max(len(p) for p in lists))
    cl = np.ascontiguousarray(ctx_lens, np.int32)
    bt = np.empty((B, width), np.int32)
    call("amp_paged_pack_block_table", flat.ctypes.data, starts.ctypes.data, cl.ctypes.data, B,
         width, bt.ctypes.data)
    return bt


def pool_bytes(num_pages: int, Hkv: int, D: int) -> int:
    """Bytes of one contiguous K or V pool [num_pages][Hkv][16][D] bf16."""
    return int(lib().amp_paged_pool_bytes(num_pages, Hkv, D))
