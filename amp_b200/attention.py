"""FlashAttention-2 forward: host-side mirror of kernels/flash_attn.cuh.

``launch_flash_attn_bf16(Q, K, V, O, lse, B, S_q, S_kv, cfg)`` mirrors
``AMP::launch_flash_attn_bf16`` (kernels/flash_attn.cuh:50-58) with the same
AttnCfg fields (flash_attn.cuh:26-36).  The tile fields Br/Bc are accepted for
source compatibility; the sm_100a kernel always uses 128x128 tiles.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ._lib import call


@dataclass
class AttnCfg:
    num_q_heads: int = 1
    num_kv_heads: int = 1
    head_dim: int = 128
    causal: bool = True
    scale: float = 0.0      # 0 -> 1/sqrt(head_dim)
    Br: int = 32
    Bc: int = 64


def _check(t, shape, name, dtype=torch.bfloat16):
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous() or tuple(t.shape) != shape:
        raise ValueError(f"{name}: expected contiguous {dtype} CUDA tensor {shape}, "
                         f"got {t.dtype} {tuple(t.shape)}")


def launch_flash_attn_bf16(Q, K, V, O, lse, B: int, S_q: int, S_kv: int, cfg: AttnCfg) -> None:
    Hq, Hkv, D = cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim
    _check(Q, (B, Hq, S_q, D), "Q")
    _check(K, (B, Hkv, S_kv, D), "K")
    _check(V, (B, Hkv, S_kv, D), "V")
    _check(O, (B, Hq, S_q, D), "O")
    if lse is not None:
        _check(lse, (B, Hq, S_q), "lse", torch.float32)
    call("amp_flash_attn_fwd_bf16_dev", Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(),
         lse.data_ptr() if lse is not None else None, B, Hq, Hkv, S_q, S_kv, D,
         1 if cfg.causal else 0, float(cfg.scale), torch.cuda.current_stream(Q.device).cuda_stream)


def flash_attn_fwd(q, k, v, causal: bool = True, scale: float = 0.0):
    """Convenience form: returns (O, lse) for [B,H,S,D] bf16 CUDA tensors."""
    B, Hq, S_q, D = q.shape
    Hkv, S_kv = k.shape[1], k.shape[2]
    O = torch.empty_like(q)
    lse = torch.empty(B, Hq, S_q, dtype=torch.float32, device=q.device)
    launch_flash_attn_bf16(q, k, v, O, lse, B, S_q, S_kv,
                           AttnCfg(Hq, Hkv, D, causal, scale))
    return O, lse


def flash_attn_bwd(q, k, v, o, do, lse, causal: bool = True, scale: float = 0.0,
                   workspace: torch.Tensor | None = None):
    """Backward of flash_attn_fwd: returns (dQ, dK, dV) from the forward's q, k, v,
    o, lse and the upstream gradient do (all [B,H,S,D] bf16 CUDA tensors; lse fp32)."""
    B, Hq, S_q, D = q.shape
    Hkv, S_kv = k.shape[1], k.shape[2]
    _check(q, (B, Hq, S_q, D), "q")
    _check(k, (B, Hkv, S_kv, D), "k")
    _check(v, (B, Hkv, S_kv, D), "v")
    _check(o, (B, Hq, S_q, D), "o")
    _check(do, (B, Hq, S_q, D), "do")
    _check(lse, (B, Hq, S_q), "lse", torch.float32)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    from ._lib import lib
    ws_b = int(lib().amp_flash_attn_bwd_workspace_bytes(B, Hq, S_q))
    ws = workspace if workspace is not None else torch.empty(ws_b, dtype=torch.uint8,
                                                             device=q.device)
    call("amp_flash_attn_bwd_bf16_dev", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
         do.data_ptr(), lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, Hq, Hkv,
         S_q, S_kv, D, 1 if causal else 0, float(scale), ws.data_ptr(), ws.numel(),
         torch.cuda.current_stream(q.device).cuda_stream)
    return dq, dk, dv
