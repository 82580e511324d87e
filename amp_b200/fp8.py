"""FP8 E4M3 amax-scaled quantise / dequantise on the device.

Host-side mirror of the reference's FP8 codec surface (``AMP::fp8::f32_to_e4m3``
and ``e4m3_to_f32``, include/fp8.hpp:15-63), lifted from scalars to whole
device tensors with a per-tensor amax scale.  All arithmetic runs in
libamp_b200.so; torch only provides device memory and the current stream.
"""
from __future__ import annotations

import torch

from ._lib import call, lib

E4M3_MAX = 448.0


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _check_bf16(x: torch.Tensor) -> None:
    if not x.is_cuda or x.dtype != torch.bfloat16 or not x.is_contiguous():
        raise ValueError("expected a contiguous bfloat16 CUDA tensor")


def workspace_bytes(n: int) -> int:
    return int(lib().amp_fp8_quant_workspace_bytes(n))


def quantize_e4m3(x: torch.Tensor, workspace: torch.Tensor | None = None,
                  out: torch.Tensor | None = None, scale: torch.Tensor | None = None,
                  amax: torch.Tensor | None = None):
    """Per-tensor quantise: returns (codes uint8 shaped like x, scale float32[1]).

    scale = amax/448 (1 if amax == 0); codes = E4M3_RNE_sat(x / scale).
    """
    _check_bf16(x)
    n = x.numel()
    dev = x.device
    q = out if out is not None else torch.empty(x.shape, dtype=torch.uint8, device=dev)
    s = scale if scale is not None else torch.empty(1, dtype=torch.float32, device=dev)
    ws_b = workspace_bytes(n)
    ws = workspace if workspace is not None else torch.empty(ws_b, dtype=torch.uint8, device=dev)
    call("amp_fp8_quant_e4m3_dev", x.data_ptr(), n, q.data_ptr(), s.data_ptr(),
         amax.data_ptr() if amax is not None else None, ws.data_ptr(), ws.numel(), _stream(dev))
    return q, s


def amax_bf16(x: torch.Tensor, workspace: torch.Tensor | None = None,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """max |x| of a bf16 tensor into a float32[1] device tensor (NaN ignored)."""
    _check_bf16(x)
    dev = x.device
    a = out if out is not None else torch.empty(1, dtype=torch.float32, device=dev)
    ws_b = workspace_bytes(x.numel())
    ws = workspace if workspace is not None else torch.empty(ws_b, dtype=torch.uint8, device=dev)
    call("amp_fp8_amax_bf16_dev", x.data_ptr(), x.numel(), a.data_ptr(), ws.data_ptr(),
         ws.numel(), _stream(dev))
    return a


def amax_allreduce_peer(x: torch.Tensor, mailboxes, workspace: torch.Tensor | None = None,
                        out: torch.Tensor | None = None) -> torch.Tensor:
    """max |x| over the shards of every rank: this rank's amax swapped with the
    others through `mailboxes` (a collective.PeerMailboxes); no NCCL call."""
    _check_bf16(x)
    dev = x.device
    a = out if out is not None else torch.empty(1, dtype=torch.float32, device=dev)
    ws_b = workspace_bytes(x.numel())
    ws = workspace if workspace is not None else torch.empty(ws_b, dtype=torch.uint8, device=dev)
    call("amp_fp8_amax_allreduce_peer_dev", x.data_ptr(), x.numel(), a.data_ptr(), ws.data_ptr(),
         ws.numel(), mailboxes.table.data_ptr(), mailboxes.g.rank, mailboxes.g.world,
         mailboxes.next_seq(), _stream(dev))
    return a


def quantize_e4m3_from_amax(x: torch.Tensor, amax: torch.Tensor,
                            out: torch.Tensor | None = None,
                            scale: torch.Tensor | None = None):
    """Quantise with an externally supplied amax (e.g. all-reduced over ranks)."""
    _check_bf16(x)
    dev = x.device
    q = out if out is not None else torch.empty(x.shape, dtype=torch.uint8, device=dev)
    s = scale if scale is not None else torch.empty(1, dtype=torch.float32, device=dev)
    call("amp_fp8_quant_e4m3_from_amax_dev", x.data_ptr(), x.numel(), amax.data_ptr(),
         q.data_ptr(), s.data_ptr(), _stream(dev))
    return q, s


def dequantize_e4m3(q: torch.Tensor, scale: torch.Tensor,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16_RNE(e4m3_to_f32(q) * scale)."""
    if not q.is_cuda or q.dtype != torch.uint8 or not q.is_contiguous():
        raise ValueError("expected a contiguous uint8 CUDA tensor of E4M3 codes")
    dev = q.device
    y = out if out is not None else torch.empty(q.shape, dtype=torch.bfloat16, device=dev)
    call("amp_fp8_dequant_e4m3_dev", q.data_ptr(), q.numel(), scale.data_ptr(), y.data_ptr(),
         _stream(dev))
    return y
