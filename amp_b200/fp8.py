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


def _check_buf(t: torch.Tensor | None, dtype, n: int, device, name: str) -> None:
    """A caller-supplied buffer (None: allocated here) holds at least n elements of
    dtype, contiguous, on the input's device: the kernels write through its pointer."""
    if t is None:
        return
    if not t.is_cuda or t.device != device or t.dtype != dtype or not t.is_contiguous() \
            or t.numel() < n:
        raise ValueError(f"{name}: expected a contiguous {dtype} tensor of >= {n} elements on "
                         f"{device}, got {t.dtype} {tuple(t.shape)} on {t.device}")


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
    ws_b = workspace_bytes(n)
    _check_buf(out, torch.uint8, n, dev, "out")
    _check_buf(scale, torch.float32, 1, dev, "scale")
    _check_buf(amax, torch.float32, 1, dev, "amax")
    _check_buf(workspace, torch.uint8, ws_b, dev, "workspace")
    q = out if out is not None else torch.empty(x.shape, dtype=torch.uint8, device=dev)
    s = scale if scale is not None else torch.empty(1, dtype=torch.float32, device=dev)
    ws = workspace if workspace is not None else torch.empty(ws_b, dtype=torch.uint8, device=dev)
    call("amp_fp8_quant_e4m3_dev", x.data_ptr(), n, q.data_ptr(), s.data_ptr(),
         amax.data_ptr() if amax is not None else None, ws.data_ptr(), ws.numel(), _stream(dev))
    return q, s


def amax_bf16(x: torch.Tensor, workspace: torch.Tensor | None = None,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """max |x| of a bf16 tensor into a float32[1] device tensor (NaN ignored)."""
    _check_bf16(x)
    dev = x.device
    ws_b = workspace_bytes(x.numel())
    _check_buf(out, torch.float32, 1, dev, "out")
    _check_buf(workspace, torch.uint8, ws_b, dev, "workspace")
    a = out if out is not None else torch.empty(1, dtype=torch.float32, device=dev)
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
    ws_b = workspace_bytes(x.numel())
    _check_buf(out, torch.float32, 1, dev, "out")
    _check_buf(workspace, torch.uint8, ws_b, dev, "workspace")
    a = out if out is not None else torch.empty(1, dtype=torch.float32, device=dev)
    ws = workspace if workspace is not None else torch.empty(ws_b, dtype=torch.uint8, device=dev)
    with mailboxes.sequence() as seq:
        call("amp_fp8_amax_allreduce_peer_dev", x.data_ptr(), x.numel(), a.data_ptr(),
             ws.data_ptr(), ws.numel(), mailboxes.table.data_ptr(), mailboxes.g.rank,
             mailboxes.g.world, seq, _stream(dev))
    return a


def quantize_e4m3_from_amax(x: torch.Tensor, amax: torch.Tensor,
                            out: torch.Tensor | None = None,
                            scale: torch.Tensor | None = None):
    """Quantise with an externally supplied amax (e.g. all-reduced over ranks)."""
    _check_bf16(x)
    dev = x.device
    _check_buf(amax, torch.float32, 1, dev, "amax")
    _check_buf(out, torch.uint8, x.numel(), dev, "out")
    _check_buf(scale, torch.float32, 1, dev, "scale")
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
    _check_buf(scale, torch.float32, 1, dev, "scale")
    _check_buf(out, torch.bfloat16, q.numel(), dev, "out")
    y = out if out is not None else torch.empty(q.shape, dtype=torch.bfloat16, device=dev)
    call("amp_fp8_dequant_e4m3_dev", q.data_ptr(), q.numel(), scale.data_ptr(), y.data_ptr(),
         _stream(dev))
    return y
