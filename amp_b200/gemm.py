"""GEMM launchers: host-side mirror of AMP's kernels/matmul.cuh API.

``launch_matmul(cfg, dA, dB, dC, M, N, K)`` mirrors ``AMP::launch_matmul``
(kernels/matmul.cuh:96-98): row-major fp32 operands on the device, the
TileCfg names one of AMP's four tile configs.  All work is done by
libamp_b200.so; tensors are torch device tensors.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ._lib import call

FP32_TILES = ((16, 16, 16), (32, 16, 16), (32, 32, 16), (32, 32, 32))


@dataclass
class TileCfg:
    """AMP's TileCfg (kernels/matmul.cuh:85-91): BM, BN, BK (+ FP8 scales)."""
    BM: int = 32
    BN: int = 32
    BK: int = 32
    scale_a: float = 1.0
    scale_b: float = 1.0


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _check(t: torch.Tensor, dtype, shape, name):
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous() or tuple(t.shape) != shape:
        raise ValueError(f"{name}: expected contiguous {dtype} CUDA tensor of shape {shape}, "
                         f"got {t.dtype} {tuple(t.shape)} on {t.device}")


def launch_matmul(cfg: TileCfg, dA: torch.Tensor, dB: torch.Tensor, dC: torch.Tensor,
                  M: int, N: int, K: int) -> None:
    """C = A @ B in fp32 (AMP::launch_matmul), accumulated in the order and
    rounding of AMP's CPU reference GEMM (bit-identical to it)."""
    _check(dA, torch.float32, (M, K), "A")
    _check(dB, torch.float32, (K, N), "B")
    _check(dC, torch.float32, (M, N), "C")
    call("amp_gemm_fp32_tile_dev", cfg.BM, cfg.BN, cfg.BK, dA.data_ptr(), dB.data_ptr(),
         dC.data_ptr(), M, N, K, _stream(dA))


def matmul_fp32(A: torch.Tensor, B: torch.Tensor, exact: bool = False) -> torch.Tensor:
    """C = A @ B in fp32.  exact=False: FFMA (one rounding per multiply-add);
    exact=True: product and sum rounded separately, k ascending, as AMP's CPU
    reference GEMM does (bit-identical to it)."""
    M, K = A.shape
    N = B.shape[1]
    C = torch.empty((M, N), dtype=torch.float32, device=A.device)
    _check(A, torch.float32, (M, K), "A")
    _check(B, torch.float32, (K, N), "B")
    call("amp_gemm_fp32_exact_dev" if exact else "amp_gemm_fp32_dev", A.data_ptr(), B.data_ptr(),
         C.data_ptr(), M, N, K, _stream(A))
    return C


def matmul_fp32_3xtf32(A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """C = A @ B for fp32 operands on the tensor cores (three TF32 products),
    opt-in: faster than matmul_fp32 at large sizes, with an error that grows with
    K (see amp_gemm_fp32_3xtf32_dev)."""
    M, K = A.shape
    N = B.shape[1]
    _check(A, torch.float32, (M, K), "A")
    _check(B, torch.float32, (K, N), "B")
    C = torch.empty((M, N), dtype=torch.float32, device=A.device)
    call("amp_gemm_fp32_3xtf32_dev", A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, _stream(A))
    return C


AMP_DTYPE = {torch.float32: 0, torch.bfloat16: 1}


def launch_matmul_bf16(dA: torch.Tensor, dB: torch.Tensor, dC: torch.Tensor,
                       M: int, N: int, K: int) -> None:
    """C = A @ B on the tensor cores (AMP::launch_matmul_bf16): A [M,K], B [K,N]
    bf16 row-major; C [M,N] fp32 (AMP's contract) or bf16."""
    _check(dA, torch.bfloat16, (M, K), "A")
    _check(dB, torch.bfloat16, (K, N), "B")
    if dC.dtype not in AMP_DTYPE:
        raise ValueError("C must be float32 or bfloat16")
    _check(dC, dC.dtype, (M, N), "C")
    call("amp_gemm_bf16_dev", dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), AMP_DTYPE[dC.dtype],
         M, N, K, _stream(dA))


def _scale_tensor(s, n, device, name):
    if isinstance(s, torch.Tensor):
        if s.dtype != torch.float32 or not s.is_cuda or not s.is_contiguous() or s.numel() != n:
            raise ValueError(f"{name}: expected a contiguous float32 CUDA tensor of {n} values")
        return s
    return torch.full((n,), float(s), dtype=torch.float32, device=device)


def launch_matmul_fp8e4m3(dA: torch.Tensor, dB: torch.Tensor, dC: torch.Tensor,
                          M: int, N: int, K: int, scale_a=1.0, scale_b=1.0) -> None:
    """C = (A8 @ B8) * sa * sb (AMP::launch_matmul_fp8e4m3).

    A [M,K] and B [K,N] hold E4M3 codes (uint8 or float8_e4m3fn).  Scales are
    per tensor (python floats or 1-element tensors, as in the reference) or
    per row of A ([M] tensor) and per column of B ([N] tensor)."""
    for t, shape, nm in ((dA, (M, K), "A"), (dB, (K, N), "B")):
        if t.dtype not in (torch.uint8, torch.float8_e4m3fn):
            raise ValueError(f"{nm}: expected E4M3 codes (uint8 / float8_e4m3fn)")
        _check(t, t.dtype, shape, nm)
    if dC.dtype not in AMP_DTYPE:
        raise ValueError("C must be float32 or bfloat16")
    _check(dC, dC.dtype, (M, N), "C")
    rowcol = isinstance(scale_a, torch.Tensor) and scale_a.numel() == M and M != 1 or \
        isinstance(scale_b, torch.Tensor) and scale_b.numel() == N and N != 1
    if rowcol:
        sa = _scale_tensor(scale_a, M, dA.device, "scale_a")
        sb = _scale_tensor(scale_b, N, dA.device, "scale_b")
        mode = 2
    else:
        sa = _scale_tensor(scale_a, 1, dA.device, "scale_a")
        sb = _scale_tensor(scale_b, 1, dA.device, "scale_b")
        mode = 1
    call("amp_gemm_fp8e4m3_dev", dA.data_ptr(), dB.data_ptr(), sa.data_ptr(), sb.data_ptr(), mode,
         dC.data_ptr(), AMP_DTYPE[dC.dtype], M, N, K, _stream(dA))


def launch_matmul_fp8e4m3_ex(dA: torch.Tensor, dB: torch.Tensor, dC: torch.Tensor,
                             M: int, N: int, K: int, scale_a, scale_b, scale_c=None,
                             amax_c: torch.Tensor | None = None) -> None:
    """FP8 GEMM with output-side quantisation (AMP's GemmDesc d_scale_c / d_amax_c).

    dC float32 / bfloat16: C = v;  uint8 / float8_e4m3fn: E4M3 codes of v / scale_c
    (the quantiser's encode).  amax_c, a float32[1] device tensor, receives max |v|.
    v = scale_a * scale_b * (A8 @ B8); scales as in launch_matmul_fp8e4m3."""
    for t, shape, nm in ((dA, (M, K), "A"), (dB, (K, N), "B")):
        if t.dtype not in (torch.uint8, torch.float8_e4m3fn):
            raise ValueError(f"{nm}: expected E4M3 codes (uint8 / float8_e4m3fn)")
        _check(t, t.dtype, shape, nm)
    if dC.dtype in (torch.uint8, torch.float8_e4m3fn):
        c_dtype = 2
        if scale_c is None:
            raise ValueError("an E4M3 C needs scale_c")
    elif dC.dtype in AMP_DTYPE:
        c_dtype = AMP_DTYPE[dC.dtype]
    else:
        raise ValueError("C must be float32, bfloat16 or E4M3 codes")
    _check(dC, dC.dtype, (M, N), "C")
    rowcol = isinstance(scale_a, torch.Tensor) and scale_a.numel() == M and M != 1 or \
        isinstance(scale_b, torch.Tensor) and scale_b.numel() == N and N != 1
    n_a, n_b, mode = (M, N, 2) if rowcol else (1, 1, 1)
    sa = _scale_tensor(scale_a, n_a, dA.device, "scale_a")
    sb = _scale_tensor(scale_b, n_b, dA.device, "scale_b")
    sc = _scale_tensor(scale_c, 1, dA.device, "scale_c") if scale_c is not None else None
    if amax_c is not None and (amax_c.dtype != torch.float32 or amax_c.numel() < 1
                               or not amax_c.is_cuda):
        raise ValueError("amax_c must be a float32 CUDA tensor")
    call("amp_gemm_fp8e4m3_ex_dev", dA.data_ptr(), dB.data_ptr(), sa.data_ptr(), sb.data_ptr(),
         mode, dC.data_ptr(), c_dtype, sc.data_ptr() if sc is not None else None,
         amax_c.data_ptr() if amax_c is not None else None, M, N, K, _stream(dA))
