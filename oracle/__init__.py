"""CPU oracle for AMP's hot path -- TEST INFRASTRUCTURE ONLY.

This package is the checker: only tests/, ``__graft_entry__.smoke()`` and
bench.py's CPU-baseline / reference legs may import it.  The product
(``amp_b200``) never imports or calls anything here.

  * ``liboracle.so`` (oracle.c): bit-exact E4M3 codec, amax quantiser,
    AMP's fp32 CPU GEMM and an fp64 GEMM.
  * ``attention.py``: fp64 FlashAttention-2 forward / paged-KV restatement.
  * ``parity_dump.py``: the oracle ("B") side of the parity dumps of the
    extension ops, in the dump tool's file layout.
  * ``_ref/`` (built by ``make -C oracle ref`` from the reference sources in
    place): AMP's own FP8 codec and its ``amp_validate_kernel`` binary.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libampref.so"
REF_VALIDATOR = HERE / "_ref" / "amp_validate_kernel"

_o: C.CDLL | None = None
_r: C.CDLL | None = None


def build(ref: bool = False) -> None:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    if ref:
        subprocess.run(["make", "-s", "-C", str(HERE), "ref"], check=True)


def _vp(a: np.ndarray) -> int:
    return a.ctypes.data


def lib() -> C.CDLL:
    global _o
    if _o is None:
        if not LIB.exists():
            build()
        o = C.CDLL(str(LIB))
        vp, i64, i32, f32 = C.c_void_p, C.c_int64, C.c_int, C.c_float
        sig = {
            "orc_bf16_to_f32": (f32, [C.c_uint16]),
            "orc_f32_to_bf16": (C.c_uint16, [f32]),
            "orc_e4m3_to_f32": (f32, [C.c_uint8]),
            "orc_f32_to_e4m3_rne": (C.c_uint8, [f32]),
            "orc_f32_to_e4m3_ampcompat": (C.c_uint8, [f32]),
            "orc_f32_to_e4m3_rne_n": (None, [vp, i64, vp]),
            "orc_f32_to_e4m3_ampcompat_n": (None, [vp, i64, vp]),
            "orc_amax_bf16": (f32, [vp, i64]),
            "orc_scale_from_amax": (f32, [f32]),
            "orc_inv_scale": (f32, [f32]),
            "orc_quant_e4m3": (None, [vp, i64, vp, vp, vp]),
            "orc_quant_e4m3_with_amax": (None, [vp, i64, f32, vp]),
            "orc_dequant_e4m3": (None, [vp, i64, f32, vp]),
            "orc_quant_e4m3_rows": (None, [vp, i64, i64, vp, vp]),
            "orc_quant_e4m3_cols": (None, [vp, i64, i64, vp, vp]),
            "orc_gemm_fp32_amp": (None, [vp, vp, vp, i32, i32, i32]),
            "orc_gemm_f64": (None, [vp, vp, vp, i32, i32, i32]),
            "orc_amp_harness_fill": (None, [C.c_uint, vp, i64, vp, i64]),
        }
        for k, (res, args) in sig.items():
            f = getattr(o, k)
            f.restype, f.argtypes = res, args
        _o = o
    return _o


def ref_lib() -> C.CDLL | None:
    """AMP's own codec compiled from the reference sources, or None if not built."""
    global _r
    if _r is None and REF_LIB.exists():
        r = C.CDLL(str(REF_LIB))
        r.ref_f32_to_e4m3.restype, r.ref_f32_to_e4m3.argtypes = C.c_uint8, [C.c_float]
        r.ref_e4m3_to_f32.restype, r.ref_e4m3_to_f32.argtypes = C.c_float, [C.c_uint8]
        r.ref_f32_to_e4m3_n.restype = None
        r.ref_f32_to_e4m3_n.argtypes = [C.c_void_p, C.c_int64, C.c_void_p]
        r.ref_quant_dequant_bf16.restype = C.c_float
        r.ref_quant_dequant_bf16.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_int]
        _r = r
    return _r


_rg: C.CDLL | None = None
REF_GEMM_LIB = HERE / "_ref" / "libampref_gemm.so"


def ref_gemm_lib() -> C.CDLL | None:
    """AMP's cpu_reference_gemm compiled from the reference sources, or None."""
    global _rg
    if _rg is None and REF_GEMM_LIB.exists():
        g = C.CDLL(str(REF_GEMM_LIB))
        vp, i32 = C.c_void_p, C.c_int
        g.ref_cpu_reference_gemm.restype = None
        g.ref_cpu_reference_gemm.argtypes = [vp, vp, vp, i32, i32, i32]
        g.ref_cpu_reference_gemm_mt.restype = None
        g.ref_cpu_reference_gemm_mt.argtypes = [vp, vp, vp, i32, i32, i32, i32]
        _rg = g
    return _rg


# --------------------------------------------------------------------------
# numpy conveniences (bf16 carried as uint16 bit patterns)
# --------------------------------------------------------------------------

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (vectorised restatement)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) & 0x8000 | 0x7FC0).astype(np.uint16)
    return r


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)


def e4m3_encode(x: np.ndarray, mode: str = "rne") -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    q = np.empty(x.shape, np.uint8)
    fn = lib().orc_f32_to_e4m3_rne_n if mode == "rne" else lib().orc_f32_to_e4m3_ampcompat_n
    fn(_vp(x), x.size, _vp(q))
    return q


def e4m3_decode_table() -> np.ndarray:
    return np.array([lib().orc_e4m3_to_f32(i) for i in range(256)], np.float32)


def quant_e4m3(x_bf16: np.ndarray):
    """Per-tensor quantise; returns (codes, scale, amax)."""
    x = np.ascontiguousarray(x_bf16, np.uint16)
    q = np.empty(x.shape, np.uint8)
    s, a = C.c_float(), C.c_float()
    lib().orc_quant_e4m3(_vp(x), x.size, _vp(q), C.byref(s), C.byref(a))
    return q, s.value, a.value


def quant_e4m3_with_amax(x_bf16: np.ndarray, amax: float) -> np.ndarray:
    x = np.ascontiguousarray(x_bf16, np.uint16)
    q = np.empty(x.shape, np.uint8)
    lib().orc_quant_e4m3_with_amax(_vp(x), x.size, amax, _vp(q))
    return q


def dequant_e4m3(q: np.ndarray, scale: float) -> np.ndarray:
    q = np.ascontiguousarray(q, np.uint8)
    y = np.empty(q.shape, np.uint16)
    lib().orc_dequant_e4m3(_vp(q), q.size, scale, _vp(y))
    return y


def quant_e4m3_rows(x_bf16: np.ndarray):
    x = np.ascontiguousarray(x_bf16, np.uint16)
    rows, cols = x.shape
    q = np.empty(x.shape, np.uint8)
    s = np.empty(rows, np.float32)
    lib().orc_quant_e4m3_rows(_vp(x), rows, cols, _vp(q), _vp(s))
    return q, s


def quant_e4m3_cols(x_bf16: np.ndarray):
    x = np.ascontiguousarray(x_bf16, np.uint16)
    rows, cols = x.shape
    q = np.empty(x.shape, np.uint8)
    s = np.empty(cols, np.float32)
    lib().orc_quant_e4m3_cols(_vp(x), rows, cols, _vp(q), _vp(s))
    return q, s


def gemm_fp32_amp(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """AMP's cpu_reference_gemm (fp32 accumulate, i-j-k)."""
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    M, K = A.shape
    N = B.shape[1]
    Cm = np.empty((M, N), np.float32)
    lib().orc_gemm_fp32_amp(_vp(A), _vp(B), _vp(Cm), M, N, K)
    return Cm


def gemm_f64(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    return np.asarray(A, np.float64) @ np.asarray(B, np.float64)


def amp_harness_inputs(M: int, N: int, K: int, seed: int = 42):
    """Inputs exactly as tests/amp_validate_kernel.cpp:84-86 generates them."""
    A = np.empty(M * K, np.float32)
    B = np.empty(K * N, np.float32)
    lib().orc_amp_harness_fill(seed, _vp(A), A.size, _vp(B), B.size)
    return A.reshape(M, K), B.reshape(K, N)


def ref_sched_lib() -> C.CDLL | None:
    """AMP's Scheduler + PagePoolFast (CPU backend) behind a C driver, if built."""
    path = HERE / "_ref" / "libampref_sched.so"
    if not path.exists():
        return None
    r = C.CDLL(str(path))
    vp, i32 = C.c_void_p, C.c_int
    r.refsched_create.restype, r.refsched_create.argtypes = vp, [i32] * 5
    r.refsched_destroy.restype, r.refsched_destroy.argtypes = None, [vp]
    r.refsched_add.restype, r.refsched_add.argtypes = i32, [vp, i32, i32]
    r.refsched_step.restype = i32
    r.refsched_step.argtypes = [vp, vp, vp, vp, i32, i32]
    return r


class RefScheduler:
    """Steps AMP's own scheduler and returns each batch as numpy arrays:
    entries [n, 5] (seq id, is_prefill, n_tokens, prefill_start, ctx) and the
    per-entry page lists."""

    def __init__(self, lib_, page_tokens=16, max_pages=2048, max_batch_tokens=4096,
                 max_seqs=256, max_prefill=512):
        self.r = lib_
        self.h = lib_.refsched_create(page_tokens, max_pages, max_batch_tokens, max_seqs,
                                      max_prefill)

    def add(self, prompt_len: int, max_new_tokens: int) -> int:
        return self.r.refsched_add(self.h, prompt_len, max_new_tokens)

    def step(self, cap: int = 1024, pages_cap: int = 1 << 16):
        ent = np.zeros((cap, 5), np.int32)
        pages = np.zeros(pages_cap, np.int32)
        start = np.zeros(cap + 1, np.int32)
        n = self.r.refsched_step(self.h, _vp(ent), _vp(pages), _vp(start), cap, pages_cap)
        if n < 0:
            raise RuntimeError(f"refsched_step: {n}")
        return ent[:n].copy(), [pages[start[i]:start[i + 1]].copy() for i in range(n)]

    def close(self):
        if self.h:
            self.r.refsched_destroy(self.h)
            self.h = None


def max_rel_err(out: np.ndarray, ref: np.ndarray) -> float:
    """AMP's metric: max |out-ref| / max(1, |ref|) (amp_validate_kernel.cpp:103-109)."""
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    if out.size == 0:
        return 0.0
    return float(np.max(np.abs(out - ref) / np.maximum(1.0, np.abs(ref))))
