"""AMP's own GPU kernels beside amp_b200's, on the same device inputs.

oracle/_ref/libampref_gpu.so is built from the reference sources in place by
`make -C oracle ref_gpu` (kernels/matmul.cu's FP32 tiled and BF16 WMMA GEMMs,
the cuBLASLt FP8 GEMM behind kernels/matmul.cu:235-270, kernels/flash_attn.cu's
FA2 forward).  Each test checks that the two implementations agree and prints
both times (run with -s to see them); the FA2 comparisons use sequence lengths
that are multiples of AMP's 32-row query tile, the sizes for which its kernel's
barriers are uniform.
"""
import ctypes
from pathlib import Path

import pytest
import torch

from amp_b200 import fp8, workloads
from amp_b200._lib import lib

pytestmark = pytest.mark.gpu
REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libampref_gpu.so"
V = ctypes.c_void_p


@pytest.fixture(scope="module")
def ref(cuda):
    if not REF.exists():
        pytest.skip("oracle/_ref/libampref_gpu.so is not built (make -C oracle ref_gpu)")
    r = ctypes.CDLL(str(REF))
    r.refgpu_last_error.restype = ctypes.c_char_p
    return r


def ok(r, rc):
    assert rc == 0, r.refgpu_last_error().decode()


def time_ms(fn, reps=5):
    fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    return sorted(ts)[len(ts) // 2]


def report(what, ref_ms, amp_ms, flop, unit="TFLOP/s"):
    # flop / ms / 1e9 = TFLOP/s
    print(f"\n  {what}: AMP {ref_ms:.3f} ms ({flop / ref_ms / 1e9:.1f} {unit}) | "
          f"amp_b200 {amp_ms:.3f} ms ({flop / amp_ms / 1e9:.1f} {unit}) | "
          f"x{ref_ms / amp_ms:.1f}")


def rel(a, b):
    return float((a.double() - b.double()).abs().max() / max(1.0, b.double().abs().max()))


@pytest.mark.parametrize("tile", [(16, 16, 16), (32, 16, 16), (32, 32, 16), (32, 32, 32)])
def test_fp32_gemm_vs_amp_kernel(tile, ref):
    M = N = K = 1024
    A, B = (torch.from_numpy(x).cuda() for x in workloads.gemm_fp32_inputs(M, N, K, seed=0))
    C_ref = torch.empty(M, N, device="cuda")
    C = torch.empty(M, N, device="cuda")
    fr = lambda: ok(ref, ref.refgpu_matmul_fp32(*tile, V(A.data_ptr()), V(B.data_ptr()),
                                                 V(C_ref.data_ptr()), M, N, K))
    fa = lambda: lib().amp_gemm_fp32_tile_dev(*tile, V(A.data_ptr()), V(B.data_ptr()),
                                              V(C.data_ptr()), M, N, K, None)
    report(f"fp32 GEMM {M}^3 tile {tile}", time_ms(fr), time_ms(fa), 2.0 * M * N * K, "TFLOP/s")
    assert rel(C, C_ref) < 1e-4


@pytest.mark.parametrize("S", [1024, 4096])
def test_bf16_gemm_vs_amp_wmma(S, ref):
    g = torch.Generator(device="cuda").manual_seed(S)
    A = torch.randn(S, S, generator=g, device="cuda").to(torch.bfloat16)
    B = torch.randn(S, S, generator=g, device="cuda").to(torch.bfloat16)
    C_ref = torch.empty(S, S, device="cuda")
    C = torch.empty(S, S, device="cuda")
    fr = lambda: ok(ref, ref.refgpu_matmul_bf16(V(A.data_ptr()), V(B.data_ptr()),
                                                 V(C_ref.data_ptr()), S, S, S))
    fa = lambda: lib().amp_gemm_bf16_dev(V(A.data_ptr()), V(B.data_ptr()), V(C.data_ptr()), 0,
                                         S, S, S, None)
    report(f"bf16 GEMM {S}^3 (fp32 out)", time_ms(fr, 3), time_ms(fa), 2.0 * S ** 3, "TFLOP/s")
    assert rel(C, C_ref) < 1e-4


def test_fp8_gemm_vs_amp_cublaslt(ref):
    M = N = K = 4096
    g = torch.Generator(device="cuda").manual_seed(8)
    A = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    Bm = torch.randn(K, N, generator=g, device="cuda").to(torch.bfloat16)
    qa, sa = fp8.quantize_e4m3(A)
    qb, sb = fp8.quantize_e4m3(Bm)
    C_ref = torch.empty(M, N, device="cuda")
    C = torch.empty(M, N, device="cuda")
    rc = ref.refgpu_matmul_fp8e4m3(V(qa.data_ptr()), V(qb.data_ptr()), V(C_ref.data_ptr()),
                                   M, N, K, ctypes.c_float(sa.item()), ctypes.c_float(sb.item()))
    if rc != 0:
        msg = ref.refgpu_last_error().decode()
        print(f"\n  FP8 E4M3 GEMM {M}^3: AMP's cuBLASLt path failed here: {msg}")
        pytest.skip("AMP's cuBLASLt FP8 path does not run here: " + msg)
    fr = lambda: ok(ref, ref.refgpu_matmul_fp8e4m3(
        V(qa.data_ptr()), V(qb.data_ptr()), V(C_ref.data_ptr()), M, N, K,
        ctypes.c_float(sa.item()), ctypes.c_float(sb.item())))
    fa = lambda: lib().amp_gemm_fp8e4m3_dev(V(qa.data_ptr()), V(qb.data_ptr()), V(sa.data_ptr()),
                                            V(sb.data_ptr()), 1, V(C.data_ptr()), 0, M, N, K, None)
    report(f"FP8 E4M3 GEMM {M}^3 (cuBLASLt via AMP's VendorGemm, per call scale upload)",
           time_ms(fr), time_ms(fa), 2.0 * M * N * K, "TFLOP/s")
    assert rel(C, C_ref) < 1e-3


@pytest.mark.parametrize("causal", [True, False])
def test_flash_attn_vs_amp_kernel(causal, ref):
    B, H, S, D = 1, 8, 512, 128
    g = torch.Generator(device="cuda").manual_seed(int(causal))
    q, k, v = (torch.randn(B, H, S, D, generator=g, device="cuda").to(torch.bfloat16)
               for _ in range(3))
    o_ref, o = torch.empty_like(q), torch.empty_like(q)
    l_ref, l = (torch.empty(B, H, S, device="cuda") for _ in range(2))
    ok(ref, ref.refgpu_flash_attn_bf16(V(q.data_ptr()), V(k.data_ptr()), V(v.data_ptr()),
                                       V(o_ref.data_ptr()), V(l_ref.data_ptr()), B, H, H, S, S,
                                       D, int(causal), ctypes.c_float(0.0)))
    assert lib().amp_flash_attn_fwd_bf16_dev(V(q.data_ptr()), V(k.data_ptr()), V(v.data_ptr()),
                                             V(o.data_ptr()), V(l.data_ptr()), B, H, H, S, S, D,
                                             int(causal), ctypes.c_float(0.0), None) == 0
    torch.cuda.synchronize()
    assert rel(o.float(), o_ref.float()) < 2e-2
    assert float((l - l_ref).abs().max()) < 2e-3


def test_flash_attn_timing_vs_amp_kernel(ref):
    # B=4 H=32 D=128 causal as in the bench, at S=1024 so AMP's scalar kernel
    # stays well under a second
    B, H, S, D = 4, 32, 1024, 128
    g = torch.Generator(device="cuda").manual_seed(3)
    q, k, v = (torch.randn(B, H, S, D, generator=g, device="cuda").to(torch.bfloat16)
               for _ in range(3))
    o_ref, o = torch.empty_like(q), torch.empty_like(q)
    l_ref, l = (torch.empty(B, H, S, device="cuda") for _ in range(2))
    fr = lambda: ok(ref, ref.refgpu_flash_attn_bf16(
        V(q.data_ptr()), V(k.data_ptr()), V(v.data_ptr()), V(o_ref.data_ptr()),
        V(l_ref.data_ptr()), B, H, H, S, S, D, 1, ctypes.c_float(0.0)))
    fa = lambda: lib().amp_flash_attn_fwd_bf16_dev(
        V(q.data_ptr()), V(k.data_ptr()), V(v.data_ptr()), V(o.data_ptr()), V(l.data_ptr()),
        B, H, H, S, S, D, 1, ctypes.c_float(0.0), None)
    flops = 4.0 * B * H * D * S * (S + 1) / 2
    report(f"FA2 fwd causal B={B} H={H} S={S} D={D}", time_ms(fr, 3), time_ms(fa), flops,
           "TFLOP/s")
    assert rel(o.float(), o_ref.float()) < 2e-2
