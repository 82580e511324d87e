"""bf16 and FP8 E4M3 tensor-core GEMM on the B200 vs the fp64 oracle.

Bars (AMP's metric, max|x-ref|/max(1,|ref|)): bf16 < 2e-2, FP8 < 6e-2 against
an fp64 GEMM of the exact operand values (the dequantised codes for FP8).
"""
import numpy as np
import pytest
import torch

import oracle
from amp_b200 import gemm
from amp_b200._lib import AmpError, lib

pytestmark = pytest.mark.gpu
TOL_BF16 = 2e-2
TOL_FP8 = 6e-2


def bf16_operands(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    A = torch.randn(M, K, generator=g).to(torch.bfloat16)
    B = torch.randn(K, N, generator=g).to(torch.bfloat16)
    return A, B


def run_bf16(A, B, out_dtype=torch.float32):
    M, K = A.shape
    N = B.shape[1]
    dA, dB = A.cuda(), B.cuda()
    dC = torch.full((M, N), float("nan"), dtype=out_dtype, device="cuda")
    gemm.launch_matmul_bf16(dA, dB, dC, M, N, K)
    torch.cuda.synchronize()
    assert lib().amp_device_status(1) == 0
    return dC.float().cpu().numpy()


def ref64(A, B):
    return A.double().numpy() @ B.double().numpy()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (128, 256, 128), (256, 512, 1024),
                                   (100, 72, 40), (1, 8, 8), (300, 264, 200), (129, 257 + 7, 72)])
@pytest.mark.parametrize("out", [torch.float32, torch.bfloat16])
def test_bf16_small_and_ragged(M, N, K, out, cuda, amp_lib):
    A, B = bf16_operands(M, N, K, seed=M + N + K)
    C = run_bf16(A, B, out)
    err = oracle.max_rel_err(C, ref64(A, B))
    assert err < TOL_BF16, err


def test_bf16_4096_cube_fp32_out(cuda, amp_lib):
    A, B = bf16_operands(4096, 4096, 4096, seed=1)
    C = run_bf16(A, B)
    assert oracle.max_rel_err(C, ref64(A, B)) < TOL_BF16


def test_bf16_8192_cube_bf16_out(cuda, amp_lib):
    A, B = bf16_operands(8192, 8192, 8192, seed=2)
    C = run_bf16(A, B, torch.bfloat16)
    assert oracle.max_rel_err(C, ref64(A, B)) < TOL_BF16


@pytest.mark.parametrize("M,N,K", [(2488, 2008, 1000), (4096 + 136, 4096 - 56, 512)])
@pytest.mark.parametrize("out", [torch.float32, torch.bfloat16])
def test_bf16_pair_tiles_ragged(M, N, K, out, cuda, amp_lib):
    """Sizes with >= 74 tiles of 256 x 256 run on SM pairs (2-SM MMAs); M and N
    here end inside the second CTA's half of a tile."""
    A, B = bf16_operands(M, N, K, seed=M + 2 * N)
    C = run_bf16(A, B, out)
    assert oracle.max_rel_err(C, ref64(A, B)) < TOL_BF16


def test_bf16_rejects_unaligned_k(cuda, amp_lib):
    A, B = bf16_operands(64, 64, 60, seed=0)
    with pytest.raises(AmpError, match="multiples"):
        run_bf16(A, B)


def fp8_operands(M, N, K, seed):
    rng = np.random.default_rng(seed)
    a = oracle.f32_to_bf16_bits(rng.standard_normal((M, K), dtype=np.float32))
    b = oracle.f32_to_bf16_bits(rng.standard_normal((K, N), dtype=np.float32))
    qa, sa = oracle.quant_e4m3_rows(a)
    qb, sb = oracle.quant_e4m3_cols(b)
    return qa, sa, qb, sb, a, b


def run_fp8(qa, sa, qb, sb, out=torch.bfloat16):
    M, K = qa.shape
    N = qb.shape[1]
    dC = torch.full((M, N), float("nan"), dtype=out, device="cuda")
    gemm.launch_matmul_fp8e4m3(torch.from_numpy(qa).cuda(), torch.from_numpy(qb).cuda(), dC,
                               M, N, K, torch.from_numpy(sa).cuda(), torch.from_numpy(sb).cuda())
    torch.cuda.synchronize()
    assert lib().amp_device_status(1) == 0
    return dC.float().cpu().numpy()


def fp8_ref(qa, sa, qb, sb):
    dec = oracle.e4m3_decode_table().astype(np.float64)
    Af = dec[qa] * sa.astype(np.float64)[:, None]
    Bf = dec[qb] * sb.astype(np.float64)[None, :]
    return Af @ Bf


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (256, 512, 512), (100, 80, 48),
                                   (333, 272, 1024), (2440, 2000, 1008)])
@pytest.mark.parametrize("out", [torch.float32, torch.bfloat16])
def test_fp8_rowcol_scales_small(M, N, K, out, cuda, amp_lib):
    qa, sa, qb, sb, _, _ = fp8_operands(M, N, K, seed=M * 3 + N)
    C = run_fp8(qa, sa, qb, sb, out)
    assert oracle.max_rel_err(C, fp8_ref(qa, sa, qb, sb)) < TOL_FP8


def test_fp8_per_tensor_scale(cuda, amp_lib):
    rng = np.random.default_rng(5)
    M, N, K = 256, 256, 256
    a = oracle.f32_to_bf16_bits(rng.standard_normal((M, K), dtype=np.float32))
    b = oracle.f32_to_bf16_bits(rng.standard_normal((K, N), dtype=np.float32))
    qa, sa, _ = oracle.quant_e4m3(a)
    qb, sb, _ = oracle.quant_e4m3(b)
    dC = torch.empty((M, N), dtype=torch.float32, device="cuda")
    gemm.launch_matmul_fp8e4m3(torch.from_numpy(qa).cuda(), torch.from_numpy(qb).cuda(), dC,
                               M, N, K, sa, sb)
    torch.cuda.synchronize()
    ref = fp8_ref(qa, np.full(M, sa, np.float32), qb, np.full(N, sb, np.float32))
    assert oracle.max_rel_err(dC.cpu().numpy(), ref) < TOL_FP8


def test_fp8_4096_cube_vs_prequant(cuda, amp_lib):
    qa, sa, qb, sb, a, b = fp8_operands(4096, 4096, 4096, seed=9)
    C = run_fp8(qa, sa, qb, sb)
    assert oracle.max_rel_err(C, fp8_ref(qa, sa, qb, sb)) < TOL_FP8
    # information, not the bar: against the unquantised bf16 operands the error
    # is E4M3 quantisation noise (3 mantissa bits), a few percent of the range
    pre = oracle.bf16_bits_to_f32(a).astype(np.float64) @ oracle.bf16_bits_to_f32(b).astype(
        np.float64)
    assert np.abs(C - pre).max() / np.abs(pre).max() < 0.1


@pytest.mark.parametrize("M,N,K,rowcol", [(512, 768, 1024, True), (300, 784, 512, True),
                                          (2440, 2000, 512, True),
                                          (256, 256, 256, False)])
def test_fp8_output_quantisation_and_amax(M, N, K, rowcol, cuda, amp_lib):
    """amax_c is max |v| of the fp32 result exactly, and the E4M3 C is the
    quantiser's encode of that same fp32 result with scale_c = amax/448 --
    bit-exact against the oracle's codec applied to the kernel's own fp32 C."""
    if rowcol:
        qa, sa, qb, sb, _, _ = fp8_operands(M, N, K, seed=M + N)
        sa_d, sb_d = torch.from_numpy(sa).cuda(), torch.from_numpy(sb).cuda()
    else:
        rng = np.random.default_rng(M)
        qa, s_a, _ = oracle.quant_e4m3(oracle.f32_to_bf16_bits(
            rng.standard_normal((M, K), dtype=np.float32)))
        qb, s_b, _ = oracle.quant_e4m3(oracle.f32_to_bf16_bits(
            rng.standard_normal((K, N), dtype=np.float32)))
        sa_d, sb_d = s_a, s_b
    A8, B8 = torch.from_numpy(qa).cuda(), torch.from_numpy(qb).cuda()
    amax = torch.full((1,), -1.0, device="cuda")
    C32 = torch.empty(M, N, device="cuda")
    gemm.launch_matmul_fp8e4m3_ex(A8, B8, C32, M, N, K, sa_d, sb_d, amax_c=amax)
    torch.cuda.synchronize()
    c32 = C32.cpu().numpy()
    assert amax.item() == np.abs(c32).max()
    # bf16 output: same amax (taken before the conversion)
    amax_b = torch.zeros(1, device="cuda")
    Cb = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    gemm.launch_matmul_fp8e4m3_ex(A8, B8, Cb, M, N, K, sa_d, sb_d, amax_c=amax_b)
    # E4M3 output with the delayed-scaling scale of this result
    scale_c = np.float32(amax.item()) / np.float32(448.0)
    C8 = torch.empty(M, N, dtype=torch.uint8, device="cuda")
    amax_8 = torch.zeros(1, device="cuda")
    gemm.launch_matmul_fp8e4m3_ex(A8, B8, C8, M, N, K, sa_d, sb_d, scale_c=float(scale_c),
                                  amax_c=amax_8)
    torch.cuda.synchronize()
    assert lib().amp_device_status(1) == 0
    assert amax_b.item() == amax.item() and amax_8.item() == amax.item()
    inv = np.float32(oracle.lib().orc_inv_scale(ctypes_float(scale_c)))
    want = oracle.e4m3_encode((c32 * inv).astype(np.float32))
    assert np.array_equal(C8.cpu().numpy(), want)
    # and the dequantised codes stay within E4M3's half-step of the fp64 GEMM
    ref = fp8_ref(qa, np.broadcast_to(np.float32(sa_d) if not rowcol else sa, (M,)).astype(np.float32),
                  qb, np.broadcast_to(np.float32(sb_d) if not rowcol else sb, (N,)).astype(np.float32))
    dec = oracle.e4m3_decode_table().astype(np.float64)[C8.cpu().numpy()] * float(scale_c)
    assert np.abs(dec - ref).max() <= 0.07 * np.abs(ref).max()


def ctypes_float(x):
    import ctypes
    return ctypes.c_float(float(x))


def test_allgather_gemm_single_rank(cuda):
    """The fused all-gather GEMM on a group of one: the epilogue writes into the
    rank's own replicated C and the kernel's completion exchange posts to itself."""
    from amp_b200 import sharded
    from amp_b200._lib import lib
    from amp_b200.collective import CommGroup, PeerBuffer
    M, N, K = 384, 512, 320
    g = torch.Generator(device="cuda").manual_seed(21)
    A = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    B = torch.randn(K, N, generator=g, device="cuda").to(torch.bfloat16)
    ref = torch.empty(M, N, dtype=torch.float32, device="cuda")
    gemm.launch_matmul_bf16(A, B, ref, M, N, K)
    for dtype in (torch.bfloat16, torch.float32):
        pb = PeerBuffer(CommGroup(), M, N, dtype)
        try:
            for _ in range(3):
                C = sharded.matmul_allgather(A, B, pb)
                torch.cuda.synchronize()
                assert torch.equal(C.float(), ref.to(dtype).float())
            assert lib().amp_device_status(1) == 0
        finally:
            pb.close()
