"""FP8 E4M3 quantise/dequantise on the B200 vs the oracle: codes bit-exact.

Full size is the 2^26-element workload (N(0,1) + 0.1% N(0,50) outliers);
small and ragged sizes cover the vector/tail split and misaligned pointers.
"""
import numpy as np
import pytest
import torch

import oracle
from amp_b200 import fp8, workloads
from amp_b200._lib import call

pytestmark = pytest.mark.gpu


def to_dev_bf16(bits: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(bits.view(np.int16).copy()).to(device).view(torch.bfloat16)


def bits_of(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def same_bf16(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    nan_a = (a & 0x7FFF) > 0x7F80
    nan_b = (b & 0x7FFF) > 0x7F80
    return (a == b) | (nan_a & nan_b)


def check(bits: np.ndarray, cuda):
    x = to_dev_bf16(bits, cuda)
    q, s = fp8.quantize_e4m3(x)
    y = fp8.dequantize_e4m3(q, s)
    torch.cuda.synchronize()
    q_ref, s_ref, a_ref = oracle.quant_e4m3(bits)
    assert s.item() == np.float32(s_ref)
    got = q.cpu().numpy()
    bad = np.nonzero(got != q_ref)[0]
    assert bad.size == 0, f"{bad.size} code mismatches, first at {bad[:5]}: " \
        f"x={oracle.bf16_bits_to_f32(bits[bad[:5]])} got={got[bad[:5]]} want={q_ref[bad[:5]]}"
    y_ref = oracle.dequant_e4m3(q_ref, s_ref)
    assert same_bf16(bits_of(y), y_ref).all()


@pytest.mark.parametrize("n", [1, 7, 15, 16, 17, 255, 4096, 4099, 100_003])
def test_small_and_ragged(n, cuda, amp_lib):
    check(workloads.quant_input_numpy(n, seed=n), cuda)


def test_full_size_workload_bit_exact(cuda, amp_lib):
    check(workloads.quant_input_numpy(workloads.QUANT_N, seed=0), cuda)


def test_empty_tensor(cuda, amp_lib):
    x = torch.empty(0, dtype=torch.bfloat16, device=cuda)
    q, s = fp8.quantize_e4m3(x)
    assert q.numel() == 0 and s.item() == 1.0
    assert fp8.dequantize_e4m3(q, s).numel() == 0


def test_zeros_and_signed_zero(cuda, amp_lib):
    bits = np.array([0x0000, 0x8000] * 20, np.uint16)
    check(bits, cuda)


def test_saturation_nan_inf_and_subnormals(cuda, amp_lib):
    vals = np.array([448, -448, 464, 465, 1e30, -1e30, 2 ** -9, 2 ** -10, 3 * 2 ** -10,
                     7.5 * 2 ** -9, 0.0, -0.0, 1.0, -1.0, 0.3, 100.0] * 3, np.float32)
    bits = oracle.f32_to_bf16_bits(vals)
    check(bits, cuda)
    # a NaN element: ignored by amax, encodes to the NaN code
    bits_nan = bits.copy()
    bits_nan[5] = 0x7FC1
    bits_nan[9] = 0xFFC0
    check(bits_nan, cuda)


def test_misaligned_pointers_use_scalar_path(cuda, amp_lib):
    bits = workloads.quant_input_numpy(10_001, seed=5)
    base = to_dev_bf16(np.concatenate([np.zeros(1, np.uint16), bits]), cuda)
    x = base[1:]  # 2-byte offset: not 16-byte aligned
    assert x.data_ptr() % 16 != 0
    qbuf = torch.empty(bits.size + 3, dtype=torch.uint8, device=cuda)
    q = qbuf[3:]
    fp8.quantize_e4m3(x, out=q)
    q_ref, _, _ = oracle.quant_e4m3(bits)
    assert (q.cpu().numpy() == q_ref).all()


def test_sharded_amax_then_encode(cuda, amp_lib):
    bits = workloads.quant_input_numpy(1 << 20, seed=9)
    x = to_dev_bf16(bits, cuda)
    a = fp8.amax_bf16(x)
    q, s = fp8.quantize_e4m3_from_amax(x, a)
    q_ref, s_ref, a_ref = oracle.quant_e4m3(bits)
    assert a.item() == np.float32(a_ref) and s.item() == np.float32(s_ref)
    assert (q.cpu().numpy() == q_ref).all()
    # a larger external amax (e.g. another rank's) changes the codes as the oracle says
    a2 = torch.tensor([a_ref * 3.0], dtype=torch.float32, device=cuda)
    q2, _ = fp8.quantize_e4m3_from_amax(x, a2)
    assert (q2.cpu().numpy() == oracle.quant_e4m3_with_amax(bits, np.float32(a_ref * 3.0))).all()


def test_host_pointer_entry_points(cuda, amp_lib):
    import ctypes as C
    bits = workloads.quant_input_numpy(123_457, seed=11)
    q = np.empty(bits.size, np.uint8)
    y = np.empty(bits.size, np.uint16)
    s = C.c_float()
    call("amp_user_fp8_quant_e4m3", bits.ctypes.data, bits.size, q.ctypes.data, C.byref(s),
         y.ctypes.data)
    q_ref, s_ref, _ = oracle.quant_e4m3(bits)
    assert s.value == np.float32(s_ref) and (q == q_ref).all()
    assert same_bf16(y, oracle.dequant_e4m3(q_ref, s_ref)).all()
    y2 = np.empty_like(y)
    call("amp_user_fp8_dequant_e4m3", q.ctypes.data, q.size, s.value, y2.ctypes.data)
    assert same_bf16(y2, y).all()


def test_every_bf16_value_over_many_scales(cuda, amp_lib):
    """Every finite bf16 value against the oracle under scales spread over 40
    binades (amax injected), including subnormal-range and saturating codes."""
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    finite = (bits & 0x7F80) != 0x7F80
    bits = bits[finite]
    x = to_dev_bf16(bits, cuda)
    rng = np.random.default_rng(77)
    amaxes = np.concatenate([np.float32(448.0) * np.ldexp(1.0 + rng.random(150), rng.integers(-20, 20, 150)),
                             rng.uniform(100, 500, 50), [1e-40, 3e38]]).astype(np.float32)
    for a in amaxes:
        q, _ = fp8.quantize_e4m3_from_amax(x, torch.tensor([a], device=cuda))
        want = oracle.quant_e4m3_with_amax(bits, a)
        got = q.cpu().numpy()
        assert np.array_equal(got, want), (a, np.count_nonzero(got != want))


def test_caller_buffers_are_checked_before_launch(cuda, amp_lib):
    """Buffers a caller hands in are checked on the host (dtype, device, size),
    since the kernels write through their pointers."""
    x = torch.zeros(1000, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError, match="out"):
        fp8.quantize_e4m3(x, out=torch.empty(999, dtype=torch.uint8, device=cuda))
    with pytest.raises(ValueError, match="scale"):
        fp8.quantize_e4m3(x, scale=torch.empty(1, dtype=torch.float64, device=cuda))
    with pytest.raises(ValueError, match="workspace"):
        fp8.quantize_e4m3(x, workspace=torch.empty(16, dtype=torch.uint8, device=cuda))
    with pytest.raises(ValueError, match="amax"):
        fp8.quantize_e4m3_from_amax(x, torch.zeros(1))
    with pytest.raises(ValueError, match="out"):
        fp8.amax_bf16(x, out=torch.empty(1, dtype=torch.float16, device=cuda))
    q, s = fp8.quantize_e4m3(x)
    with pytest.raises(ValueError, match="out"):
        fp8.dequantize_e4m3(q, s, out=torch.empty(1000, dtype=torch.float32, device=cuda))
    with pytest.raises(ValueError, match="scale"):
        fp8.dequantize_e4m3(q, s.cpu())
    torch.cuda.synchronize()
