"""The host mirror checks its arguments before any library call: tensors that
are not on a CUDA device (here: every tensor, there is no GPU) raise ValueError
and nothing reaches libamp_b200.so."""
import pytest
import torch

from amp_b200 import attention, fp8, gemm, paged


@pytest.fixture
def no_library_calls(monkeypatch):
    def fail(*a, **k):
        raise AssertionError("the library was called with unchecked arguments")
    for mod in (attention, fp8, gemm, paged):
        monkeypatch.setattr(mod, "call", fail)


def bf16(*shape):
    return torch.zeros(shape, dtype=torch.bfloat16)


CASES = {
    "matmul_fp32": lambda: gemm.launch_matmul(gemm.TileCfg(), torch.zeros(4, 4), torch.zeros(4, 4),
                                              torch.zeros(4, 4), 4, 4, 4),
    "matmul_bf16": lambda: gemm.launch_matmul_bf16(bf16(8, 8), bf16(8, 8), torch.zeros(8, 8),
                                                   8, 8, 8),
    "matmul_fp8": lambda: gemm.launch_matmul_fp8e4m3(torch.zeros(16, 16, dtype=torch.uint8),
                                                     torch.zeros(16, 16, dtype=torch.uint8),
                                                     torch.zeros(16, 16), 16, 16, 16),
    "matmul_fp8_wrong_type": lambda: gemm.launch_matmul_fp8e4m3(bf16(16, 16), bf16(16, 16),
                                                                torch.zeros(16, 16), 16, 16, 16),
    "flash_attn": lambda: attention.flash_attn_fwd(bf16(1, 2, 8, 128), bf16(1, 2, 8, 128),
                                                   bf16(1, 2, 8, 128)),
    "quantize": lambda: fp8.quantize_e4m3(bf16(64)),
    "quantize_fp32_input": lambda: fp8.quantize_e4m3(torch.zeros(64)),
    "dequantize": lambda: fp8.dequantize_e4m3(torch.zeros(64, dtype=torch.uint8), torch.ones(1)),
    "paged_decode": lambda: paged.paged_attn_decode(
        bf16(1, 8, 128), bf16(2, 2, 16, 128), bf16(2, 2, 16, 128),
        torch.zeros(1, 2, dtype=torch.int32), torch.ones(1, dtype=torch.int32), 16),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_host_tensors_are_rejected_before_the_library(name, no_library_calls):
    with pytest.raises(ValueError):
        CASES[name]()
