"""Pins the GEMM oracle against AMP's own CPU reference GEMM.

tests/golden/amp_harness_gemm.json records AMP's validator run on the oracle's
restatement (max_rel_err 0); when the reference tree is present the restated
loop is also compared bit for bit with AMP's cpu_reference_gemm compiled from
tests/amp_validate_kernel.cpp.
"""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

GOLD = json.loads((Path(__file__).parent / "golden" / "amp_harness_gemm.json").read_text())


@pytest.mark.parametrize("case", GOLD["cases"], ids=lambda c: f"{c['M']}x{c['N']}x{c['K']}")
def test_harness_inputs_and_loop_match_golden(case, oracle_lib):
    A, B = oracle_lib.amp_harness_inputs(case["M"], case["N"], case["K"], case["seed"])
    assert hashlib.sha256(A.tobytes() + B.tobytes()).hexdigest() == case["inputs_sha256"]
    C = oracle_lib.gemm_fp32_amp(A, B)
    assert hashlib.sha256(C.tobytes()).hexdigest() == case["oracle_sha256"]
    # AMP's validator ran the same computation through its own loop: zero error
    assert case["validator_exit"] == 0 and case["validator_max_rel_err"] == 0
    # the dump prints 6 significant digits; the sums agree to that precision
    assert abs(case["output_sum"] - float(C.astype(np.float64).sum())) < 1e-3 * max(
        1.0, abs(case["output_sum"]))


def test_fp64_oracle_is_within_amp_bar_of_amp_loop(oracle_lib):
    A, B = oracle_lib.amp_harness_inputs(96, 96, 96, 42)
    assert oracle_lib.max_rel_err(oracle_lib.gemm_fp32_amp(A, B), oracle_lib.gemm_f64(A, B)) < 1e-3


def test_restated_loop_is_bit_identical_to_reference_function(oracle_lib):
    g = oracle_lib.ref_gemm_lib()
    if g is None:
        pytest.skip("oracle/_ref/libampref_gemm.so not built (reference tree absent)")
    for (M, N, K, seed) in [(96, 96, 96, 42), (37, 53, 71, 1), (128, 64, 300, 9)]:
        A, B = oracle_lib.amp_harness_inputs(M, N, K, seed)
        want = np.empty((M, N), np.float32)
        g.ref_cpu_reference_gemm(A.ctypes.data, B.ctypes.data, want.ctypes.data, M, N, K)
        assert np.array_equal(oracle_lib.gemm_fp32_amp(A, B).view(np.uint32), want.view(np.uint32))
        mt = np.empty((M, N), np.float32)
        g.ref_cpu_reference_gemm_mt(A.ctypes.data, B.ctypes.data, mt.ctypes.data, M, N, K, 3)
        assert np.array_equal(mt.view(np.uint32), want.view(np.uint32))


def test_attention_backward_oracle_matches_autograd():
    """The fp64 chain-rule backward the GPU backward is checked against agrees with
    torch autograd (an independent implementation) in fp64, causal and GQA."""
    import torch
    from oracle import attention as ref
    rng = np.random.default_rng(0)
    B, Hq, Hkv, S, D = 1, 4, 2, 37, 16
    q, k, v, do = (rng.standard_normal(s) for s in
                   ((B, Hq, S, D), (B, Hkv, S, D), (B, Hkv, S, D), (B, Hq, S, D)))
    for causal in (True, False):
        dq, dk, dv = ref.flash_attn_bwd(q, k, v, do, causal)
        tq, tk, tv = (torch.tensor(x, requires_grad=True) for x in (q, k, v))
        kk, vv = (t.repeat_interleave(Hq // Hkv, dim=1) for t in (tk, tv))
        s = tq @ kk.transpose(-1, -2) / np.sqrt(D)
        if causal:
            s = s.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool), 1), float("-inf"))
        (torch.softmax(s, -1) @ vv).backward(torch.tensor(do))
        for got, want in ((dq, tq.grad), (dk, tk.grad), (dv, tv.grad)):
            assert np.abs(got - want.numpy()).max() < 1e-12
