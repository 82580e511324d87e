"""fp32 GEMM (AMP's plugin contract) on the B200 vs the oracle.

Bars: the exact form (the plugin, launch_matmul / the tile launcher behind the
parity dump) is bit-identical to AMP's own fp32 CPU GEMM (the oracle's
restatement of cpu_reference_gemm, itself pinned against the reference's
compiled loop), and within AMP's metric max|x-ref|/max(1,|ref|) < 1e-3 of
fp64; the FFMA form is within 1e-3 of fp64.
"""
import json
import subprocess

import numpy as np
import pytest
import torch

import oracle
from amp_b200 import gemm, workloads, LIB_PATH
from amp_b200._lib import AmpError, call

pytestmark = pytest.mark.gpu
TOL = 1e-3


def run_dev(A, B, tile=(32, 32, 32)):
    M, K = A.shape
    N = B.shape[1]
    dA = torch.from_numpy(A).cuda()
    dB = torch.from_numpy(B).cuda()
    dC = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    gemm.launch_matmul(gemm.TileCfg(*tile), dA, dB, dC, M, N, K)
    torch.cuda.synchronize()
    return dC.cpu().numpy()


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (33, 17, 5), (96, 96, 96), (127, 129, 65),
                                   (256, 8, 300), (3, 1000, 7), (200, 300, 1)])
def test_ragged_shapes_vs_fp64(M, N, K, cuda, amp_lib):
    A, B = workloads.gemm_fp32_inputs(M, N, K, seed=M * 7 + N)
    C = run_dev(A, B)
    assert np.array_equal(C, oracle.gemm_fp32_amp(A, B))
    assert oracle.max_rel_err(C, oracle.gemm_f64(A, B)) < TOL


@pytest.mark.parametrize("tile", gemm.FP32_TILES)
def test_config_1024_cube_all_tiles(tile, cuda, amp_lib):
    A, B = workloads.gemm_fp32_inputs(1024, 1024, 1024, seed=0)
    C = run_dev(A, B, tile)
    assert np.array_equal(C, oracle.gemm_fp32_amp(A, B))
    assert oracle.max_rel_err(C, oracle.gemm_f64(A, B)) < TOL


def test_amp_harness_inputs_vs_amp_cpu_reference(cuda, amp_lib):
    # AMP's own input generator (values in [-10, 9.99]) and AMP's fp32 CPU GEMM:
    # the comparison amp_verify_matmul / amp_validate_kernel make.
    A, B = oracle.amp_harness_inputs(96, 96, 96, seed=42)
    C = run_dev(A, B, (16, 16, 16))
    assert np.array_equal(C, oracle.gemm_fp32_amp(A, B))
    assert oracle.max_rel_err(C, oracle.gemm_f64(A, B)) < TOL


def test_harness_inputs_at_large_k_stay_exact_where_ffma_drifts(cuda, amp_lib):
    """At 2048^3 on AMP's [-10, 10] harness inputs the exact form still equals
    the CPU reference bit for bit; the FFMA form drifts from it (reported)."""
    A, B = oracle.amp_harness_inputs(2048, 2048, 2048, seed=42)
    ref = oracle.gemm_fp32_amp(A, B)
    C = run_dev(A, B)
    assert np.array_equal(C, ref)
    fast = gemm.matmul_fp32(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda())
    torch.cuda.synchronize()
    print("FFMA form vs AMP's CPU GEMM at 2048^3:", oracle.max_rel_err(fast.cpu().numpy(), ref))


def test_big_tile_path_large_shape(cuda, amp_lib):
    A, B = workloads.gemm_fp32_inputs(2048, 1536, 512, seed=3)
    C = run_dev(A, B)
    assert np.array_equal(C, oracle.gemm_fp32_amp(A, B))
    assert oracle.max_rel_err(C, oracle.gemm_f64(A, B)) < TOL


def test_unaligned_k_uses_scalar_loads(cuda, amp_lib):
    A, B = workloads.gemm_fp32_inputs(130, 66, 63, seed=4)
    C = run_dev(A, B)
    assert np.array_equal(C, oracle.gemm_fp32_amp(A, B))
    assert oracle.max_rel_err(C, oracle.gemm_f64(A, B)) < TOL


@pytest.mark.parametrize("M,N,K", [(1024, 1024, 1024), (2048, 1536, 512), (130, 66, 63)])
def test_ffma_form_vs_fp64(M, N, K, cuda, amp_lib):
    A, B = workloads.gemm_fp32_inputs(M, N, K, seed=11)
    C = gemm.matmul_fp32(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda())
    torch.cuda.synchronize()
    assert oracle.max_rel_err(C.cpu().numpy(), oracle.gemm_f64(A, B)) < TOL


def test_unknown_tile_is_an_error(cuda, amp_lib):
    A, B = workloads.gemm_fp32_inputs(8, 8, 8)
    with pytest.raises(AmpError, match="unknown FP32 tile cfg"):
        run_dev(A, B, (64, 64, 16))


def test_host_pointer_plugin_symbol(cuda, amp_lib):
    A, B = oracle.amp_harness_inputs(200, 150, 100, seed=5)
    C = np.zeros((200, 150), np.float32)
    call("amp_user_gemm_fp32", A.ctypes.data, B.ctypes.data, C.ctypes.data, 200, 150, 100)
    assert np.array_equal(C, oracle.gemm_fp32_amp(A, B))


@pytest.mark.skipif(not oracle.REF_VALIDATOR.exists(), reason="oracle/_ref not built")
@pytest.mark.parametrize("args", [[], ["1024", "1024", "1024"], ["512", "384", "200", "7"]])
def test_amp_validate_kernel_accepts_library(args, tmp_path, cuda, amp_lib):
    """AMP's own validator (tests/amp_validate_kernel.cpp, built unchanged from
    the reference sources) dlopens libamp_b200.so and checks it vs its CPU GEMM."""
    out = tmp_path / "dump.json"
    p = subprocess.run([str(oracle.REF_VALIDATOR), str(LIB_PATH), str(out), *args],
                       capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stdout + p.stderr
    assert "PASS" in p.stdout
    d = json.loads(out.read_text())
    assert d["tiles"][0]["max_rel_err_vs_cpu"] == 0     # bit-identical to AMP's CPU GEMM
    M = int(args[0]) if args else 96
    N = int(args[1]) if args else 96
    assert len(d["tiles"][0]["output"]) == M * N


def test_parity_dump_tool_schema_and_values(tmp_path, cuda, amp_lib):
    tool = LIB_PATH.parent / "tools" / "bin" / "amp_b200_parity_dump"
    out = tmp_path / "a.json"
    p = subprocess.run([str(tool), str(out), "96", "96", "96"], capture_output=True, text=True,
                       timeout=300)
    assert p.returncode == 0, p.stdout + p.stderr
    d = json.loads(out.read_text())
    assert (d["M"], d["N"], d["K"], d["seed"]) == (96, 96, 96, 42)
    assert [(t["bm"], t["bn"], t["bk"]) for t in d["tiles"]] == list(gemm.FP32_TILES)
    A, B = oracle.amp_harness_inputs(96, 96, 96, seed=42)
    ref = oracle.gemm_fp32_amp(A, B)
    for t in d["tiles"]:
        assert set(t) == {"bm", "bn", "bk", "gflops", "latency_ms", "max_rel_err_vs_cpu", "output"}
        # parity_check.py's rule: |a-b|/max(1,|b|) < 1e-3 (dump values carry 6 digits)
        assert oracle.max_rel_err(np.asarray(t["output"]).reshape(96, 96), ref) < TOL
        assert t["max_rel_err_vs_cpu"] == 0


@pytest.mark.parametrize("M,N,K", [(1024, 1024, 1024), (300, 200, 516), (7, 1000, 64)])
def test_3xtf32_opt_in_path(M, N, K, cuda, amp_lib):
    """The opt-in tensor-core fp32 GEMM (three TF32 products): within the 1e-3 bar
    on U[-1,1] inputs at these sizes; ragged M/N and tiles past the edges included."""
    A, B = workloads.gemm_fp32_inputs(M, N, K, seed=3)
    C = gemm.matmul_fp32_3xtf32(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda())
    torch.cuda.synchronize()
    assert oracle.max_rel_err(C.cpu().numpy(), oracle.gemm_f64(A, B)) < 5e-4


def test_3xtf32_rejects_shapes_tma_cannot_load(cuda, amp_lib):
    A = torch.zeros(8, 6, device="cuda")
    B = torch.zeros(6, 8, device="cuda")
    with pytest.raises(AmpError):
        gemm.matmul_fp32_3xtf32(A, B)


def test_staging_buffers_are_released_on_request(cuda, amp_lib):
    """The host-pointer entry points keep grow-only staging buffers; AMP's plugin
    contract frees device buffers before returning, which amp_release_staging
    (or AMP_B200_RELEASE_STAGING=1, below) provides."""
    S = 2048
    A, B = workloads.gemm_fp32_inputs(S, S, S, seed=1)
    C = np.zeros((S, S), np.float32)
    call("amp_user_gemm_fp32", A.ctypes.data, B.ctypes.data, C.ctypes.data, S, S, S)
    free_before, _ = torch.cuda.mem_get_info(cuda)
    call("amp_release_staging")
    free_after, _ = torch.cuda.mem_get_info(cuda)
    assert free_after - free_before >= 3 * S * S * 4 - (4 << 20), (free_before, free_after)
    call("amp_user_gemm_fp32", A.ctypes.data, B.ctypes.data, C.ctypes.data, S, S, S)
    assert np.array_equal(C, oracle.gemm_fp32_amp(A, B))


@pytest.mark.skipif(not oracle.REF_VALIDATOR.exists(), reason="oracle/_ref not built")
def test_amp_validate_kernel_with_per_call_release(tmp_path, cuda, amp_lib):
    import os
    out = tmp_path / "dump.json"
    p = subprocess.run([str(oracle.REF_VALIDATOR), str(LIB_PATH), str(out), "512", "512", "512"],
                       capture_output=True, text=True, timeout=600,
                       env={**os.environ, "AMP_B200_RELEASE_STAGING": "1"})
    assert p.returncode == 0 and "PASS" in p.stdout, p.stdout + p.stderr
    assert json.loads(out.read_text())["tiles"][0]["max_rel_err_vs_cpu"] == 0
