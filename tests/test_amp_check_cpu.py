"""The drop-in kernel file fits AMP's scripts/amp_check.sh: the recipe
oracle/amp_check_build.sh ran the reference's own script on it, which
generated its wrapper around amp_b200_gemm_fp32 and compiled it with its own
command line into oracle/_ref/libamp_check_cuda.so.  (Validating that library
needs a GPU: tests/test_amp_check_gpu.py.)"""
import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "oracle" / "_ref"
KERNEL = ROOT / "amp_b200" / "dropin" / "amp_b200_gemm_fp32.cu"

needs_build = pytest.mark.skipif(not (REF / "libamp_check_cuda.so").exists(),
                                 reason="oracle/_ref not built (AMP sources absent)")


@needs_build
def test_amp_check_generated_and_compiled_the_wrapper():
    w = (REF / "amp_check_wrapper.cu").read_text()
    inc = re.search(r'#include "([^"]+)"', w)
    assert inc and Path(inc.group(1)).name == KERNEL.name
    assert "amp_b200_gemm_fp32<<<grid, block>>>(dA, dB, dC, M, N, K);" in w
    # the plugin symbol AMP's validator resolves with dlsym
    lib = C.CDLL(str(REF / "libamp_check_cuda.so"))
    assert hasattr(lib, "amp_user_gemm_fp32")


def test_kernel_file_compiles_for_sm_100a_without_spills(tmp_path):
    r = subprocess.run(["nvcc", "-c", "-gencode", "arch=compute_100a,code=sm_100a", "-Xptxas",
                        "-v", str(KERNEL), "-o", str(tmp_path / "k.o")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert "0 bytes spill stores" in r.stderr and "0 bytes stack frame" in r.stderr, r.stderr
    smem = int(re.search(r"(\d+) bytes smem", r.stderr).group(1))
    assert smem <= 48 * 1024          # amp_check.sh launches with no dynamic shared memory
