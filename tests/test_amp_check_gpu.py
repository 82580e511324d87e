"""AMP's one-command checker, scripts/amp_check.sh, on the drop-in kernel file.

oracle/_ref/libamp_check_cuda.so is the plugin library amp_check.sh itself
generated and compiled around amp_b200/dropin/amp_b200_gemm_fp32.cu (its
wrapper, its bare `nvcc -shared` command: compute_52 PTX that the driver
compiles for the B200; recipe oracle/amp_check_build.sh).  Here its last step
runs: AMP's own validator, built from the reference sources, loads that
library, calls amp_user_gemm_fp32 on its harness inputs and compares with
cpu_reference_gemm.  The kernel accumulates in the CPU reference's order and
rounding, so the bar is max_rel_err == 0, not just AMP's 1e-3.
"""
import json
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
VALIDATOR = ROOT / "oracle" / "_ref" / "amp_validate_kernel"
PLUGIN = ROOT / "oracle" / "_ref" / "libamp_check_cuda.so"

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mnk", [None, (512, 512, 512), (1024, 1024, 1024), (100, 70, 33),
                                 (257, 513, 1000), (1, 1, 1), (2048, 64, 4096)])
def test_amp_check_library_passes_amp_validator_exactly(cuda, tmp_path, mnk):
    assert VALIDATOR.exists() and PLUGIN.exists(), \
        "oracle/_ref is not built: run `make -C oracle ref` where the AMP sources are present"
    dump = tmp_path / "dump.json"
    args = [str(VALIDATOR), str(PLUGIN), str(dump)] + ([str(v) for v in mnk] if mnk else [])
    r = subprocess.run(args, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PASS" in r.stdout, r.stdout
    d = json.loads(dump.read_text())
    M, N, K = mnk or (96, 96, 96)       # the validator's default size
    assert (d["M"], d["N"], d["K"], d["seed"]) == (M, N, K, 42)
    tile = d["tiles"][0]
    assert (tile["bm"], tile["bn"], tile["bk"]) == (0, 0, 0)
    assert len(tile["output"]) == M * N
    assert tile["max_rel_err_vs_cpu"] == 0, r.stdout
