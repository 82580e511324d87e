"""The dump contract.  golden/b200_parity_dump_96.json is the parity dump tool's
own output on a B200 (golden/make_b200_dump.sh).  write_dump below reproduces
that file byte for byte from its values (parity_dump.cpp's write_json: keys, key
order, 6-significant-digit stream formatting), so dumps written here are dumps
as the tool writes them.  AMP's own scripts/parity_check.py (where the AMP
sources are present, AMP_REF) passes the B200 dump against the oracle's, passes
identical outputs, fails a perturbed one and refuses another shape/seed; AMP's
synthetic FAIL fixtures fail the same way.  (write_dump: oracle/parity_dump.py.)"""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from amp_b200.gemm import FP32_TILES
from oracle.parity_dump import write_dump

AMP_REF = Path(os.environ.get("AMP_REF", "/root/reference"))
PARITY = AMP_REF / "scripts" / "parity_check.py"
needs_amp = pytest.mark.skipif(not PARITY.exists(), reason="AMP's parity_check.py not present")
B200_DUMP = Path(__file__).resolve().parent / "golden" / "b200_parity_dump_96.json"


def parity(a, b):
    return subprocess.run([sys.executable, str(PARITY), str(a), str(b)], capture_output=True,
                          text=True, timeout=120)


@pytest.fixture(scope="module")
def harness_c(oracle_lib):
    A, B = oracle_lib.amp_harness_inputs(96, 96, 96, 42)
    return oracle_lib.gemm_fp32_amp(A, B).astype(np.float32)


def entries(C):
    return [(bm, bn, bk, 1234.5, 0.0123, 0.0, C.ravel()) for (bm, bn, bk) in FP32_TILES]


@needs_amp
def test_identical_outputs_pass(tmp_path, harness_c):
    write_dump(tmp_path / "a.json", "nvidia", 96, 96, 96, 42, entries(harness_c))
    write_dump(tmp_path / "b.json", "cpu-oracle", 96, 96, 96, 42, entries(harness_c))
    r = parity(tmp_path / "a.json", tmp_path / "b.json")
    assert r.returncode == 0, r.stdout + r.stderr
    assert "FAIL" not in r.stdout


@needs_amp
def test_one_perturbed_element_fails(tmp_path, harness_c):
    bad = harness_c.copy()
    bad[5, 7] += np.float32(2e-3) * max(1.0, abs(float(bad[5, 7])))
    write_dump(tmp_path / "a.json", "nvidia", 96, 96, 96, 42, entries(bad))
    write_dump(tmp_path / "b.json", "cpu-oracle", 96, 96, 96, 42, entries(harness_c))
    r = parity(tmp_path / "a.json", tmp_path / "b.json")
    assert r.returncode == 1 and "FAIL" in r.stdout, r.stdout


@needs_amp
def test_other_seed_is_not_comparable(tmp_path, harness_c):
    write_dump(tmp_path / "a.json", "nvidia", 96, 96, 96, 42, entries(harness_c))
    write_dump(tmp_path / "b.json", "cpu-oracle", 96, 96, 96, 43, entries(harness_c))
    r = parity(tmp_path / "a.json", tmp_path / "b.json")
    assert r.returncode == 1 and "not comparable" in r.stdout


@needs_amp
def test_amp_synthetic_fail_fixtures_fail():
    fx = AMP_REF / "tests" / "fixtures"
    r = parity(fx / "synthetic_fail_a.json", fx / "synthetic_fail_b.json")
    assert r.returncode == 1 and "FAIL" in r.stdout


def _tiles(d):
    return [(t["bm"], t["bn"], t["bk"], t["gflops"], t["latency_ms"], t["max_rel_err_vs_cpu"],
             t["output"]) for t in d["tiles"]]


def test_writer_mirror_reproduces_the_b200_dump_byte_for_byte(tmp_path):
    import json
    d = json.loads(B200_DUMP.read_text())
    write_dump(tmp_path / "again.json", d["vendor"], d["M"], d["N"], d["K"], d["seed"], _tiles(d))
    assert (tmp_path / "again.json").read_text() == B200_DUMP.read_text()


def test_b200_dump_is_within_the_bar_of_the_oracle(harness_c):
    import json
    import oracle
    d = json.loads(B200_DUMP.read_text())
    assert (d["M"], d["N"], d["K"], d["seed"]) == (96, 96, 96, 42)
    assert [(t["bm"], t["bn"], t["bk"]) for t in d["tiles"]] == list(FP32_TILES)
    for t in d["tiles"]:
        got = np.asarray(t["output"], np.float64).reshape(96, 96)
        assert oracle.max_rel_err(got, harness_c) < 1e-3
        assert t["max_rel_err_vs_cpu"] < 1e-3


@needs_amp
def test_b200_dump_passes_amp_parity_check_against_the_oracle(tmp_path, harness_c):
    write_dump(tmp_path / "oracle.json", "cpu-oracle", 96, 96, 96, 42, entries(harness_c))
    r = parity(B200_DUMP, tmp_path / "oracle.json")
    assert r.returncode == 0, r.stdout + r.stderr
    assert "FAIL" not in r.stdout


EXT_DUMPS = {"bf16": ("b200_parity_dump_bf16_96.json", (96, 96, 96)),
             "fp8": ("b200_parity_dump_fp8_96.json", (96, 96, 96)),
             "quant": ("b200_parity_dump_quant_4096.json", (4096, 1, 1))}


@pytest.mark.parametrize("op", sorted(EXT_DUMPS))
def test_b200_extension_dumps_are_the_tools_layout(op, tmp_path):
    import json
    path = B200_DUMP.parent / EXT_DUMPS[op][0]
    d = json.loads(path.read_text())
    write_dump(tmp_path / "again.json", d["vendor"], d["M"], d["N"], d["K"], d["seed"], _tiles(d))
    assert (tmp_path / "again.json").read_text() == path.read_text()


@needs_amp
@pytest.mark.parametrize("op", sorted(EXT_DUMPS))
def test_b200_extension_dumps_pass_amp_parity_check_against_the_oracle(op, tmp_path, oracle_lib):
    """The bf16 / FP8 GEMM and quantiser dumps the tool wrote on a B200
    (golden/make_b200_dump.sh) against the oracle's dumps of the same op, through
    AMP's parity_check.py unchanged."""
    from oracle.parity_dump import write_op_dump
    name, (M, N, K) = EXT_DUMPS[op]
    write_op_dump(tmp_path / "oracle.json", op, M, N, K)
    r = parity(B200_DUMP.parent / name, tmp_path / "oracle.json")
    assert r.returncode == 0, r.stdout + r.stderr
    assert "FAIL" not in r.stdout
