"""The parity dump tool's extension ops on the B200 against the oracle's dumps.

amp_b200_parity_dump --op bf16 | fp8 | quant writes AMP's dump schema
(tests/parity_dump.cpp:85-107 of the reference); oracle/parity_dump.py writes
the oracle's side from the same harness fill.  Each pair must pass the rule of
AMP's scripts/parity_check.py, restated here for the GPU box, where AMP's
sources are absent: equal (M, N, K, seed), entries matched on (bm, bn, bk),
|a - b| / max(1, |b|) < 1e-3 for every output (parity_check.py:25,36-37,55-61,
84-89).  The quantiser's codes and dequantised values must be equal exactly.
(AMP's own parity_check.py runs on the committed B200 dumps of these ops in
tests/test_parity_contract_cpu.py.)
"""
import json
import subprocess

import numpy as np
import pytest

from amp_b200 import LIB_PATH
from oracle import parity_dump

pytestmark = pytest.mark.gpu
TOOL = LIB_PATH.parent / "tools" / "bin" / "amp_b200_parity_dump"
TOL = 1e-3


def parity_rule(a: dict, b: dict) -> float:
    """Worst |a - b| / max(1, |b|) over every matched entry (parity_check.py's rule)."""
    assert (a["M"], a["N"], a["K"], a["seed"]) == (b["M"], b["N"], b["K"], b["seed"])
    ta = {(t["bm"], t["bn"], t["bk"]): t for t in a["tiles"]}
    tb = {(t["bm"], t["bn"], t["bk"]): t for t in b["tiles"]}
    assert ta.keys() == tb.keys()
    worst = 0.0
    for key in ta:
        x = np.asarray(ta[key]["output"], np.float64)
        y = np.asarray(tb[key]["output"], np.float64)
        assert x.shape == y.shape, key
        worst = max(worst, float((np.abs(x - y) / np.maximum(1.0, np.abs(y))).max()))
    return worst


@pytest.mark.parametrize("op,mnk", [("bf16", (512, 512, 512)), ("fp8", (512, 512, 512)),
                                    ("bf16", (96, 160, 64)), ("fp8", (256, 128, 96)),
                                    ("quant", (65536, 1, 1)), ("quant", (4099, 1, 1))])
def test_extension_op_dump_passes_parity_rule_against_oracle(op, mnk, cuda, amp_lib, tmp_path):
    M, N, K = mnk
    a_path, b_path = tmp_path / "b200.json", tmp_path / "oracle.json"
    r = subprocess.run([str(TOOL), str(a_path), str(M), str(N), str(K), "--op", op],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    parity_dump.write_op_dump(b_path, op, M, N, K)
    a, b = json.loads(a_path.read_text()), json.loads(b_path.read_text())
    worst = parity_rule(a, b)
    if op == "quant":
        assert worst == 0.0          # codes (bm = 0) and dequantised values (bm = 1) exact
    else:
        assert worst < TOL, worst
    for t in a["tiles"]:
        assert t["max_rel_err_vs_cpu"] < (TOL if op != "quant" else 1e-12)
