"""Generate the golden fixtures under tests/golden/ from the REFERENCE itself.

Run in a checkout where the AMP sources are available (default
/root/reference, override with AMP_REF):

    make -C oracle ref && python tests/golden/make_golden.py

Writes:
  fp8_e4m3_ref_codec.json -- AMP's own host codec (include/fp8.hpp:15-63,
      compiled from the reference sources into oracle/_ref/libampref.so)
      evaluated on: the probes of tests/verify_fixes.cpp:29-46, every E4M3
      decode, every positive E4M3 midpoint and a seeded sample of the
      quantiser's input distribution.  torch's float8_e4m3fn (a third-party
      round-to-nearest-even implementation) is recorded beside it.
  amp_harness_gemm.json -- AMP's own validator (tests/amp_validate_kernel.cpp,
      built into oracle/_ref/amp_validate_kernel) run on a CPU plugin that
      computes with the oracle's restatement of cpu_reference_gemm; records
      the validator's verdict and a digest of the dumped output.
"""
from __future__ import annotations

import ctypes as C
import hashlib
import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
import oracle  # noqa: E402

OUT = Path(__file__).resolve().parent
AMP_REF = Path(os.environ.get("AMP_REF", "/root/reference"))

VERIFY_FIXES_PROBES = [256.0, 260.0, 288.0, 300.0, 320.0, 350.0, 384.0, 400.0, 416.0, 440.0, 448.0]


def torch_rne(x: np.ndarray) -> list[int]:
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x, np.float32))
    return t.to(torch.float8_e4m3fn).view(torch.uint8).numpy().astype(int).tolist()


def fp8_fixture() -> dict:
    r = oracle.ref_lib()
    if r is None:
        raise SystemExit("oracle/_ref/libampref.so missing: run `make -C oracle ref` first")
    dec = [r.ref_e4m3_to_f32(i) for i in range(256)]
    # positive finite E4M3 values in increasing order and their midpoints
    pos = sorted({v for v in dec if np.isfinite(v) and v > 0})
    mids = [(a + b) / 2 for a, b in zip(pos[:-1], pos[1:])]
    rng = np.random.default_rng(20240601)
    sample = rng.standard_normal(4096).astype(np.float32) * np.float32(448.0 / 4.5)
    sample[::97] *= 50
    edges = [0.0, -0.0, 2.0 ** -10, 2.0 ** -9, 1.5 * 2 ** -9, 7.5 * 2 ** -9, 2.0 ** -6,
             447.0, 448.0, 455.0, 464.0, 465.0, 1e6]

    def enc(vals):
        a = np.asarray(vals, np.float32)
        return [int(r.ref_f32_to_e4m3(float(v))) for v in a], a

    codes_probe, _ = enc(VERIFY_FIXES_PROBES)
    codes_mid, a_mid = enc(mids)
    codes_edge, a_edge = enc(edges)
    codes_sample, _ = enc(sample)
    return {
        "generator": "tests/golden/make_golden.py",
        "reference_codec": "include/fp8.hpp:15-63 compiled via oracle/ref_amp_shim.cpp",
        "decode": [None if not np.isfinite(v) else float(v) for v in dec],
        "verify_fixes_probes": {"x": VERIFY_FIXES_PROBES, "amp": codes_probe,
                                "torch_rne": torch_rne(np.array(VERIFY_FIXES_PROBES))},
        "midpoints": {"x": [float(v) for v in a_mid], "amp": codes_mid,
                      "torch_rne": torch_rne(a_mid)},
        "edges": {"x": [float(v) for v in a_edge], "amp": codes_edge},
        "sample": {"x_f32_hex": [format(int(u), "08x") for u in sample.view(np.uint32)],
                   "amp": codes_sample, "torch_rne": torch_rne(sample)},
    }


CPU_PLUGIN_SRC = r"""
#include <stdlib.h>
typedef void (*gemm_fn)(const float*, const float*, float*, int, int, int);
static gemm_fn g;
#include <dlfcn.h>
int amp_user_gemm_fp32(const float* A, const float* B, float* C, int M, int N, int K) {
    if (!g) {
        void* h = dlopen(getenv("ORACLE_LIB"), RTLD_NOW);
        if (!h) return 2;
        g = (gemm_fn)dlsym(h, "orc_gemm_fp32_amp");
        if (!g) return 3;
    }
    g(A, B, C, M, N, K);
    return 0;
}
"""


def harness_fixture() -> dict:
    validator = oracle.REF_VALIDATOR
    if not validator.exists():
        raise SystemExit("oracle/_ref/amp_validate_kernel missing: run `make -C oracle ref`")
    cases = []
    with tempfile.TemporaryDirectory() as td:
        src = Path(td) / "cpu_plugin.c"
        so = Path(td) / "libcpu_plugin.so"
        src.write_text(CPU_PLUGIN_SRC)
        subprocess.run(["gcc", "-O2", "-fPIC", "-shared", "-o", str(so), str(src), "-ldl"],
                       check=True)
        env = dict(os.environ, ORACLE_LIB=str(oracle.LIB))
        for (M, N, K, seed) in [(96, 96, 96, 42), (64, 48, 80, 7), (33, 17, 5, 3)]:
            dump = Path(td) / "dump.json"
            p = subprocess.run([str(validator), str(so), str(dump), str(M), str(N), str(K),
                                str(seed)], capture_output=True, text=True, env=env)
            d = json.loads(dump.read_text())
            out = np.asarray(d["tiles"][0]["output"], np.float64)
            A, B = oracle.amp_harness_inputs(M, N, K, seed)
            mine = oracle.gemm_fp32_amp(A, B)
            cases.append({
                "M": M, "N": N, "K": K, "seed": seed,
                "validator_exit": p.returncode,
                "validator_max_rel_err": d["tiles"][0]["max_rel_err_vs_cpu"],
                "dump_keys": sorted(d.keys()),
                "tile_keys": sorted(d["tiles"][0].keys()),
                "output_first8": out[:8].tolist(),
                "output_sum": float(out.sum()),
                "oracle_sum": float(mine.astype(np.float64).sum()),
                "oracle_sha256": hashlib.sha256(mine.tobytes()).hexdigest(),
                "inputs_sha256": hashlib.sha256(A.tobytes() + B.tobytes()).hexdigest(),
            })
    return {"generator": "tests/golden/make_golden.py",
            "validator": "tests/amp_validate_kernel.cpp built as oracle/_ref/amp_validate_kernel",
            "cases": cases}


def main() -> None:
    oracle.build(ref=True)
    (OUT / "fp8_e4m3_ref_codec.json").write_text(json.dumps(fp8_fixture(), indent=1) + "\n")
    (OUT / "amp_harness_gemm.json").write_text(json.dumps(harness_fixture(), indent=1) + "\n")
    print("wrote", OUT / "fp8_e4m3_ref_codec.json", OUT / "amp_harness_gemm.json")


if __name__ == "__main__":
    main()
