"""The extension ops of the parity dump tool (--op bf16 | fp8 | quant), on CPU.

* The tool's host arithmetic -- bf16 rounding, E4M3 decode and round-to-nearest-
  even saturating encode, and the per-tensor quantiser it uses for its
  max_rel_err_vs_cpu field -- compiled from amp_b200/tools/parity_dump.cpp
  itself, agrees bit for bit with the oracle.
* The oracle's side of each op's dump (oracle/parity_dump.py) is deterministic,
  passes AMP's parity_check.py against itself and agrees with an independent
  torch computation.
The tool's device side runs in the GPU test of the dump tool."""
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from oracle import parity_dump

ROOT = Path(__file__).resolve().parents[1]
AMP_REF = Path(os.environ.get("AMP_REF", "/root/reference"))
PARITY = AMP_REF / "scripts" / "parity_check.py"

DRIVER = r"""
#define main parity_dump_main
#include "parity_dump.cpp"
#undef main
#include <cstdio>
#include <string>
#include <vector>
static std::vector<char> slurp(const char* p) {
    std::vector<char> b;
    FILE* f = std::fopen(p, "rb");
    if (!f) return b;
    char buf[65536];
    size_t n;
    while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) b.insert(b.end(), buf, buf + n);
    std::fclose(f);
    return b;
}
static void spit(const char* p, const void* d, size_t n) {
    FILE* f = std::fopen(p, "wb");
    std::fwrite(d, 1, n, f);
    std::fclose(f);
}
int main(int argc, char** argv) {
    if (argc < 4) return 2;
    const std::string mode = argv[1];
    const std::vector<char> in = slurp(argv[2]);
    if (mode == "code" || mode == "bf16") {
        const size_t n = in.size() / 4;
        const float* x = reinterpret_cast<const float*>(in.data());
        if (mode == "code") {
            std::vector<uint8_t> q(n);
            for (size_t i = 0; i < n; ++i) q[i] = e4m3_code(x[i]);
            spit(argv[3], q.data(), n);
        } else {
            std::vector<uint16_t> h(n);
            for (size_t i = 0; i < n; ++i) h[i] = bf16_rne(x[i]);
            spit(argv[3], h.data(), 2 * n);
        }
    } else if (mode == "value") {
        std::vector<float> v(256);
        for (int c = 0; c < 256; ++c) v[c] = e4m3_value((uint8_t)c);
        spit(argv[3], v.data(), 4 * 256);
    } else if (mode == "quant") {
        std::vector<uint16_t> x(in.size() / 2);
        std::memcpy(x.data(), in.data(), in.size());
        const Quantised q = quantise_host(x);
        std::vector<char> out(q.q.begin(), q.q.end());
        out.insert(out.end(), reinterpret_cast<const char*>(&q.scale),
                   reinterpret_cast<const char*>(&q.scale) + 4);
        spit(argv[3], out.data(), out.size());
    } else {
        return 2;
    }
    return 0;
}
"""


@pytest.fixture(scope="module")
def driver(tmp_path_factory, amp_lib):
    from amp_b200.build import ARCH, PKG, nvcc
    d = tmp_path_factory.mktemp("tool_driver")
    src = d / "driver.cpp"
    src.write_text(DRIVER)
    exe = d / "driver"
    r = subprocess.run([nvcc(), "-O2", "-std=c++17", "-x", "cu", *ARCH,
                        "-I", str(ROOT / "include"), "-I", str(ROOT / "amp_b200" / "tools"),
                        str(src), "-o", str(exe), "-L", str(PKG), "-lamp_b200",
                        "-Xlinker", f"-rpath={PKG}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]

    def run(mode, data: np.ndarray, dtype):
        i, o = d / "in.bin", d / "out.bin"
        i.write_bytes(np.ascontiguousarray(data).tobytes())
        p = subprocess.run([str(exe), mode, str(i), str(o)], capture_output=True, text=True)
        assert p.returncode == 0, p.stderr
        return np.frombuffer(o.read_bytes(), dtype)
    return run


def probe_floats(oracle_lib) -> np.ndarray:
    dec = oracle_lib.e4m3_decode_table()
    fin = np.sort(np.unique(dec[np.isfinite(dec) & (dec >= 0)]))
    mids = (fin[:-1] + fin[1:]) / 2                       # every tie
    rng = np.random.default_rng(11)
    wide = rng.standard_normal(200_000).astype(np.float32) * np.exp2(
        rng.integers(-14, 12, 200_000)).astype(np.float32)
    edges = np.array([0.0, -0.0, 448, 449, 463.9, 464, 465, 1e30, np.inf, -np.inf, np.nan,
                      2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -10, 2.0 ** -6, 7.5 * 2.0 ** -9,
                      1e-30], np.float32)
    x = np.concatenate([fin, -fin, mids, -mids, np.nextafter(mids, 0), np.nextafter(mids, 1e9),
                        wide, edges]).astype(np.float32)
    return x


def test_tool_e4m3_encode_matches_the_oracle(driver, oracle_lib):
    x = probe_floats(oracle_lib)
    got = driver("code", x, np.uint8)
    assert np.array_equal(got, oracle_lib.e4m3_encode(x))


def test_tool_e4m3_decode_matches_the_oracle(driver, oracle_lib):
    got = driver("value", np.zeros(1, np.float32), np.float32)
    want = oracle_lib.e4m3_decode_table()
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(got[~np.isnan(want)], want[~np.isnan(want)])


def test_tool_bf16_rounding_matches_the_oracle(driver, oracle_lib):
    rng = np.random.default_rng(5)
    bits = rng.integers(0, 2 ** 32, 300_000, dtype=np.uint64).astype(np.uint32)
    bits[:4] = [0x7F800000, 0xFF800000, 0x7FC00001, 0x3F808000]     # inf, -inf, nan, tie
    x = bits.view(np.float32)
    assert np.array_equal(driver("bf16", x, np.uint16), oracle_lib.f32_to_bf16_bits(x))


@pytest.mark.parametrize("case", ["workload", "harness", "zeros", "nan_inside", "tiny"])
def test_tool_quantiser_matches_the_oracle(case, driver, oracle_lib):
    from amp_b200 import workloads
    if case == "workload":
        x16 = workloads.quant_input_numpy(1 << 16, seed=3)
    elif case == "harness":
        a, _ = oracle_lib.amp_harness_inputs(5000, 1, 1, 42)
        x16 = oracle_lib.f32_to_bf16_bits(a.ravel())
    elif case == "zeros":
        x16 = np.zeros(100, np.uint16)
    elif case == "nan_inside":
        x16 = oracle_lib.f32_to_bf16_bits(np.array([1.0, np.nan, -300.0, 2e-3], np.float32))
    else:
        x16 = oracle_lib.f32_to_bf16_bits(np.array([1e-38, -3e-39, 5e-40], np.float32))
    out = driver("quant", x16.astype(np.uint16), np.uint8)
    q, scale = out[:-4], np.frombuffer(out[-4:].tobytes(), np.float32)[0]
    q_ref, s_ref, _ = oracle_lib.quant_e4m3(x16)
    assert scale == np.float32(s_ref)
    assert np.array_equal(q, q_ref)


@pytest.mark.parametrize("op,dims", [("bf16", (96, 64, 48)), ("fp8", (64, 96, 32)),
                                     ("quant", (3000, 1, 1))])
def test_oracle_dump_is_deterministic_and_matches_torch(op, dims, tmp_path, oracle_lib):
    M, N, K = dims
    a, b = tmp_path / "a.json", tmp_path / "b.json"
    parity_dump.write_op_dump(a, op, M, N, K, seed=42)
    parity_dump.write_op_dump(b, op, M, N, K, seed=42)
    assert a.read_text() == b.read_text()
    d = json.loads(a.read_text())
    if op == "quant":
        assert (d["M"], d["N"], d["K"]) == (M, 1, 1)
        assert [t["bm"] for t in d["tiles"]] == [0, 1]
        x, _ = oracle_lib.amp_harness_inputs(M, 1, 1, 42)
        xt = torch.from_numpy(x.ravel()).to(torch.bfloat16).float()
        scale = np.float32(xt.abs().max().item()) / np.float32(448)
        inv = np.float32(1) / scale
        codes = (xt * float(inv)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
        assert np.array_equal(np.asarray(d["tiles"][0]["output"], np.uint8), codes)
        return
    A, B = oracle_lib.amp_harness_inputs(M, N, K, 42)
    At = torch.from_numpy(A).to(torch.bfloat16).double()
    Bt = torch.from_numpy(B).to(torch.bfloat16).double()
    if op == "bf16":
        want = (At @ Bt).numpy()
    else:
        def q(t):
            s = np.float32(t.abs().max().item()) / np.float32(448)
            codes = (t.float() * float(np.float32(1) / s)).to(torch.float8_e4m3fn)
            return codes.double(), float(s)
        qa, sa = q(At)
        qb, sb = q(Bt)
        want = (qa @ qb).numpy() * (sa * sb)
    got = np.asarray(d["tiles"][0]["output"], np.float64).reshape(M, N)
    assert oracle.max_rel_err(got, want) < 1e-5


@pytest.mark.skipif(not PARITY.exists(), reason="AMP's parity_check.py not present")
@pytest.mark.parametrize("op", ["bf16", "fp8", "quant"])
def test_oracle_dumps_pass_amp_parity_check(op, tmp_path):
    dims = (3000, 1, 1) if op == "quant" else (64, 64, 32)
    parity_dump.write_op_dump(tmp_path / "a.json", op, *dims, vendor="nvidia")
    parity_dump.main([str(tmp_path / "b.json"), *map(str, dims), "--op", op])
    r = subprocess.run([sys.executable, str(PARITY), str(tmp_path / "a.json"),
                        str(tmp_path / "b.json")], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
