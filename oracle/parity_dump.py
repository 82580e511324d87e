"""CPU-oracle side of the parity dumps -- TEST INFRASTRUCTURE ONLY (the checker).

For the extension ops of amp_b200/tools/parity_dump.cpp (``--op bf16 | fp8 |
quant``) this writes the dump that AMP's scripts/parity_check.py compares with
the tool's, unchanged: the same header (M, N, K, seed), the same entries (bm, bn,
bk), outputs computed by the oracle from the same inputs -- the harness fill of
tests/amp_validate_kernel.cpp:84-86 (srand(seed), (rand() % 2000 - 1000) / 100),
rounded to bf16:
  bf16   C = A B in fp64 of the bf16 operands
  fp8    A and B quantised per tensor by the oracle's quantiser, C = sa sb (A8 B8)
         in fp64 of the decoded codes
  quant  n = M values: entry bm = 0 the E4M3 codes, bm = 1 the dequantised values

    python -m oracle.parity_dump --op bf16 out.json M N K [--seed S] [--vendor TAG]
"""
from __future__ import annotations

import argparse
from pathlib import Path

import numpy as np

from . import (amp_harness_inputs, bf16_bits_to_f32, dequant_e4m3, e4m3_decode_table,
               f32_to_bf16_bits, gemm_f64, quant_e4m3)


def write_dump(path, vendor: str, M: int, N: int, K: int, seed: int, entries) -> None:
    """The dump file exactly as parity_dump.cpp's write_json lays it out: keys, key
    order, one line per entry, floats as std::ostream prints them (%g).  entries:
    (bm, bn, bk, gflops, latency_ms, max_rel_err_vs_cpu, output values)."""
    g = lambda v: "%g" % v
    lines = ["{", f'  "vendor": "{vendor}",', f'  "M": {M}, "N": {N}, "K": {K}, "seed": {seed},',
             '  "tiles": [']
    for i, (bm, bn, bk, gflops, ms, err, out) in enumerate(entries):
        body = ",".join(g(v) for v in out)
        lines.append(f'    {{"bm": {bm}, "bn": {bn}, "bk": {bk}, "gflops": {g(gflops)}, '
                     f'"latency_ms": {g(ms)}, "max_rel_err_vs_cpu": {g(err)}, "output": [{body}]}}'
                     + ("," if i + 1 != len(entries) else ""))
    lines += ["  ]", "}"]
    Path(path).write_text("\n".join(lines) + "\n")


def op_outputs(op: str, M: int, N: int, K: int, seed: int):
    """(header M, N, K, [(bm, output values)]) of one extension op."""
    if op == "quant":
        x, _ = amp_harness_inputs(M, 1, 1, seed)          # the first M values of the fill
        x16 = f32_to_bf16_bits(x.ravel())
        q, s, _ = quant_e4m3(x16)
        y = bf16_bits_to_f32(dequant_e4m3(q, s))
        return (M, 1, 1), [(0, q.astype(np.float64)), (1, y.astype(np.float64))]
    A, B = amp_harness_inputs(M, N, K, seed)
    a16, b16 = f32_to_bf16_bits(A), f32_to_bf16_bits(B)
    if op == "bf16":
        C = gemm_f64(bf16_bits_to_f32(a16), bf16_bits_to_f32(b16))
    elif op == "fp8":
        dec = e4m3_decode_table().astype(np.float64)
        qa, sa, _ = quant_e4m3(a16)
        qb, sb, _ = quant_e4m3(b16)
        C = (dec[qa] @ dec[qb]) * (np.float64(sa) * np.float64(sb))
    else:
        raise ValueError(f"unknown op {op!r} (bf16, fp8, quant)")
    return (M, N, K), [(0, C.astype(np.float32).ravel())]


def write_op_dump(path, op: str, M: int, N: int, K: int, seed: int = 42,
                  vendor: str = "cpu-oracle") -> None:
    (m, n, k), outs = op_outputs(op, M, N, K, seed)
    write_dump(path, vendor, m, n, k, seed, [(bm, 0, 0, 0.0, 0.0, 0.0, out) for bm, out in outs])


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("out")
    ap.add_argument("M", type=int)
    ap.add_argument("N", type=int)
    ap.add_argument("K", type=int)
    ap.add_argument("--op", required=True, choices=["bf16", "fp8", "quant"])
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--vendor", default="cpu-oracle")
    a = ap.parse_args(argv)
    write_op_dump(a.out, a.op, a.M, a.N, a.K, a.seed, a.vendor)


if __name__ == "__main__":
    main()
