#!/bin/sh
# Regenerates the parity dump tool's own outputs on one B200 (AMP's harness
# inputs, srand(42)):
#   b200_parity_dump_96.json         fp32, M = N = K = 96, the four tile entries
#   b200_parity_dump_bf16_96.json    --op bf16, 96^3
#   b200_parity_dump_fp8_96.json     --op fp8, 96^3
#   b200_parity_dump_quant_4096.json --op quant, n = 4096
# Needs a GPU and the built tool (python -m amp_b200.build).  The gflops and
# latency_ms fields change from run to run; the outputs do not.
set -e
cd "$(dirname "$0")/../.."
T=amp_b200/tools/bin/amp_b200_parity_dump
G=tests/golden
$T $G/b200_parity_dump_96.json 96 96 96
$T $G/b200_parity_dump_bf16_96.json 96 96 96 --op bf16
$T $G/b200_parity_dump_fp8_96.json 96 96 96 --op fp8
$T $G/b200_parity_dump_quant_4096.json 4096 1 1 --op quant
