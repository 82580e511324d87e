#!/bin/sh
# Regenerates b200_parity_dump_96.json: the parity dump tool's own output on one
# B200 (AMP's harness inputs srand(42), M = N = K = 96, the four tile entries).
# Needs a GPU and the built tool (python -m amp_b200.build).  The gflops and
# latency_ms fields change from run to run; the outputs do not.
set -e
cd "$(dirname "$0")/../.."
amp_b200/tools/bin/amp_b200_parity_dump tests/golden/b200_parity_dump_96.json 96 96 96
