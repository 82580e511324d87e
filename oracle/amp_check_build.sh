#!/bin/bash
# Runs AMP's own one-command checker, scripts/amp_check.sh, on the drop-in
# kernel file amp_b200/dropin/amp_b200_gemm_fp32.cu and keeps what it builds:
#
#   oracle/_ref/libamp_check_cuda.so   the plugin library amp_check.sh compiled
#                                      (its generated wrapper around the kernel,
#                                      its own nvcc command line)
#   oracle/_ref/amp_check_wrapper.cu   the wrapper source it generated
#
# Test infrastructure, like the rest of oracle/: the GPU test
# (tests/test_amp_check_gpu.py) runs AMP's validator, oracle/_ref/
# amp_validate_kernel, on that library -- the last step of amp_check.sh, which
# needs a GPU.  Here the script runs on a machine that may have none, so two
# stand-ins sit in front of it on PATH and in a scratch copy of AMP's tree:
#   * `nvidia-smi` answers "present" (amp_check.sh:48 picks nvcc only when it
#     does; nvcc cross-compiles without a GPU);
#   * `nvcc` runs the real nvcc with exactly the arguments amp_check.sh gives
#     (amp_check.sh:111) and then copies the wrapper and the library out;
#   * build/amp_validate_kernel is a stub that only prints its arguments.
# The script is copied into the scratch tree so that its PROJECT_DIR (and its
# dump path) never point into the read-only AMP checkout.
set -euo pipefail
AMP_REF=${AMP_REF:-/root/reference}
HERE=$(cd "$(dirname "$0")" && pwd)
REPO=$(dirname "$HERE")
OUT="$HERE/_ref"
KERNEL="$REPO/amp_b200/dropin/amp_b200_gemm_fp32.cu"
REAL_NVCC=${NVCC:-$(command -v nvcc || echo /usr/local/cuda/bin/nvcc)}
WORK=$(mktemp -d)
trap 'rm -rf "$WORK"' EXIT
mkdir -p "$WORK/proj/scripts" "$WORK/proj/build" "$WORK/bin" "$OUT"
cp "$AMP_REF/scripts/amp_check.sh" "$WORK/proj/scripts/amp_check.sh"

cat > "$WORK/bin/nvidia-smi" <<'SH'
#!/bin/sh
exit 0
SH
cat > "$WORK/bin/nvcc" <<SH
#!/bin/bash
"$REAL_NVCC" "\$@" || exit \$?
src=""; lib=""; prev=""
for a in "\$@"; do
    case "\$a" in *.cu) src="\$a";; esac
    [ "\$prev" = "-o" ] && lib="\$a"
    prev="\$a"
done
cp "\$src" "$OUT/amp_check_wrapper.cu"
cp "\$lib" "$OUT/libamp_check_cuda.so.tmp"
mv "$OUT/libamp_check_cuda.so.tmp" "$OUT/libamp_check_cuda.so"
SH
cat > "$WORK/proj/build/amp_validate_kernel" <<'SH'
#!/bin/sh
echo "amp_validate_kernel $* (run on a GPU by tests/test_amp_check_gpu.py)"
SH
chmod +x "$WORK/bin/nvidia-smi" "$WORK/bin/nvcc" "$WORK/proj/build/amp_validate_kernel"

PATH="$WORK/bin:$PATH" bash "$WORK/proj/scripts/amp_check.sh" "$KERNEL" amp_b200_gemm_fp32 \
    512 512 512 "$WORK/dump.json" > "$WORK/amp_check.log" 2>&1 || {
    cat "$WORK/amp_check.log" >&2
    exit 1
}
grep -q "=== Validating against CPU reference" "$WORK/amp_check.log"
test -s "$OUT/libamp_check_cuda.so"
