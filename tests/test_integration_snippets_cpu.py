"""The C++ stubs in INTEGRATION.md compile against include/amp_b200.h (and the
scheduler and collective stubs against AMP's own include/scheduler.hpp and
include/collective.hpp where the AMP sources are present, AMP_REF).
Definitions compile at file scope; statement fragments compile inside a
function, with their free variables declared at the types the entry points
take, so a stub that passes a wrong type fails here."""
import os
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
AMP_REF = Path(os.environ.get("AMP_REF", "/root/reference"))
CUDA_INC = Path("/usr/local/cuda/include")
BLOCKS = re.findall(r"```cpp\n(.*?)```", (ROOT / "INTEGRATION.md").read_text(), flags=re.S)

PRELUDE = r"""
#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <vector>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include "amp_b200.h"
%(sched)s
int world, rank, M, N, K, S, bh_per_rank, max_pages, max_pages_total, max_ctx, Hq, Hkv, D, Np;
amp_comm* comm;
void* dC;
int64_t n;
size_t ws_bytes;
cudaStream_t s;
const __nv_bfloat16* x;
float *d_amax, *d_scale, *d_lse;
void *ws, *d_out, *d_ws;
uint8_t* q;
const void *dA, *dB_r, *dQ_r, *dK_r, *dV_r, *d_q, *d_kpool, *d_vpool;
void* const* d_cs;
void* const* d_os;
float* const* d_lses;
void** d_boxes;
int32_t *d_table, *d_ctx;
unsigned next_seq();
void comm_allgather_bytes(const void* send, void* recv, size_t bytes_per_rank);
%(batch)s
"""


def compiles(code: str, tmp: Path, sched: bool) -> subprocess.CompletedProcess:
    src = tmp / "snippet.cpp"
    src.write_text(code)
    inc = ["-I", str(ROOT / "include"), "-I", str(CUDA_INC)]
    if sched:
        inc += ["-I", str(AMP_REF / "include"), "-DAMP_BACKEND_CUDA"]
    return subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-Wall", *inc, str(src)],
                          capture_output=True, text=True)


def test_there_are_stubs_to_check():
    assert len(BLOCKS) >= 5


@pytest.mark.parametrize("i", range(len(BLOCKS)))
def test_integration_stub_compiles(i, tmp_path):
    block = BLOCKS[i]
    sched = "AMP::" in block and "Batch" in block
    coll = "CommGroup" in block
    header = "scheduler.hpp" if sched else "collective.hpp" if coll else None
    if header and not (AMP_REF / "include" / header).exists():
        pytest.skip(f"AMP's {header} not present")
    prelude = PRELUDE % {"sched": f'#include "{header}"' if header else "",
                         "batch": "AMP::ScheduledBatch batch;" if sched else ""}
    sched = bool(header)
    at_file_scope = compiles(prelude + block, tmp_path, sched)
    if at_file_scope.returncode == 0:
        return
    in_function = compiles(prelude + "void stub() {\n" + block + "\n}\n", tmp_path, sched)
    assert in_function.returncode == 0, (
        f"INTEGRATION.md C++ block {i} compiles neither at file scope nor in a function:\n"
        + in_function.stderr[-3000:])
