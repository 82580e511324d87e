"""The NCCL collective layer of the C ABI (amp_comm_*, the reference's
include/collective.hpp ops) and the NCCL forms of the sharded GEMM and
attention, driven without torch.distributed.

* In-process, a one-rank communicator: every op and both sharded operations
  give bit-identical results to the unsharded entry points.
* The C++ host tools/bin/amp_b200_sharded forks one process per GPU, builds
  the communicator through the C ABI alone and checks the gathered result bit
  for bit against the unsharded operation on each rank: world 1 always, world
  2 where the box has two GPUs.
"""
import ctypes as C
import json
import subprocess

import pytest
import torch

from amp_b200 import LIB_PATH
from amp_b200._lib import call, lib

pytestmark = pytest.mark.gpu

F32, BF16, I32, MAX, SUM = 0, 1, 3, 1, 0
TOOL = LIB_PATH.parent / "tools" / "bin" / "amp_b200_sharded"


@pytest.fixture
def comm1(cuda, amp_lib):
    uid = (C.c_ubyte * 128)()
    call("amp_comm_unique_id", uid)
    comm = C.c_void_p()
    call("amp_comm_init_rank", C.byref(comm), 0, 1, cuda.index or 0, uid)
    yield comm
    torch.cuda.synchronize(cuda)
    call("amp_comm_destroy", comm)


def _s(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def test_one_rank_collectives(comm1, cuda):
    r, w, d = C.c_int(), C.c_int(), C.c_int()
    call("amp_comm_rank", comm1, C.byref(r), C.byref(w), C.byref(d))
    assert (r.value, w.value, d.value) == (0, 1, cuda.index or 0)
    x = torch.randn(1000, device=cuda)
    y = x.clone()
    call("amp_comm_allreduce_max_f32", comm1, y.data_ptr(), y.numel(), _s(cuda))
    i = torch.arange(77, dtype=torch.int32, device=cuda)
    call("amp_comm_allreduce", comm1, i.data_ptr(), i.numel(), I32, SUM, _s(cuda))
    g = torch.empty_like(x)
    call("amp_comm_allgather", comm1, x.data_ptr(), g.data_ptr(), x.numel(), F32, _s(cuda))
    b = x.to(torch.bfloat16)
    b0 = b.clone()
    call("amp_comm_broadcast", comm1, b.data_ptr(), b.numel(), BF16, 0, _s(cuda))
    call("amp_comm_barrier", comm1, _s(cuda))
    torch.cuda.synchronize(cuda)
    assert torch.equal(y, x) and torch.equal(g, x) and torch.equal(b, b0)
    assert torch.equal(i, torch.arange(77, dtype=torch.int32, device=cuda))


@pytest.mark.parametrize("fp8", [False, True])
def test_one_rank_sharded_gemm_equals_plain(comm1, cuda, fp8):
    M, N, K = 512, 768, 320
    a = torch.randn(M, K, device=cuda)
    bm = torch.randn(K, N, device=cuda)
    if fp8:
        A = a.to(torch.float8_e4m3fn).view(torch.uint8)
        B = bm.to(torch.float8_e4m3fn).view(torch.uint8)
        sa = torch.rand(M, device=cuda) + 0.5
        sb = torch.rand(N, device=cuda) + 0.5
    else:
        A, B = a.to(torch.bfloat16), bm.to(torch.bfloat16)
    C_sh = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    C_ref = torch.empty_like(C_sh)
    ws_bytes = lib().amp_gemm_sharded_workspace_bytes(M, N, 1, BF16)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda)
    if fp8:
        call("amp_gemm_fp8e4m3_sharded_dev", comm1, A.data_ptr(), B.data_ptr(), sa.data_ptr(),
             sb.data_ptr(), 2, C_sh.data_ptr(), BF16, M, N, K, ws.data_ptr(), ws_bytes, _s(cuda))
        call("amp_gemm_fp8e4m3_dev", A.data_ptr(), B.data_ptr(), sa.data_ptr(), sb.data_ptr(), 2,
             C_ref.data_ptr(), BF16, M, N, K, _s(cuda))
    else:
        call("amp_gemm_bf16_sharded_dev", comm1, A.data_ptr(), B.data_ptr(), C_sh.data_ptr(), BF16,
             M, N, K, ws.data_ptr(), ws_bytes, _s(cuda))
        call("amp_gemm_bf16_dev", A.data_ptr(), B.data_ptr(), C_ref.data_ptr(), BF16, M, N, K,
             _s(cuda))
    torch.cuda.synchronize(cuda)
    assert torch.equal(C_sh.view(torch.int16), C_ref.view(torch.int16))


@pytest.mark.parametrize("hq,hkv", [(8, 8), (8, 2)])
def test_one_rank_sharded_attention_equals_plain(comm1, cuda, hq, hkv):
    B, S, D = 2, 384, 128
    q = torch.randn(B, hq, S, D, device=cuda).to(torch.bfloat16)
    k = torch.randn(B, hkv, S, D, device=cuda).to(torch.bfloat16)
    v = torch.randn(B, hkv, S, D, device=cuda).to(torch.bfloat16)
    o1, o2 = torch.empty_like(q), torch.empty_like(q)
    l1 = torch.empty(B, hq, S, device=cuda)
    l2 = torch.empty_like(l1)
    call("amp_flash_attn_fwd_sharded_dev", comm1, q.data_ptr(), k.data_ptr(), v.data_ptr(),
         o1.data_ptr(), l1.data_ptr(), B, hq, hkv, S, S, D, 1, 0.0, _s(cuda))
    call("amp_flash_attn_fwd_bf16_dev", q.data_ptr(), k.data_ptr(), v.data_ptr(), o2.data_ptr(),
         l2.data_ptr(), B, hq, hkv, S, S, D, 1, 0.0, _s(cuda))
    torch.cuda.synchronize(cuda)
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16)) and torch.equal(l1, l2)


def _run_tool(world, op, mnk=("1024", "2048", "512")):
    r = subprocess.run([str(TOOL), str(world), *mnk, "--op", op], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = [json.loads(x) for x in r.stdout.splitlines() if x.startswith("{")]
    assert sorted(x["rank"] for x in lines) == list(range(world)), r.stdout
    assert all(x["mismatched_bytes"] == 0 and x["max_over_ranks"] == 0 for x in lines), r.stdout


@pytest.mark.parametrize("op", ["bf16", "fp8", "attn", "attn_gqa"])
def test_cpp_host_one_rank(cuda, amp_lib, op):
    _run_tool(1, op)


@pytest.mark.multigpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("op", ["bf16", "fp8", "attn", "attn_gqa"])
def test_cpp_host_two_ranks_bit_identical_to_one_gpu(cuda, amp_lib, op):
    _run_tool(2, op)
