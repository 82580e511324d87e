"""Sharded kernels over NCCL on 2 GPUs vs the unsharded single-GPU result.

Skipped on boxes with fewer than two GPUs.  Each rank is a separate process
(one process per GPU), NVLS off, short process-group timeout.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from amp_b200 import fp8, sharded, workloads, gemm, attention
        dev = torch.device("cuda", rank)
        # quantise: shard of a global tensor, global amax
        full = workloads.quant_input_numpy(1 << 20, seed=3)
        n = full.size // world
        x_full = torch.from_numpy(full.view(np.int16).copy()).to(dev).view(torch.bfloat16)
        q_shard, s_shard = sharded.quantize_e4m3_sharded(x_full[rank * n:(rank + 1) * n])
        q_ref, s_ref = fp8.quantize_e4m3(x_full)
        assert torch.equal(q_shard, q_ref[rank * n:(rank + 1) * n]) and s_shard.item() == s_ref.item()
        # the same through the peer mailboxes (NVLink stores instead of NCCL); several
        # calls so both parity rows of the mailboxes are used and reused
        from amp_b200._lib import call, lib
        from amp_b200.collective import CommGroup, PeerMailboxes
        mb = PeerMailboxes(CommGroup.current())
        try:
            for _ in range(5):
                q_p, s_p = sharded.quantize_e4m3_sharded(x_full[rank * n:(rank + 1) * n],
                                                         mailboxes=mb)
                assert torch.equal(q_p, q_ref[rank * n:(rank + 1) * n])
                assert s_p.item() == s_ref.item()
            v = torch.tensor([rank + 1.5], dtype=torch.float32, device=dev)
            m = torch.empty(1, dtype=torch.float32, device=dev)
            for _ in range(3):
                call("amp_peer_allreduce_max_f32", v.data_ptr(), m.data_ptr(),
                     mb.table.data_ptr(), rank, world, mb.next_seq(), None)
                torch.cuda.synchronize()
                assert m.item() == world + 0.5
            assert lib().amp_device_status(1) == 0
        finally:
            mb.close()
        # N-split GEMM + gather
        g = torch.Generator(device=dev).manual_seed(5)
        A = torch.randn(512, 256, generator=g, device=dev).to(torch.bfloat16)
        B = torch.randn(256, 1024, generator=g, device=dev).to(torch.bfloat16)
        w = 1024 // world
        C = sharded.matmul_bf16_sharded(A, B[:, rank * w:(rank + 1) * w].contiguous())
        C_ref = torch.empty(512, 1024, dtype=torch.bfloat16, device=dev)
        gemm.launch_matmul_bf16(A, B, C_ref, 512, 1024, 256)
        assert torch.equal(C, C_ref)
        # the same with the all-gather fused into the GEMM epilogue (stores into every
        # rank's C over NVLink); a barrier between calls, so nobody still reads C
        from amp_b200.collective import PeerBuffer
        pb = PeerBuffer(CommGroup.current(), 512, 1024, torch.bfloat16)
        try:
            for _ in range(3):
                Cf = sharded.matmul_allgather(A, B[:, rank * w:(rank + 1) * w].contiguous(), pb)
                torch.cuda.synchronize()
                assert torch.equal(Cf, C_ref)
                dist.barrier()
            # FP8 operands, per-row / per-column scales, into the same buffer
            a8 = (A.float() / 4).to(torch.float8_e4m3fn).view(torch.uint8).contiguous()
            b8 = (B.float() / 4).to(torch.float8_e4m3fn).view(torch.uint8).contiguous()
            sa = torch.rand(512, generator=g, device=dev) + 0.5
            sb = torch.rand(1024, generator=g, device=dev) + 0.5
            C8_ref = torch.empty(512, 1024, dtype=torch.bfloat16, device=dev)
            gemm.launch_matmul_fp8e4m3(a8, b8, C8_ref, 512, 1024, 256, sa, sb)
            C8 = sharded.matmul_allgather(a8, b8[:, rank * w:(rank + 1) * w].contiguous(), pb,
                                          sa, sb[rank * w:(rank + 1) * w].contiguous())
            torch.cuda.synchronize()
            assert torch.equal(C8, C8_ref)
            assert lib().amp_device_status(1) == 0
        finally:
            pb.close()
        # (batch*head)-split attention + gather
        qa, ka, va = (torch.randn(2, 4, 256, 128, generator=g, device=dev).to(torch.bfloat16)
                      for _ in range(3))
        O, L = sharded.flash_attn_sharded(qa, ka, va, True)
        O_ref, L_ref = attention.flash_attn_fwd(qa, ka, va, True)
        assert torch.equal(O, O_ref) and torch.equal(L, L_ref)
        # the same with the all-gather fused into the attention epilogue; S = 200
        # leaves a partial last query tile
        po = PeerBuffer(CommGroup.current(), 2 * 4 * 200, 128, torch.bfloat16)
        pl = PeerBuffer(CommGroup.current(), 2 * 4, 200, torch.float32, mailboxes=po.mailboxes)
        try:
            qb, kb, vb = (t[:, :, :200].contiguous() for t in (qa, ka, va))
            Ob_ref, Lb_ref = attention.flash_attn_fwd(qb, kb, vb, True)
            for _ in range(2):
                Of, Lf = sharded.flash_attn_allgather(qb, kb, vb, True, po, pl)
                torch.cuda.synchronize()
                assert torch.equal(Of, Ob_ref) and torch.equal(Lf, Lb_ref)
                dist.barrier()
            assert lib().amp_device_status(1) == 0
        finally:
            pl.close()
            po.close()
        torch.cuda.synchronize()
        q.put((rank, "ok"))
    except Exception as e:
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_ops_match_single_gpu(amp_lib):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert all(v == "ok" for v in res.values()), res
