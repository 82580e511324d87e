"""Sharding and collective logic on world_size 2 over gloo (CPU, no GPU).

Each rank computes its shard with the oracle (numpy/torch CPU maths stands in
for the kernel); the collectives and layouts of amp_b200.collective are the
same code the NCCL path runs.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, fn_name, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import test_collective_cpu as mod
        getattr(mod, fn_name)(rank, world)
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent, which fails the test
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def run_ranks(fn_name, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn_name, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert all(v == "ok" for v in res.values()), res


# ---- rank bodies -------------------------------------------------------
def body_global_amax(rank, world):
    import oracle
    from amp_b200 import workloads
    from amp_b200.collective import CommGroup, global_amax
    g = CommGroup.current()
    full = workloads.quant_input_numpy(4096 * world, seed=5)
    shard = full[rank * 4096:(rank + 1) * 4096]
    local = torch.tensor([oracle.quant_e4m3(shard)[2]], dtype=torch.float32)
    global_amax(g, local)
    q_full, s_full, a_full = oracle.quant_e4m3(full)
    assert local.item() == np.float32(a_full)
    # encoding the shard with the global amax reproduces the unsharded codes
    q_shard = oracle.quant_e4m3_with_amax(shard, local.item())
    assert (q_shard == q_full[rank * 4096:(rank + 1) * 4096]).all()


def body_gather_columns(rank, world):
    from amp_b200.collective import CommGroup, column_range, gather_columns
    g = CommGroup.current()
    rng = np.random.default_rng(0)
    A = torch.from_numpy(rng.standard_normal((64, 32)))
    B = torch.from_numpy(rng.standard_normal((32, 256)))
    lo, hi = column_range(256, g, align=64)
    C = gather_columns(g, A @ B[:, lo:hi].contiguous())
    assert torch.allclose(C, A @ B)


def body_gather_heads(rank, world):
    from oracle import attention as ref
    from amp_b200.collective import CommGroup, gather_heads, head_range
    g = CommGroup.current()
    rng = np.random.default_rng(1)
    q, k, v = (rng.standard_normal((2, 4, 40, 16)) for _ in range(3))
    lo, hi = head_range(8, g)
    qs, ks, vs = (t.reshape(8, 40, 16)[lo:hi][None] for t in (q, k, v))
    o, lse = ref.flash_attn_fwd(qs, ks, vs, True)
    O = gather_heads(g, torch.from_numpy(o[0])).reshape(2, 4, 40, 16).numpy()
    L = gather_heads(g, torch.from_numpy(lse[0])).reshape(2, 4, 40).numpy()
    O_ref, L_ref = ref.flash_attn_fwd(q, k, v, True)
    assert np.allclose(O, O_ref) and np.allclose(L, L_ref)


def body_other_collectives(rank, world):
    from amp_b200.collective import CommGroup, allreduce, barrier, broadcast, reduce_scatter
    g = CommGroup.current()
    t = torch.tensor([float(rank + 1)])
    assert allreduce(g, t.clone(), "sum").item() == world * (world + 1) / 2
    b = broadcast(g, torch.tensor([rank * 10.0]), root=1)
    assert b.item() == 10.0
    rs = reduce_scatter(g, torch.arange(world * 3, dtype=torch.float32).reshape(world, 3))
    assert torch.equal(rs, world * torch.arange(rank * 3, rank * 3 + 3, dtype=torch.float32))
    barrier(g)


def body_mailbox_resync_after_one_rank_raises(rank, world):
    """Rank 1 rejects an exchange before its launch (a check that failed on it
    alone) while rank 0 used the number; resync() puts both on one counter."""
    from amp_b200.collective import CommGroup, PeerMailboxes
    mb = object.__new__(PeerMailboxes)
    mb.g, mb.seq = CommGroup.current(), 6
    try:
        with mb.sequence() as seq:
            assert seq == 7
            if rank == 1:
                raise ValueError("rejected on this rank only")
    except ValueError:
        pass
    assert mb.seq == (7 if rank == 0 else 6)
    assert mb.resync() == 7
    with mb.sequence() as seq:
        got = torch.tensor([seq])
    both = [torch.zeros(1, dtype=got.dtype) for _ in range(world)]
    dist.all_gather(both, got)
    assert [int(t) for t in both] == [8] * world


@pytest.mark.parametrize("body", ["body_global_amax", "body_gather_columns", "body_gather_heads",
                                  "body_other_collectives",
                                  "body_mailbox_resync_after_one_rank_raises"])
def test_two_ranks_gloo(body):
    run_ranks(body)


def test_single_rank_is_identity():
    from amp_b200.collective import CommGroup, allgather, column_range, gather_columns
    g = CommGroup()
    x = torch.arange(6.0).reshape(2, 3)
    assert torch.equal(allgather(g, x)[0], x)
    assert torch.equal(gather_columns(g, x), x)
    assert column_range(256, g, 64) == (0, 256)
    with pytest.raises(ValueError):
        column_range(100, CommGroup(0, 3), 1)


def test_mailbox_sequence_alternates_parity_across_the_wrap():
    """Exchanges use mailbox row seq & 1; two consecutive exchanges in one row would
    let a fast rank overwrite a value a slow rank has not read."""
    from amp_b200.collective import PeerMailboxes
    mb = object.__new__(PeerMailboxes)
    mb.seq = 0
    first = [mb.next_seq() for _ in range(4)]
    assert first == [1, 2, 3, 4]
    mb.seq = 0xFFFFFFFE - 3
    seqs = [mb.next_seq() for _ in range(8)]
    assert 0 not in seqs and max(seqs) <= 0xFFFFFFFE
    assert all((a ^ b) & 1 for a, b in zip(seqs, seqs[1:])), seqs
    assert seqs[2] == 0xFFFFFFFE and seqs[3] == 1


def test_sequence_number_is_given_back_when_nothing_was_launched():
    """An exchange that raises before its launch must not use up a sequence number
    (the next exchange would reuse the last one's row)."""
    from amp_b200.collective import PeerMailboxes
    mb = object.__new__(PeerMailboxes)
    mb.seq = 0xFFFFFFFE
    with pytest.raises(RuntimeError):
        with mb.sequence() as seq:
            assert seq == 1
            raise RuntimeError("rejected before launch")
    assert mb.seq == 0xFFFFFFFE
    with mb.sequence() as seq:
        assert seq == 1
    assert mb.seq == 1 and mb.next_seq() == 2
