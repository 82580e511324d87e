"""Collectives for sharded use of the kernels: the thin NCCL layer.

Mirrors the operations of the reference's include/collective.hpp
(allreduce / allgather / broadcast / reduce_scatter / barrier,
collective.hpp:79-104, CommGroup collective.hpp:34-40) on top of
torch.distributed, whose NCCL backend runs over NVLink / NVSwitch on a B200
node.  Only two exchanges sit on the hot path: a 1-float all-reduce(MAX) of
the FP8 amax and the all-gather that reassembles a sharded output.  The
functions are backend-agnostic (gloo on CPU runs them in tests).
"""
from __future__ import annotations

import contextlib
import ctypes as C
from dataclasses import dataclass

import torch
import torch.distributed as dist

_OPS = {"sum": dist.ReduceOp.SUM, "max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN,
        "prod": dist.ReduceOp.PRODUCT}


@dataclass
class CommGroup:
    """The reference's CommGroup (rank, world, device) over a process group."""
    rank: int = 0
    world: int = 1
    device_id: int = 0
    group: object = None

    @classmethod
    def current(cls, group=None) -> "CommGroup":
        if not dist.is_available() or not dist.is_initialized():
            return cls()
        dev = torch.cuda.current_device() if torch.cuda.is_available() else 0
        return cls(dist.get_rank(group), dist.get_world_size(group), dev, group)


def allreduce(g: CommGroup, buf: torch.Tensor, op: str = "sum") -> torch.Tensor:
    if g.world > 1:
        dist.all_reduce(buf, op=_OPS[op], group=g.group)
    return buf


def broadcast(g: CommGroup, buf: torch.Tensor, root: int = 0) -> torch.Tensor:
    if g.world > 1:
        dist.broadcast(buf, src=root, group=g.group)
    return buf


def allgather(g: CommGroup, send: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out[r] = send of rank r (out has a leading world dimension)."""
    out = out if out is not None else send.new_empty((g.world, *send.shape))
    if g.world == 1:
        out[0].copy_(send)
    else:
        # the concatenated-along-dim-0 form is accepted by every backend
        flat = out.view(g.world * send.shape[0], *send.shape[1:]) if send.dim() else out
        dist.all_gather_into_tensor(flat, send.contiguous(), group=g.group)
    return out


def reduce_scatter(g: CommGroup, send: torch.Tensor, op: str = "sum") -> torch.Tensor:
    """send has a leading world dimension; returns this rank's reduced slice."""
    out = send.new_empty(send.shape[1:])
    if g.world == 1:
        out.copy_(send[0])
    else:
        flat = send.contiguous().view(-1, *send.shape[2:]) if send.dim() > 1 else send
        dist.reduce_scatter_tensor(out, flat, op=_OPS[op], group=g.group)
    return out


def barrier(g: CommGroup) -> None:
    if g.world > 1:
        dist.barrier(group=g.group)


# ----------------------------------------------------------------------
# partitioning of the three sharded workloads
# ----------------------------------------------------------------------
def column_range(n: int, g: CommGroup, align: int = 1) -> tuple[int, int]:
    """This rank's [start, stop) of n columns; every shard a multiple of `align`."""
    if n % (g.world * align):
        raise ValueError(f"{n} columns do not split into {g.world} shards of multiples of {align}")
    w = n // g.world
    return g.rank * w, (g.rank + 1) * w


def gather_columns(g: CommGroup, c_shard: torch.Tensor) -> torch.Tensor:
    """All-gather N-sharded C blocks [M, N/p] and lay them out as row-major [M, N]."""
    parts = allgather(g, c_shard)                 # [p, M, N/p]
    return parts.permute(1, 0, 2).reshape(c_shard.shape[0], -1)


def head_range(bh: int, g: CommGroup) -> tuple[int, int]:
    """This rank's contiguous slice of the flattened batch*heads of attention."""
    if bh % g.world:
        raise ValueError(f"{bh} batch*heads do not split over {g.world} ranks")
    w = bh // g.world
    return g.rank * w, (g.rank + 1) * w


def gather_heads(g: CommGroup, o_shard: torch.Tensor) -> torch.Tensor:
    """All-gather (batch*head)-sharded outputs [bh/p, ...] into [bh, ...]."""
    parts = allgather(g, o_shard)
    return parts.reshape(-1, *o_shard.shape[1:])


def global_amax(g: CommGroup, local_amax: torch.Tensor) -> torch.Tensor:
    """1-float all-reduce(MAX): the per-tensor amax of a tensor sharded over ranks."""
    return allreduce(g, local_amax, "max")


class PeerMailboxes:
    """Each rank's small device mailbox, opened by every other rank of the node
    through CUDA IPC, so one-word exchanges (the quantiser's amax) travel as a
    single NVLink store per peer instead of an NCCL all-reduce.

    Collective: every rank of `g` constructs it, and closes it, at the same point.
    `table` is the device array of mailbox pointers the kernels take."""

    def __init__(self, g: CommGroup):
        from ._lib import call, lib
        self.g, self.seq = g, 0
        n = int(lib().amp_peer_handle_bytes())
        handle = (C.c_ubyte * n)()
        own = C.c_void_p()
        call("amp_peer_mailbox_create", C.byref(own), handle)
        self.own = own.value
        handles = [bytes(handle)]
        if g.world > 1:
            handles = [None] * g.world
            dist.all_gather_object(handles, bytes(handle), group=g.group)
        ptrs, self._opened = [], []
        for r, hb in enumerate(handles):
            if r == g.rank:
                ptrs.append(self.own)
                continue
            p = C.c_void_p()
            call("amp_peer_mailbox_open", (C.c_ubyte * n).from_buffer_copy(hb), C.byref(p))
            ptrs.append(p.value)
            self._opened.append(p.value)
        self.table = torch.tensor(ptrs, dtype=torch.int64,
                                  device=torch.device("cuda", torch.cuda.current_device()))

    def next_seq(self) -> int:
        """Sequence number of the next exchange (the same on every rank): 1, 2, ...,
        2**32 - 2, then 1 again.  An exchange uses mailbox row seq & 1, so consecutive
        numbers must alternate in parity, also across the wrap (2**32 - 2 is even)."""
        self.seq = self.seq % 0xFFFFFFFE + 1
        return self.seq

    @contextlib.contextmanager
    def sequence(self):
        """The sequence number of one exchange, given back if the body raises (the
        exchange was never launched): a number used up without its exchange would
        make the next exchange reuse the last one's row.

        This keeps the ranks in step when every rank raises alike, which is the
        case for argument checks that depend only on shapes and types every rank
        shares.  If only some ranks raise, the others have launched and used the
        number (their exchange ends in the device timeout status): call
        `resync()` on every rank before the next exchange."""
        prev = self.seq
        seq = self.next_seq()
        try:
            yield seq
        except BaseException:
            self.seq = prev
            raise

    def resync(self) -> int:
        """Collective: agree on the sequence counter after an exchange that failed
        on some ranks only.  Every rank takes the largest counter of the group, so
        the next exchange has one number everywhere and a row no rank used last."""
        if self.g.world > 1:
            dev = (torch.device("cuda", torch.cuda.current_device())
                   if dist.get_backend(self.g.group) == "nccl" else torch.device("cpu"))
            t = torch.tensor([self.seq], dtype=torch.int64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.g.group)
            self.seq = int(t.item())
        return self.seq

    def close(self) -> None:
        from ._lib import call
        if self.own is None:
            return
        torch.cuda.synchronize()
        barrier(self.g)                 # nobody posts any more
        for p in self._opened:
            call("amp_peer_mailbox_close", p)
        barrier(self.g)                 # every peer has unmapped this rank's mailbox
        call("amp_peer_mailbox_free", self.own)
        self.own, self._opened = None, []


_TYPESTR = {torch.bfloat16: "<i2", torch.float32: "<f4", torch.uint8: "|u1"}


class _CudaArray:
    """Zero-copy view of a raw device pointer (__cuda_array_interface__)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3}


class PeerBuffer:
    """A [rows, cols] output replicated on every rank of `g`, which the other
    ranks write into directly over NVLink (CUDA IPC): the C of the all-gather
    GEMM.  `tensor` is this rank's copy, `table` the device array of every
    rank's pointer that the kernels take, `mailboxes` the completion mailboxes.

    Collective: every rank constructs it, and closes it, at the same point."""

    def __init__(self, g: CommGroup, rows: int, cols: int, dtype=torch.bfloat16,
                 mailboxes: "PeerMailboxes | None" = None):
        from ._lib import call, lib
        if dtype not in _TYPESTR:
            raise ValueError(f"unsupported peer buffer dtype {dtype}")
        self.g, self.shape, self.dtype = g, (rows, cols), dtype
        esz = torch.tensor([], dtype=dtype).element_size()
        n = int(lib().amp_peer_handle_bytes())
        handle = (C.c_ubyte * n)()
        own = C.c_void_p()
        call("amp_peer_buffer_create", rows * cols * esz, C.byref(own), handle)
        self.own = own.value
        handles = [bytes(handle)]
        if g.world > 1:
            handles = [None] * g.world
            dist.all_gather_object(handles, bytes(handle), group=g.group)
        ptrs, self._opened = [], []
        for r in range(g.world):
            if r == g.rank:
                ptrs.append(self.own)
                continue
            p = C.c_void_p()
            call("amp_peer_mailbox_open", (C.c_ubyte * n).from_buffer_copy(handles[r]), C.byref(p))
            ptrs.append(p.value)
            self._opened.append(p.value)
        dev = torch.device("cuda", torch.cuda.current_device())
        self.table = torch.tensor(ptrs, dtype=torch.int64, device=dev)
        # torch reads bf16 through the array interface as int16 and reinterprets it;
        # the view does not own the memory, so it must not outlive close()
        raw = torch.as_tensor(_CudaArray(self.own, (rows, cols), _TYPESTR[dtype]), device=dev)
        self.tensor = raw.view(dtype) if dtype == torch.bfloat16 else raw
        self._own_mb = mailboxes is None
        self.mailboxes = mailboxes if mailboxes is not None else PeerMailboxes(g)

    def close(self) -> None:
        from ._lib import call
        if self.own is None:
            return
        torch.cuda.synchronize()
        barrier(self.g)                 # nobody writes any more
        for p in self._opened:
            call("amp_peer_mailbox_close", p)
        barrier(self.g)                 # every peer has unmapped this rank's buffer
        self.tensor = None
        call("amp_peer_mailbox_free", self.own)
        self.own, self._opened = None, []
        if self._own_mb:
            self.mailboxes.close()
