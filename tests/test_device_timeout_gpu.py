"""The device-side failure path: a bounded wait that runs out ends its kernel
with the timeout status instead of hanging, and the GPU stays usable.

The wait is made to run out on one GPU with no peer process: a two-rank
all-reduce(max) through peer mailboxes whose second mailbox is a plain local
buffer nobody ever posts to.  With the wait limit lowered to 10 ms the kernel
gives up, amp_device_status reports AMP_ERR_TIMEOUT, and the next call (a
one-rank exchange, then a GEMM) runs normally.
"""
import ctypes as C
import time

import pytest
import torch

from amp_b200._lib import AmpError, call, lib

pytestmark = pytest.mark.gpu

AMP_ERR_TIMEOUT = -3


def test_mailbox_wait_times_out_and_the_device_recovers(cuda, amp_lib):
    dev = cuda
    own = C.c_void_p()
    handle = (C.c_ubyte * int(lib().amp_peer_handle_bytes()))()
    call("amp_peer_mailbox_create", C.byref(own), handle)
    silent = torch.zeros(int(lib().amp_peer_mailbox_bytes()) // 8, dtype=torch.int64, device=dev)
    table = torch.tensor([own.value, silent.data_ptr()], dtype=torch.int64, device=dev)
    x = torch.tensor([3.5], device=dev)
    out = torch.zeros(1, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    try:
        call("amp_device_status", 1)                       # start from a clear flag
        call("amp_set_wait_timeout_ns", 10_000_000)        # 10 ms
        t0 = time.perf_counter()
        call("amp_peer_allreduce_max_f32", x.data_ptr(), out.data_ptr(), table.data_ptr(), 0, 2,
             1, stream)
        torch.cuda.synchronize(dev)
        waited = time.perf_counter() - t0
        assert waited < 1.0, f"the kernel took {waited:.3f} s to give up on a 10 ms limit"
        with pytest.raises(AmpError) as e:
            call("amp_device_status", 1)
        assert e.value.code == AMP_ERR_TIMEOUT
        assert call("amp_device_status", 0) == 0           # the flag was cleared
        # the context is intact: a one-rank exchange and a GEMM run normally
        one = torch.tensor([own.value], dtype=torch.int64, device=dev)
        call("amp_peer_allreduce_max_f32", x.data_ptr(), out.data_ptr(), one.data_ptr(), 0, 1, 2,
             stream)
        a = torch.randn(256, 256, device=dev).to(torch.bfloat16)
        b = torch.randn(256, 256, device=dev).to(torch.bfloat16)
        c = torch.empty(256, 256, dtype=torch.bfloat16, device=dev)
        call("amp_gemm_bf16_dev", a.data_ptr(), b.data_ptr(), c.data_ptr(), 1, 256, 256, 256,
             stream)
        torch.cuda.synchronize(dev)
        assert out.item() == 3.5
        ref = a.double() @ b.double()
        err = ((c.double() - ref).abs() / ref.abs().clamp_min(1)).max().item()
        assert err < 2e-2, err
        assert call("amp_device_status", 1) == 0
    finally:
        call("amp_set_wait_timeout_ns", 0)                 # back to the 2 s default
        torch.cuda.synchronize(dev)
        call("amp_peer_mailbox_free", own.value)

