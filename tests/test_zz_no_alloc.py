"""The allocation-free quantiser entry point gives the same result as the
workspace one.

amp_fp8_quant_e4m3_noalloc_dev serves callers that cannot call cudaMalloc when
they quantise (for example an engine plugin that may only use the memory its
engine passes in, or a runtime that owns and budgets every device allocation).
It keeps its scratch in a library-owned device array instead of a caller
workspace.  This file is collected last so a failure here never hides the
other tests' results.
"""

import numpy as np
import pytest
import torch

from amp_b200 import workloads
from amp_b200._lib import call

pytestmark = pytest.mark.gpu


def _dev_bf16(bits, device):
    return torch.from_numpy(bits.view(np.int16).copy()).to(device).view(torch.bfloat16)


def _run(entry, x, with_workspace):
    dev = x.device
    q = torch.empty(x.numel(), dtype=torch.uint8, device=dev)
    scale = torch.empty(1, dtype=torch.float32, device=dev)
    amax = torch.empty(1, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    if with_workspace:
        from amp_b200._lib import lib
        ws_bytes = lib().amp_fp8_quant_workspace_bytes(x.numel())
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        call(entry, x.data_ptr(), x.numel(), q.data_ptr(), scale.data_ptr(), amax.data_ptr(),
             ws.data_ptr(), ws_bytes, stream)
    else:
        call(entry, x.data_ptr(), x.numel(), q.data_ptr(), scale.data_ptr(), amax.data_ptr(),
             stream)
    torch.cuda.synchronize(dev)
    return q.cpu().numpy(), scale.item(), amax.item()


def test_noalloc_matches_workspace_entry_point_twice_in_a_row(cuda, amp_lib):
    # Two calls in a row on different tensors through the shared scratch
    # array: a large one (one partial maximum per block of a full grid, outliers up to ~250)
    # and then a small one whose values are all far below the first call's
    # amax.  Both must give the workspace entry point's codes, scale and amax
    # exactly, i.e. the second call's result depends on its own input only.
    for n, seed in ((1 << 22) + 5, 101), (3001, 102):
        bits = workloads.quant_input_numpy(n, seed=seed)
        if n == 3001:
            bits[:] = (bits & 0x807F) | 0x3C00  # small magnitudes: amax far below call 1's
        x = _dev_bf16(bits, cuda)
        q_ref, s_ref, a_ref = _run("amp_fp8_quant_e4m3_dev", x, with_workspace=True)
        q, s, a = _run("amp_fp8_quant_e4m3_noalloc_dev", x, with_workspace=False)
        assert s == s_ref and a == a_ref, (n, s, s_ref, a, a_ref)
        assert np.array_equal(q, q_ref), f"n={n}: {np.count_nonzero(q != q_ref)} codes differ"


def test_noalloc_rejects_bad_size(cuda, amp_lib):
    from amp_b200._lib import AmpError
    with pytest.raises(AmpError) as e:
        call("amp_fp8_quant_e4m3_noalloc_dev", None, -1, None, None, None, None)
    assert e.value.code == -1
