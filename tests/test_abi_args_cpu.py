"""C-ABI argument checks that run before any CUDA call, so they answer on a
machine without a GPU: each bad argument returns its AMP_ERR_* status and a
message, and nothing is launched."""
import ctypes as C

import pytest

from amp_b200._lib import AmpError, call

AMP_ERR_INVALID = -1


def test_wait_limit_is_range_checked(amp_lib):
    with pytest.raises(AmpError) as e:
        call("amp_set_wait_timeout_ns", 10**15)
    assert e.value.code == AMP_ERR_INVALID
    assert "cap" in str(e.value)
