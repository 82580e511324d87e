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


AMP_DTYPE_BF16, AMP_DTYPE_F32, AMP_REDUCE_MAX = 1, 0, 1


def test_nccl_loads_at_run_time(amp_lib):
    """The collectives find NCCL through dlopen; the library links none."""
    assert amp_lib.amp_comm_available() == 1
    v = C.c_int()
    call("amp_comm_nccl_version", C.byref(v))
    assert v.value >= 21800


def test_missing_nccl_is_reported_not_fatal(tmp_path):
    import subprocess
    import sys
    code = ("from amp_b200._lib import lib; h = lib(); "
            "print(h.amp_comm_available(), h.amp_last_error().decode())")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                       env={**__import__("os").environ,
                            "AMP_B200_NCCL_LIB": str(tmp_path / "libnccl_absent.so")},
                       cwd=str(__import__("pathlib").Path(__file__).resolve().parents[1]))
    assert r.returncode == 0, r.stderr
    avail, msg = r.stdout.strip().split(" ", 1)
    assert avail == "0" and "NCCL is not available" in msg


@pytest.mark.parametrize("rank,world", [(0, 0), (2, 2), (-1, 4)])
def test_comm_init_rejects_bad_rank_or_world(rank, world, amp_lib):
    comm = C.c_void_p()
    uid = (C.c_ubyte * 128)()
    with pytest.raises(AmpError) as e:
        call("amp_comm_init_rank", C.byref(comm), rank, world, 0, uid)
    assert e.value.code == AMP_ERR_INVALID
    assert comm.value is None


def test_comm_ops_reject_missing_communicator_and_bad_types(amp_lib):
    buf = (C.c_float * 4)()
    for args in [("amp_comm_allreduce", None, buf, 4, AMP_DTYPE_F32, AMP_REDUCE_MAX, None),
                 ("amp_comm_allreduce", None, buf, 4, 9, AMP_REDUCE_MAX, None),
                 ("amp_comm_allreduce", None, buf, 4, AMP_DTYPE_F32, 7, None),
                 ("amp_comm_allgather", None, buf, buf, 4, AMP_DTYPE_F32, None),
                 ("amp_comm_broadcast", None, buf, 4, AMP_DTYPE_F32, 0, None),
                 ("amp_comm_barrier", None, None),
                 ("amp_gemm_bf16_sharded_dev", None, buf, buf, buf, AMP_DTYPE_BF16, 8, 8, 8, buf,
                  1 << 20, None),
                 ("amp_flash_attn_fwd_sharded_dev", None, buf, buf, buf, buf, None, 1, 1, 1, 8, 8,
                  128, 1, 0.0, None)]:
        with pytest.raises(AmpError) as e:
            call(*args)
        assert e.value.code == AMP_ERR_INVALID, args[0]
    assert call("amp_comm_destroy", None) == 0


def test_sharded_gemm_workspace_size(amp_lib):
    assert amp_lib.amp_gemm_sharded_workspace_bytes(1024, 512, 4, AMP_DTYPE_BF16) == \
        1024 * 512 * 4 * 2
    assert amp_lib.amp_gemm_sharded_workspace_bytes(1024, 512, 4, AMP_DTYPE_F32) == \
        1024 * 512 * 4 * 4
    assert amp_lib.amp_gemm_sharded_workspace_bytes(0, 512, 4, AMP_DTYPE_F32) == 0
