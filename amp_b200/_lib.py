"""ctypes binding of libamp_b200.so (the C ABI declared in include/amp_b200.h).

The library is the product: there is no Python or CPU fallback.  If the
shared object is missing or cannot be loaded, every call raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libamp_b200.so"

_vp, _i32, _i64, _sz, _f32 = C.c_void_p, C.c_int, C.c_int64, C.c_size_t, C.c_float

# name -> (restype, argtypes); every entry point declared in include/amp_b200.h
# and include/amp_plugin.h is listed here (tests check the two agree).
SIGNATURES: dict[str, tuple] = {
    "amp_last_error": (C.c_char_p, []),
    "amp_abi_version": (_i32, []),
    "amp_fp8_quant_workspace_bytes": (_sz, [_i64]),
    "amp_fp8_quant_e4m3_dev": (_i32, [_vp, _i64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "amp_fp8_amax_bf16_dev": (_i32, [_vp, _i64, _vp, _vp, _sz, _vp]),
    "amp_fp8_amax_allreduce_peer_dev": (_i32, [_vp, _i64, _vp, _vp, _sz, _vp, _i32, _i32,
                                               C.c_uint, _vp]),
    "amp_fp8_quant_e4m3_from_amax_dev": (_i32, [_vp, _i64, _vp, _vp, _vp, _vp]),
    "amp_fp8_dequant_e4m3_dev": (_i32, [_vp, _i64, _vp, _vp, _vp]),
    "amp_fp8_quant_e4m3_noalloc_dev": (_i32, [_vp, _i64, _vp, _vp, _vp, _vp]),
    "amp_user_fp8_quant_e4m3": (_i32, [_vp, _i64, _vp, _vp, _vp]),
    "amp_user_fp8_dequant_e4m3": (_i32, [_vp, _i64, _f32, _vp]),
    "amp_device_status": (_i32, [_i32]),
    "amp_set_wait_timeout_ns": (_i32, [C.c_uint64]),
    "amp_release_staging": (_i32, []),
    "amp_gemm_bf16_dev": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp]),
    "amp_gemm_fp8e4m3_dev": (_i32, [_vp, _vp, _vp, _vp, _i32, _vp, _i32, _i32, _i32, _i32, _vp]),
    "amp_gemm_fp8e4m3_ex_dev": (_i32, [_vp, _vp, _vp, _vp, _i32, _vp, _i32, _vp, _vp, _i32, _i32,
                                       _i32, _vp]),
    "amp_gemm_bf16_allgather_dev": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32, _vp, C.c_uint, _i32,
                                           _i32, _i32, _vp]),
    "amp_gemm_fp8e4m3_allgather_dev": (_i32, [_vp, _vp, _vp, _vp, _i32, _vp, _i32, _i32, _i32, _vp,
                                              C.c_uint, _i32, _i32, _i32, _vp]),
    "amp_user_gemm_bf16": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32, _i32]),
    "amp_user_gemm_fp8e4m3": (_i32, [_vp, _vp, _vp, _vp, _i32, _vp, _i32, _i32, _i32, _i32]),
    "amp_flash_attn_fwd_bf16_dev": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32,
                                           _i32, _i32, _i32, _f32, _vp]),
    "amp_flash_attn_fwd_allgather_dev": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp,
                                                C.c_uint, _i32, _i32, _i32, _i32, _i32, _i32,
                                                _i32, _f32, _vp]),
    "amp_flash_attn_bwd_workspace_bytes": (_sz, [_i32, _i32, _i32]),
    "amp_flash_attn_bwd_bf16_dev": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32,
                                           _i32, _i32, _i32, _i32, _i32, _f32, _vp, _sz, _vp]),
    "amp_user_flash_attn_fwd_bf16": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32,
                                            _i32, _i32, _i32, _f32]),
    "amp_paged_decode_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32]),
    "amp_paged_attn_decode_bf16_dev": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32,
                                              _i32, _i32, _i32, _i32, _f32, _vp, _sz, _vp]),
    "amp_paged_attn_prefill_bf16_dev": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32,
                                               _i32, _i32, _i32, _i32, _i32, _f32, _vp]),
    "amp_paged_validate_block_table": (_i32, [_vp, _vp, _i32, _i32, _i32]),
    "amp_paged_pack_block_table": (_i32, [_vp, _vp, _vp, _i32, _i32, _vp]),
    "amp_paged_pool_bytes": (_sz, [_i32, _i32, _i32]),
    "amp_gemm_fp32_dev": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32, _vp]),
    "amp_gemm_fp32_exact_dev": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32, _vp]),
    "amp_gemm_fp32_3xtf32_dev": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32, _vp]),
    "amp_gemm_fp32_tile_dev": (_i32, [_i32, _i32, _i32, _vp, _vp, _vp, _i32, _i32, _i32, _vp]),
    "amp_user_gemm_fp32": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32]),
    "amp_peer_mailbox_bytes": (_sz, []),
    "amp_peer_handle_bytes": (_i32, []),
    "amp_peer_mailbox_create": (_i32, [_vp, _vp]),
    "amp_peer_mailbox_open": (_i32, [_vp, _vp]),
    "amp_peer_buffer_create": (_i32, [_sz, _vp, _vp]),
    "amp_peer_mailbox_close": (_i32, [_vp]),
    "amp_peer_mailbox_free": (_i32, [_vp]),
    "amp_peer_allreduce_max_f32": (_i32, [_vp, _vp, _vp, _i32, _i32, C.c_uint, _vp]),
    "amp_comm_available": (_i32, []),
    "amp_comm_nccl_version": (_i32, [_vp]),
    "amp_comm_unique_id": (_i32, [_vp]),
    "amp_comm_init_rank": (_i32, [_vp, _i32, _i32, _i32, _vp]),
    "amp_comm_destroy": (_i32, [_vp]),
    "amp_comm_rank": (_i32, [_vp, _vp, _vp, _vp]),
    "amp_comm_allreduce": (_i32, [_vp, _vp, _sz, _i32, _i32, _vp]),
    "amp_comm_allreduce_max_f32": (_i32, [_vp, _vp, _sz, _vp]),
    "amp_comm_allgather": (_i32, [_vp, _vp, _vp, _sz, _i32, _vp]),
    "amp_comm_broadcast": (_i32, [_vp, _vp, _sz, _i32, _i32, _vp]),
    "amp_comm_barrier": (_i32, [_vp, _vp]),
    "amp_gemm_sharded_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32]),
    "amp_gemm_bf16_sharded_dev": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp, _sz,
                                         _vp]),
    "amp_gemm_fp8e4m3_sharded_dev": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _vp, _i32, _i32, _i32,
                                            _i32, _vp, _sz, _vp]),
    "amp_flash_attn_fwd_sharded_dev": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32,
                                              _i32, _i32, _i32, _i32, _f32, _vp]),
}


class AmpError(RuntimeError):
    """A nonzero status from the C ABI (hard failure, as in amp_plugin.h)."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


_lock = threading.Lock()
_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """Load (once) and return the CUDA library; raises if it is not built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with `python -m amp_b200.build` "
                        "(there is no CPU fallback)")
                h = C.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | os.RTLD_LOCAL)
                for name, (res, args) in SIGNATURES.items():
                    f = getattr(h, name)
                    f.restype, f.argtypes = res, args
                _lib = h
    return _lib


def call(name: str, *args) -> int:
    """Call an int-status entry point and raise AmpError on a nonzero status."""
    h = lib()
    rc = getattr(h, name)(*args)
    if rc != 0:
        msg = h.amp_last_error()
        raise AmpError(name, rc, msg.decode() if msg else "")
    return rc
