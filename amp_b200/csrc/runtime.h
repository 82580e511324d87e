// runtime.h -- host-side helpers shared by the entry points.
#pragma once
#include <cstddef>

#include <cuda.h>
#include <cuda_runtime.h>

namespace ampb {

// Returns a device buffer of at least `bytes` for staging slot `slot` on the
// current device (grow-only, kept until process exit).  Slots let one call
// hold several live buffers.  Not re-entrant across threads for one slot.
int staging_get(int slot, size_t bytes, void** out);
// Frees every staging buffer of the current device (after synchronising it).
int staging_release_current_device();
// Called by each amp_user_* entry point on success just before it returns:
// releases the staging buffers when AMP_B200_RELEASE_STAGING is set.
int staging_end_of_call();

// Per-device status word written by kernels whose bounded waits expired
// (AMP_DEV_ERR_TIMEOUT); allocated and zeroed on first use.
int device_status(int** out);

// cuTensorMapEncodeTiled from the driver (looked up once, thread-safe) applied
// with the library's fixed options: bf16 / fp32 / u8 elements (es 2 / 4 / 1),
// no interleave, 128-byte swizzle, 256-byte L2 promotion, zero out-of-bounds fill.
int encode_tmap(CUtensorMap* m, const void* base, int es, int rank, const cuuint64_t* dims,
                const cuuint64_t* strides, const cuuint32_t* box);

// Launch with programmatic stream serialization: the kernel may start while the
// previous kernel in the stream drains; it must call pdl_wait() (common.cuh)
// before touching that kernel's data.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace ampb
