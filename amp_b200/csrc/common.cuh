// common.cuh -- shared host/device helpers for the sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cstdio>

#include "../../include/amp_b200.h"
#include "../../include/amp_plugin.h"

namespace ampb {

// ---------------------------------------------------------------------------
// Host-side status handling: every C-ABI entry point returns an int status
// (0 = success) and records a message retrievable by amp_last_error().
// ---------------------------------------------------------------------------
void set_error(int code, const char* fmt, ...);
int cuda_status(cudaError_t e, const char* where);

#define AMPB_CHECK_CUDA(expr)                                         \
    do {                                                              \
        cudaError_t _e = (expr);                                      \
        if (_e != cudaSuccess) return ::ampb::cuda_status(_e, #expr); \
    } while (0)

#define AMPB_REQUIRE(cond, code, ...)                                 \
    do {                                                              \
        if (!(cond)) {                                                \
            ::ampb::set_error((code), __VA_ARGS__);                   \
            return (code);                                            \
        }                                                             \
    } while (0)

// Launch-error check after a <<<>>> launch.
#define AMPB_CHECK_LAUNCH(name) AMPB_CHECK_CUDA(cudaGetLastError())

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Number of SMs of the current device (cached per device ordinal).
int sm_count();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------

// Programmatic dependent launch (kernels launched with launch_pdl): `pdl_wait`
// blocks until the kernel before this one in the stream has completed and its
// memory is visible -- called first thing, before this kernel reads or writes
// anything the previous one touches; `pdl_trigger` lets the next kernel's CTAs
// start launching (they wait in their own pdl_wait) while this grid finishes.
// Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Streaming 128-bit global load that bypasses L1 allocation (read-once data).
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Streaming 64-bit global load, no L1 allocation.
__device__ __forceinline__ uint2 ldg_stream_v2(const void* p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
                 : "=r"(v.x), "=r"(v.y)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void stg_v4(void* p, uint4 v) {
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

// Two fp32 -> two E4M3 codes, round-to-nearest-even with saturation to
// +-448 (NaN stays NaN).  `lo` lands in bits [0,8), `hi` in bits [8,16).
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float lo, float hi) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}

// Two E4M3 codes (bits [0,8) and [8,16)) -> two exact fp16 values packed.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
    uint32_t r;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
    return r;
}

__device__ __forceinline__ float f16_lo_to_f32(uint32_t h2) {
    float f;
    asm("{ .reg .b16 lo, hi; mov.b32 {lo, hi}, %1; cvt.f32.f16 %0, lo; }" : "=f"(f) : "r"(h2));
    return f;
}
__device__ __forceinline__ float f16_hi_to_f32(uint32_t h2) {
    float f;
    asm("{ .reg .b16 lo, hi; mov.b32 {lo, hi}, %1; cvt.f32.f16 %0, hi; }" : "=f"(f) : "r"(h2));
    return f;
}

// Two fp32 -> packed bf16x2 (round-to-nearest-even); `lo` in bits [0,16).
__device__ __forceinline__ uint32_t f32x2_to_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace ampb
