// runtime.cu -- status reporting, device queries and the host-pointer staging
// pool shared by the amp_user_* entry points.
#include <cstdarg>
#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "tc_common.cuh"
#include "runtime.h"

namespace ampb {

namespace {
thread_local char g_msg[512] = "ok";
}

void set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    int off = std::snprintf(g_msg, sizeof g_msg, "[%d] ", code);
    if (off < 0) off = 0;
    std::vsnprintf(g_msg + off, sizeof g_msg - (size_t)off, fmt, ap);
    va_end(ap);
}

int cuda_status(cudaError_t e, const char* where) {
    set_error((int)e, "CUDA error %s (%s) at %s", cudaGetErrorName(e), cudaGetErrorString(e),
              where);
    return (int)e;
}

int sm_count() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
}  // namespace

int encode_tmap(CUtensorMap* m, const void* base, int es, int rank, const cuuint64_t* dims,
                const cuuint64_t* strides, const cuuint32_t* box) {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    static cudaError_t err = cudaSuccess;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
        if (err == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = (EncodeTiledFn)p;
    });
    if (!fn) {
        if (err != cudaSuccess) return cuda_status(err, "cudaGetDriverEntryPoint");
        set_error(AMP_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled not available from the driver");
        return AMP_ERR_UNSUPPORTED;
    }
    const CUtensorMapDataType dt = es == 4   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : es == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                             : CU_TENSOR_MAP_DATA_TYPE_UINT8;
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    const CUresult r = fn(m, dt, (cuuint32_t)rank, const_cast<void*>(base), dims, strides, box,
                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    AMPB_REQUIRE(r == CUDA_SUCCESS, AMP_ERR_INVALID,
                 "cuTensorMapEncodeTiled failed (%d) for a rank-%d tensor", (int)r, rank);
    return AMP_OK;
}

// Grow-only per-device staging buffers for the host-pointer entry points, so
// that repeated amp_user_* calls do not pay cudaMalloc/cudaFree each time.
namespace {
struct Slot {
    void* ptr = nullptr;
    size_t bytes = 0;
};
std::mutex g_pool_mu;
std::vector<std::vector<Slot>> g_pool;  // [device][slot]
}  // namespace

int staging_release_current_device() {
    int dev = 0;
    AMPB_CHECK_CUDA(cudaGetDevice(&dev));
    AMPB_CHECK_CUDA(cudaDeviceSynchronize());  // nothing queued may still use a buffer
    std::lock_guard<std::mutex> lk(g_pool_mu);
    if ((int)g_pool.size() <= dev) return AMP_OK;
    for (Slot& s : g_pool[dev]) {
        if (s.ptr) AMPB_CHECK_CUDA(cudaFree(s.ptr));
        s.ptr = nullptr;
        s.bytes = 0;
    }
    return AMP_OK;
}

int staging_end_of_call() {
    // AMP_B200_RELEASE_STAGING=1: every amp_user_* call returns its device
    // buffers before it returns, as include/amp_plugin.h:32-39 words the contract
    static const bool release = [] {
        const char* e = std::getenv("AMP_B200_RELEASE_STAGING");
        return e && *e && std::strcmp(e, "0") != 0;
    }();
    return release ? staging_release_current_device() : AMP_OK;
}

int staging_get(int slot, size_t bytes, void** out) {
    int dev = 0;
    AMPB_CHECK_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(g_pool_mu);
    if ((int)g_pool.size() <= dev) g_pool.resize(dev + 1);
    auto& slots = g_pool[dev];
    if ((int)slots.size() <= slot) slots.resize(slot + 1);
    Slot& s = slots[slot];
    if (s.bytes < bytes) {
        if (s.ptr) AMPB_CHECK_CUDA(cudaFree(s.ptr));
        s.ptr = nullptr;
        s.bytes = 0;
        size_t want = bytes < 256 ? 256 : bytes;
        AMPB_CHECK_CUDA(cudaMalloc(&s.ptr, want));
        s.bytes = want;
    }
    *out = s.ptr;
    return AMP_OK;
}

namespace {
std::mutex g_status_mu;
std::vector<int*> g_status;  // [device]
}  // namespace

int device_status(int** out) {
    int dev = 0;
    AMPB_CHECK_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(g_status_mu);
    if ((int)g_status.size() <= dev) g_status.resize(dev + 1, nullptr);
    if (!g_status[dev]) {
        // status word (int 0) + wait limit (u64 at byte 8), see tc_common.cuh
        struct Block { int status[2]; unsigned long long limit_ns; };
        static_assert(offsetof(Block, limit_ns) == kStatusLimitOffsetInts * sizeof(int), "layout");
        const Block init = {{AMP_DEV_OK, 0}, kWaitTimeoutNs};
        int* p = nullptr;
        AMPB_CHECK_CUDA(cudaMalloc(&p, sizeof(Block)));
        const cudaError_t e = cudaMemcpy(p, &init, sizeof(Block), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            cudaFree(p);
            return cuda_status(e, "cudaMemcpy(status block)");
        }
        g_status[dev] = p;
    }
    *out = g_status[dev];
    return AMP_OK;
}

}  // namespace ampb

extern "C" {

int amp_device_status(int clear) {
    int* p = nullptr;
    int rc = ampb::device_status(&p);
    if (rc) return rc;
    int v = 0;
    AMPB_CHECK_CUDA(cudaDeviceSynchronize());
    AMPB_CHECK_CUDA(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
    if (v && clear) AMPB_CHECK_CUDA(cudaMemset(p, 0, sizeof(int)));
    if (v == 2) {
        ampb::set_error(AMP_ERR_INVALID, "a kernel met a page id outside the KV pool "
                        "(device status 2); the affected pages were skipped");
        return AMP_ERR_INVALID;
    }
    if (v) {
        ampb::set_error(AMP_ERR_TIMEOUT, "a kernel's bounded wait expired (device status %d)", v);
        return AMP_ERR_TIMEOUT;
    }
    return AMP_OK;
}

int amp_set_wait_timeout_ns(uint64_t ns) {
    AMPB_REQUIRE(ns <= 600ull * 1000000000ull, AMP_ERR_INVALID,
                 "wait limit %llu ns is above the 600 s cap", (unsigned long long)ns);
    int* p = nullptr;
    int rc = ampb::device_status(&p);
    if (rc) return rc;
    const unsigned long long v = ns ? ns : ampb::kWaitTimeoutNs;
    // ordered after every kernel already queued on the device (blocking copy)
    AMPB_CHECK_CUDA(cudaDeviceSynchronize());
    AMPB_CHECK_CUDA(cudaMemcpy(p + ampb::kStatusLimitOffsetInts, &v, sizeof(v),
                               cudaMemcpyHostToDevice));
    return AMP_OK;
}

int amp_release_staging(void) { return ampb::staging_release_current_device(); }

const char* amp_last_error(void) { return ampb::g_msg; }

int amp_abi_version(void) { return 100; /* 0.1.0 */ }

}  // extern "C"
