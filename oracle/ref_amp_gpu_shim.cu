// ref_amp_gpu_shim.cu -- TEST INFRASTRUCTURE ONLY (a comparator, never the product).
//
// AMP's own device code -- the FP32 tiled GEMM and BF16 WMMA GEMM of
// kernels/matmul.cu, the cuBLASLt FP8 GEMM that kernels/matmul.cu:235-270
// reaches through src/gemm_vendor.cpp, and the FA2 forward of
// kernels/flash_attn.cu -- compiled in place from the reference tree for
// sm_100a (recipe: oracle/Makefile, target ref_gpu) and exposed through a C ABI
// so the GPU tests can compare outputs and times on the same inputs.
//
// The FA2 kernel leaves its loop with a `break` before a __syncthreads when a
// KV tile starts past a query row, and returns early for rows past S_q
// (kernels/flash_attn.cu:94,134).  Both are uniform across a CTA -- and so
// harmless -- exactly when S_q is a multiple of the query tile Br (32 by
// default; Bc is 32 or 64): then every row of a tile breaks together and no
// row returns.  refgpu_flash_attn_bf16 refuses any other S_q.
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "flash_attn.cuh"
#include "matmul.cuh"

#define REF_EXPORT extern "C" __attribute__((visibility("default")))

namespace {
thread_local std::string g_err;

template <class F>
int guarded(F&& f) {
    try {
        f();
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        g_err = cudaGetErrorString(e);
        return -2;
    }
    return 0;
}
}  // namespace

REF_EXPORT const char* refgpu_last_error() { return g_err.c_str(); }

REF_EXPORT int refgpu_matmul_fp32(int bm, int bn, int bk, const float* A, const float* B,
                                  float* C, int M, int N, int K) {
    return guarded([&] {
        AMP::TileCfg cfg;
        cfg.BM = bm;
        cfg.BN = bn;
        cfg.BK = bk;
        AMP::launch_matmul(cfg, A, B, C, M, N, K, 0);
    });
}

REF_EXPORT int refgpu_matmul_bf16(const void* A, const void* B, float* C, int M, int N, int K) {
    return guarded([&] {
        AMP::launch_matmul_bf16(static_cast<const __nv_bfloat16*>(A),
                                static_cast<const __nv_bfloat16*>(B), C, M, N, K, 0);
    });
}

REF_EXPORT int refgpu_matmul_fp8e4m3(const void* A, const void* B, float* C, int M, int N, int K,
                                     float scale_a, float scale_b) {
    return guarded([&] {
        AMP::launch_matmul_fp8e4m3(static_cast<const AMP_fp8_e4m3*>(A),
                                   static_cast<const AMP_fp8_e4m3*>(B), C, M, N, K, scale_a,
                                   scale_b, 0);
    });
}

REF_EXPORT int refgpu_flash_attn_bf16(const void* Q, const void* K, const void* V, void* O,
                                      float* lse, int B, int Hq, int Hkv, int S_q, int S_kv,
                                      int head_dim, int causal, float scale) {
    AMP::AttnCfg cfg;
    if (S_q % cfg.Br != 0 || (causal && S_q != S_kv)) {
        g_err = "S_q must be a multiple of Br (and S_q == S_kv when causal)";
        return -3;
    }
    cfg.num_q_heads = Hq;
    cfg.num_kv_heads = Hkv;
    cfg.head_dim = head_dim;
    cfg.causal = causal != 0;
    cfg.scale = scale;
    return guarded([&] {
        AMP::launch_flash_attn_bf16(static_cast<const AMP_bf16*>(Q), static_cast<const AMP_bf16*>(K),
                                    static_cast<const AMP_bf16*>(V), static_cast<AMP_bf16*>(O), lse,
                                    B, S_q, S_kv, cfg, 0);
    });
}
