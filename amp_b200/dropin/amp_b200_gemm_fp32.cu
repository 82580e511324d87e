// amp_b200_gemm_fp32.cu -- the fp32 GEMM as a kernel file for AMP's one-command
// checker, scripts/amp_check.sh.
//
//   bash scripts/amp_check.sh amp_b200/dropin/amp_b200_gemm_fp32.cu amp_b200_gemm_fp32 [M N K]
//
// amp_check.sh (scripts/amp_check.sh:59-106) #includes this file into a
// generated wrapper after <cuda_runtime.h>, compiles it with a bare
// `nvcc -shared -Xcompiler -fPIC` (no -arch: the code is compute_52 PTX that
// the driver compiles for the B200 when it loads), and launches
//
//   amp_b200_gemm_fp32<<<dim3((N+15)/16, (M+15)/16), dim3(16, 16)>>>(dA, dB, dC, M, N, K)
//
// with no dynamic shared memory and no stream, then hands the result to AMP's
// validator (tests/amp_validate_kernel.cpp), which compares it with
// cpu_reference_gemm (amp_validate_kernel.cpp:20-28) under a 1e-3 bar.  So
// this file is self-contained and uses nothing newer than sm_52.
//
// Results: every element is accumulated exactly as cpu_reference_gemm does
// it -- acc = 0; for k = 0 .. K-1: acc = acc + A[i][k] * B[k][j], the product
// rounded to fp32 and then the sum rounded to fp32 (no fused multiply-add,
// which the compiler would otherwise form) -- so C is bit-identical to the
// CPU reference and the validator reports max_rel_err = 0 at any size.
//
// Blocking: the launch gives one 256-thread CTA per 16 x 16 output tile.  A
// CTA that computes only 256 outputs reads two shared-memory values per
// multiply-add, so the kernel instead hands each CTA a larger tile (64 x 64,
// 16 outputs per thread, when there are enough of them to cover every SM;
// else 32 x 32; else 16 x 16) and the CTAs beyond the tile count return at
// once.  A grid-stride loop over tiles keeps it correct for any grid, too.
// Tiles of A and B pass through double-buffered shared memory (16 KiB of
// static shared memory), the next k-slab is fetched into registers while the
// current one is multiplied, and one __syncthreads separates the k-steps.
#ifndef AMP_B200_GEMM_FP32_DROPIN_CU
#define AMP_B200_GEMM_FP32_DROPIN_CU

namespace amp_b200_dropin {

constexpr int kThreads = 256;  // the (16, 16) block amp_check.sh launches
constexpr int kBK = 16;        // k-slab depth
constexpr int kMaxT = 64;      // largest tile edge
// one buffer: A slab [kBK][T + 1] (padded: the transposing stores spread over
// the banks) + B slab [kBK][T]
constexpr int kBufFloats = kBK * (kMaxT + 1) + kBK * kMaxT;

// this thread's index in its 256-thread block, whatever the block's shape
__device__ __forceinline__ int flat_tid() {
    return (int)(threadIdx.x + blockDim.x * (threadIdx.y + blockDim.y * threadIdx.z));
}

__device__ __forceinline__ unsigned sm_count() {
    unsigned n;
    asm("mov.u32 %0, %%nsmid;" : "=r"(n));
    return n;
}

template <int T>
__device__ __forceinline__ void tile_gemm(const float* __restrict__ A, const float* __restrict__ B,
                                          float* __restrict__ C, int M, int N, int K, int tile,
                                          int tiles_n, float* smem) {
    constexpr int R = T / 16;                   // outputs per thread along each edge
    constexpr int kLoadA = T * kBK / kThreads;  // A elements a thread fetches per slab
    constexpr int kLoadB = kBK * T / kThreads;  // B elements a thread fetches per slab
    constexpr int kLdA = T + 1;
    const int tid = flat_tid();
    const int tx = tid & 15, ty = tid >> 4;
    const int m0 = (tile / tiles_n) * T, n0 = (tile % tiles_n) * T;

    // buffer b: A slab at smem + b * kBufFloats, B slab kBK * kLdA floats after it
    auto a_slab = [&](int b) { return smem + b * kBufFloats; };
    auto b_slab = [&](int b) { return smem + b * kBufFloats + kBK * kLdA; };

    float acc[R][R];
#pragma unroll
    for (int i = 0; i < R; ++i)
#pragma unroll
        for (int j = 0; j < R; ++j) acc[i][j] = 0.0f;

    float ra[kLoadA], rb[kLoadB];
    // slab k0 into registers; elements outside A or B read as 0 and are never summed
    auto fetch = [&](int k0) {
#pragma unroll
        for (int l = 0; l < kLoadA; ++l) {
            const int e = tid + l * kThreads, r = e / kBK, k = e % kBK;
            const int gm = m0 + r, gk = k0 + k;
            ra[l] = (gm < M && gk < K) ? A[(size_t)gm * K + gk] : 0.0f;
        }
#pragma unroll
        for (int l = 0; l < kLoadB; ++l) {
            const int e = tid + l * kThreads, k = e / T, c = e % T;
            const int gk = k0 + k, gn = n0 + c;
            rb[l] = (gk < K && gn < N) ? B[(size_t)gk * N + gn] : 0.0f;
        }
    };
    auto stash = [&](int buf) {
#pragma unroll
        for (int l = 0; l < kLoadA; ++l) {
            const int e = tid + l * kThreads;
            a_slab(buf)[(e % kBK) * kLdA + e / kBK] = ra[l];
        }
#pragma unroll
        for (int l = 0; l < kLoadB; ++l) {
            const int e = tid + l * kThreads;
            b_slab(buf)[(e / T) * T + e % T] = rb[l];
        }
    };
    // one k-step: product rounded, then sum rounded, k ascending (the CPU's order)
    auto step = [&](const float* as, const float* bs) {
        float a[R], b[R];
#pragma unroll
        for (int i = 0; i < R; ++i) a[i] = as[ty + 16 * i];
#pragma unroll
        for (int j = 0; j < R; ++j) b[j] = bs[tx + 16 * j];
#pragma unroll
        for (int i = 0; i < R; ++i)
#pragma unroll
            for (int j = 0; j < R; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], b[j]));
    };

    const int slabs = (K + kBK - 1) / kBK;
    fetch(0);
    stash(0);
    __syncthreads();
    for (int s = 0; s < slabs; ++s) {
        const int cur = s & 1;
        if (s + 1 < slabs) fetch((s + 1) * kBK);  // global loads in flight during the math
        const int kn = K - s * kBK;               // k-steps in this slab (uniform)
        const float* as = a_slab(cur);
        const float* bs = b_slab(cur);
        if (kn >= kBK) {
#pragma unroll
            for (int kk = 0; kk < kBK; ++kk) step(as + kk * kLdA, bs + kk * T);
        } else {
            for (int kk = 0; kk < kn; ++kk) step(as + kk * kLdA, bs + kk * T);
        }
        if (s + 1 < slabs) stash(cur ^ 1);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < R; ++i) {
        const int gm = m0 + ty + 16 * i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < R; ++j) {
            const int gn = n0 + tx + 16 * j;
            if (gn < N) C[(size_t)gm * N + gn] = acc[i][j];
        }
    }
}

}  // namespace amp_b200_dropin

// C[M,N] = A[M,K] * B[K,N], row-major fp32 device buffers; 256 threads per block.
__global__ void __launch_bounds__(256)
    amp_b200_gemm_fp32(const float* A, const float* B, float* C, int M, int N, int K) {
    using namespace amp_b200_dropin;
    __shared__ float smem[2 * kBufFloats];
    if (blockDim.x * blockDim.y * blockDim.z != kThreads || M <= 0 || N <= 0) return;
    if (K <= 0) {  // an empty sum: C = 0
        const int ctas = gridDim.x * gridDim.y * gridDim.z;
        const int cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
        const int tid = flat_tid();
        for (size_t e = (size_t)cta * kThreads + tid; e < (size_t)M * N;
             e += (size_t)ctas * kThreads)
            C[e] = 0.0f;
        return;
    }
    const int ctas = gridDim.x * gridDim.y * gridDim.z;
    const int cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    const int nsm = (int)sm_count();
    const int t64n = (N + 63) / 64, t64 = ((M + 63) / 64) * t64n;
    const int t32n = (N + 31) / 32, t32 = ((M + 31) / 32) * t32n;
    const int t16n = (N + 15) / 16, t16 = ((M + 15) / 16) * t16n;
    if (t64 >= nsm) {
        for (int t = cta; t < t64; t += ctas) tile_gemm<64>(A, B, C, M, N, K, t, t64n, smem);
    } else if (t32 >= nsm) {
        for (int t = cta; t < t32; t += ctas) tile_gemm<32>(A, B, C, M, N, K, t, t32n, smem);
    } else {
        for (int t = cta; t < t16; t += ctas) tile_gemm<16>(A, B, C, M, N, K, t, t16n, smem);
    }
}

#endif  // AMP_B200_GEMM_FP32_DROPIN_CU
