// gemm_fp32.cu -- fp32 GEMM C = A * B (row-major) behind AMP's plugin contract.
//
// Replaces matmul_fp32_kernel<BM,BN,BK> (kernels/matmul.cuh:24-58 of the
// reference: one thread per C element, two shared-memory tiles, FFMA) and its
// dispatcher launch_matmul (kernels/matmul.cu:24-35).  The reference's tile
// configs (16,16,16),(32,16,16),(32,32,16),(32,32,32) remain accepted names
// (the parity dump writes one entry per config) but the work is done by a
// register-tiled kernel: each thread owns an 8x8 (or 4x4) block of C, the
// k-loop reads two float4 of A^T and two float4 of B per k from
// double-buffered shared memory, and the next k-tile is fetched from global
// memory into registers while the current one is multiplied.
//
// Two accumulation modes, both in k order within a thread, on pairs of
// adjacent output columns:
//   * fast  (amp_gemm_fp32_dev): fp32 FFMA, one rounding per multiply-add, as
//     packed fma.rn.f32x2 (two lanes' worth of work per issue slot, which is
//     what bounds this kernel);
//   * exact (amp_gemm_fp32_exact_dev, the plugin amp_user_gemm_fp32 and the
//     tile-config launcher behind the parity dump): the product rounded to
//     fp32, then the sum rounded to fp32, k ascending from 0 -- the order and
//     rounding of AMP's cpu_reference_gemm (tests/amp_validate_kernel.cpp:20-28,
//     compiled without FMA contraction), so C is bit-identical to it and AMP's
//     validator reads max_rel_err = 0 at any size.  The fast mode's error
//     against that reference grows with K (7e-4 at 1024^3 on the validator's
//     [-10, 10] inputs, close to its 1e-3 bar).  Zero-padded k beyond K adds
//     +-0 to a sum that is never -0, so it leaves the exact result unchanged.
//
// This is the fp32 GEMM of the plugin contract.  A faster tensor-core form
// (three TF32 products of a hi/lo split, amp_gemm_fp32_3xtf32_dev in
// gemm_tc.cu) is opt-in only: its fp32 accumulation inside the tensor core
// loses more than AMP's validator allows on its own harness inputs.
#include "common.cuh"
#include "runtime.h"

namespace ampb {

namespace {

// Reads H consecutive floats at p and H at p + OFF into dst[0..2H) with the
// widest aligned shared-memory vector loads.
template <int H, int OFF>
__device__ __forceinline__ void load_halves(const float* p, float* dst) {
    if constexpr (H % 4 == 0) {
#pragma unroll
        for (int i = 0; i < H; i += 4) {
            float4 v0 = *reinterpret_cast<const float4*>(p + i);
            float4 v1 = *reinterpret_cast<const float4*>(p + OFF + i);
            dst[i] = v0.x; dst[i + 1] = v0.y; dst[i + 2] = v0.z; dst[i + 3] = v0.w;
            dst[H + i] = v1.x; dst[H + i + 1] = v1.y; dst[H + i + 2] = v1.z; dst[H + i + 3] = v1.w;
        }
    } else {
        static_assert(H % 2 == 0, "thread tile halves must be even");
#pragma unroll
        for (int i = 0; i < H; i += 2) {
            float2 v0 = *reinterpret_cast<const float2*>(p + i);
            float2 v1 = *reinterpret_cast<const float2*>(p + OFF + i);
            dst[i] = v0.x; dst[i + 1] = v0.y;
            dst[H + i] = v1.x; dst[H + i + 1] = v1.y;
        }
    }
}

// Packed fp32 pairs (sm_100: one instruction for two lanes).  The exact form
// uses mul.rn / add.rn, which are never contracted into an FMA.
__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void unpk2(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma_rn2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
// Exact step on a pair: each product rounded, then each sum, as scalar
// mul.rn / add.rn (never contracted).  A packed mul.rn.f32x2 + add.rn.f32x2
// pair was measured not to reproduce the separately rounded result, so the
// exact form stays on scalar instructions.
__device__ __forceinline__ uint64_t mul_add_rn2(uint64_t acc, uint64_t a, uint64_t b) {
    float c0, c1, a0, a1, b0, b1;
    unpk2(acc, c0, c1);
    unpk2(a, a0, a1);
    unpk2(b, b0, b1);
    return pk2(__fadd_rn(c0, __fmul_rn(a0, b0)), __fadd_rn(c1, __fmul_rn(a1, b1)));
}

template <int BM, int BN, int BK, int TM, int TN>
struct Cfg {
    static constexpr int kThreads = (BM / TM) * (BN / TN);
    static constexpr int kAPerThread = BM * BK / kThreads;  // A elements loaded per thread per tile
    static constexpr int kBPerThread = BK * BN / kThreads;
    static_assert(kAPerThread % 4 == 0 && kBPerThread % 4 == 0, "tile/threads mismatch");
};

// Row-major A [M,K], B [K,N], C [M,N].  `vec` = K%4==0 && N%4==0 && 16B-aligned bases.
template <int BM, int BN, int BK, int TM, int TN, bool kExact>
__global__ void __launch_bounds__(Cfg<BM, BN, BK, TM, TN>::kThreads)
    k_gemm_fp32(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C,
                int M, int N, int K, int vec) {
    using CF = Cfg<BM, BN, BK, TM, TN>;
    constexpr int T = CF::kThreads;
    constexpr int TX = BN / TN;  // threads along N
    __shared__ __align__(16) float As[2][BK][BM + 4];  // A^T tile (k-major), padded
    __shared__ __align__(16) float Bs[2][BK][BN];

    const int tid = threadIdx.x;
    const int tx = tid % TX, ty = tid / TX;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;

    // Each thread loads kAPerThread/4 float4 of A (rows of 4 consecutive k) and
    // kBPerThread/4 float4 of B (4 consecutive n) per k-tile.
    constexpr int AV = CF::kAPerThread / 4, BV = CF::kBPerThread / 4;
    float4 ra[AV], rb[BV];

    auto load_tile = [&](int k0) {
#pragma unroll
        for (int i = 0; i < AV; ++i) {
            int idx = tid + i * T;            // over BM * (BK/4)
            int r = idx / (BK / 4), c4 = (idx % (BK / 4)) * 4;
            int gr = m0 + r, gc = k0 + c4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (gr < M) {
                const float* p = A + (int64_t)gr * K + gc;
                if (vec) {
                    if (gc < K) v = *reinterpret_cast<const float4*>(p);
                } else {
                    if (gc + 0 < K) v.x = p[0];
                    if (gc + 1 < K) v.y = p[1];
                    if (gc + 2 < K) v.z = p[2];
                    if (gc + 3 < K) v.w = p[3];
                }
            }
            ra[i] = v;
        }
#pragma unroll
        for (int i = 0; i < BV; ++i) {
            int idx = tid + i * T;            // over BK * (BN/4)
            int r = idx / (BN / 4), c4 = (idx % (BN / 4)) * 4;
            int gr = k0 + r, gc = n0 + c4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (gr < K) {
                const float* p = B + (int64_t)gr * N + gc;
                if (vec) {
                    if (gc < N) v = *reinterpret_cast<const float4*>(p);
                } else {
                    if (gc + 0 < N) v.x = p[0];
                    if (gc + 1 < N) v.y = p[1];
                    if (gc + 2 < N) v.z = p[2];
                    if (gc + 3 < N) v.w = p[3];
                }
            }
            rb[i] = v;
        }
    };
    auto store_tile = [&](int buf) {
#pragma unroll
        for (int i = 0; i < AV; ++i) {
            int idx = tid + i * T;
            int r = idx / (BK / 4), c4 = (idx % (BK / 4)) * 4;
            As[buf][c4 + 0][r] = ra[i].x;
            As[buf][c4 + 1][r] = ra[i].y;
            As[buf][c4 + 2][r] = ra[i].z;
            As[buf][c4 + 3][r] = ra[i].w;
        }
#pragma unroll
        for (int i = 0; i < BV; ++i) {
            int idx = tid + i * T;
            int r = idx / (BN / 4), c4 = (idx % (BN / 4)) * 4;
            *reinterpret_cast<float4*>(&Bs[buf][r][c4]) = rb[i];
        }
    };

    // accumulators as packed pairs of adjacent columns: acc2[i][jp] = (C[i][2jp], C[i][2jp+1])
    static_assert(TN % 2 == 0, "column pairs");
    uint64_t acc2[TM][TN / 2];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN / 2; ++j) acc2[i][j] = 0ull;

    const int ktiles = (K + BK - 1) / BK;
    if (ktiles > 0) {
        load_tile(0);
        store_tile(0);
    }
    __syncthreads();
    // Thread rows: {ty*TM/2 + i} and {BM/2 + ty*TM/2 + i}; columns likewise.
    constexpr int HM = TM / 2, HN = TN / 2;
    for (int kt = 0; kt < ktiles; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < ktiles) load_tile((kt + 1) * BK);
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            float a[TM], b[TN];
            load_halves<HM, BM / 2>(&As[buf][k][ty * HM], a);
            load_halves<HN, BN / 2>(&Bs[buf][k][tx * HN], b);
            uint64_t b2[TN / 2];
#pragma unroll
            for (int j = 0; j < TN / 2; ++j) b2[j] = pk2(b[2 * j], b[2 * j + 1]);
#pragma unroll
            for (int i = 0; i < TM; ++i) {
                const uint64_t a2 = pk2(a[i], a[i]);
#pragma unroll
                for (int j = 0; j < TN / 2; ++j) {
                    if constexpr (kExact)
                        acc2[i][j] = mul_add_rn2(acc2[i][j], a2, b2[j]);
                    else
                        acc2[i][j] = fma_rn2(a2, b2[j], acc2[i][j]);
                }
            }
        }
        if (kt + 1 < ktiles) store_tile(buf ^ 1);
        __syncthreads();
    }

    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN / 2; ++j) unpk2(acc2[i][j], acc[i][2 * j], acc[i][2 * j + 1]);
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int r = m0 + (i < HM ? ty * HM + i : BM / 2 + ty * HM + (i - HM));
        if (r >= M) continue;
#pragma unroll
        for (int hj = 0; hj < 2; ++hj) {
            const int c = n0 + hj * (BN / 2) + tx * HN;
            float* p = C + (int64_t)r * N + c;
            bool done = false;
            if constexpr (HN % 4 == 0) {
                if (vec && c + HN <= N) {
#pragma unroll
                    for (int j = 0; j < HN; j += 4)
                        *reinterpret_cast<float4*>(p + j) =
                            make_float4(acc[i][hj * HN + j], acc[i][hj * HN + j + 1],
                                        acc[i][hj * HN + j + 2], acc[i][hj * HN + j + 3]);
                    done = true;
                }
            }
            if (!done) {
#pragma unroll
                for (int j = 0; j < HN; ++j)
                    if (c + j < N) p[j] = acc[i][hj * HN + j];
            }
        }
    }
}

template <int BM, int BN, int BK, int TM, int TN, bool kExact>
int launch(const float* A, const float* B, float* C, int M, int N, int K, int vec,
           cudaStream_t st) {
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    k_gemm_fp32<BM, BN, BK, TM, TN, kExact>
        <<<grid, Cfg<BM, BN, BK, TM, TN>::kThreads, 0, st>>>(A, B, C, M, N, K, vec);
    AMPB_CHECK_LAUNCH("k_gemm_fp32");
    return AMP_OK;
}

}  // namespace

int gemm_fp32_dev(const float* A, const float* B, float* C, int M, int N, int K, bool exact,
                  cudaStream_t st) {
    AMPB_REQUIRE(M >= 0 && N >= 0 && K >= 0, AMP_ERR_INVALID, "negative GEMM size %d x %d x %d",
                 M, N, K);
    if (M == 0 || N == 0) return AMP_OK;
    AMPB_REQUIRE(A && B && C, AMP_ERR_INVALID, "NULL operand");
    const int vec = (K % 4 == 0) && (N % 4 == 0) && aligned16(A) && aligned16(B) && aligned16(C);
    // Big tiles once they fill the machine twice over; 64x64 tiles otherwise.
    const int64_t big_tiles = (int64_t)((M + 127) / 128) * ((N + 127) / 128);
    if (big_tiles >= 2 * sm_count())
        return exact ? launch<128, 128, 8, 8, 8, true>(A, B, C, M, N, K, vec, st)
                     : launch<128, 128, 8, 8, 8, false>(A, B, C, M, N, K, vec, st);
    return exact ? launch<64, 64, 16, 4, 4, true>(A, B, C, M, N, K, vec, st)
                 : launch<64, 64, 16, 4, 4, false>(A, B, C, M, N, K, vec, st);
}

bool fp32_tile_known(int bm, int bn, int bk) {
    // The tile configs AMP's dispatcher accepts (kernels/matmul.cu:29-32), plus
    // (0,0,0), the "user plugin" entry of the dump format.
    const int known[5][3] = {{16, 16, 16}, {32, 16, 16}, {32, 32, 16}, {32, 32, 32}, {0, 0, 0}};
    for (auto& t : known)
        if (t[0] == bm && t[1] == bn && t[2] == bk) return true;
    return false;
}

}  // namespace ampb

using namespace ampb;

extern "C" {

int amp_gemm_fp32_dev(const float* A, const float* B, float* C, int M, int N, int K,
                      void* stream) {
    return gemm_fp32_dev(A, B, C, M, N, K, false, as_stream(stream));
}

int amp_gemm_fp32_exact_dev(const float* A, const float* B, float* C, int M, int N, int K,
                            void* stream) {
    return gemm_fp32_dev(A, B, C, M, N, K, true, as_stream(stream));
}

int amp_gemm_fp32_tile_dev(int bm, int bn, int bk, const float* A, const float* B, float* C,
                           int M, int N, int K, void* stream) {
    AMPB_REQUIRE(fp32_tile_known(bm, bn, bk), AMP_ERR_INVALID,
                 "unknown FP32 tile cfg (%d,%d,%d)", bm, bn, bk);
    return gemm_fp32_dev(A, B, C, M, N, K, true, as_stream(stream));
}

// AMP's plugin contract (include/amp_plugin.h): host buffers in and out, all
// device work done and synchronised before returning.
int amp_user_gemm_fp32(const float* hA, const float* hB, float* hC, int M, int N, int K) {
    AMPB_REQUIRE(M >= 0 && N >= 0 && K >= 0, AMP_ERR_INVALID, "negative GEMM size");
    AMPB_REQUIRE((M == 0 || N == 0) || (hA && hB && hC), AMP_ERR_INVALID, "NULL operand");
    if (M == 0 || N == 0) return AMP_OK;
    const size_t a = (size_t)M * K * 4, b = (size_t)K * N * 4, c = (size_t)M * N * 4;
    void *dA, *dB, *dC;
    int rc;
    if ((rc = staging_get(0, a, &dA))) return rc;
    if ((rc = staging_get(1, b, &dB))) return rc;
    if ((rc = staging_get(2, c, &dC))) return rc;
    cudaStream_t st = 0;
    if (a) AMPB_CHECK_CUDA(cudaMemcpyAsync(dA, hA, a, cudaMemcpyHostToDevice, st));
    if (b) AMPB_CHECK_CUDA(cudaMemcpyAsync(dB, hB, b, cudaMemcpyHostToDevice, st));
    if ((rc = gemm_fp32_dev((const float*)dA, (const float*)dB, (float*)dC, M, N, K, true, st)))
        return rc;
    AMPB_CHECK_CUDA(cudaMemcpyAsync(hC, dC, c, cudaMemcpyDeviceToHost, st));
    AMPB_CHECK_CUDA(cudaStreamSynchronize(st));
    return staging_end_of_call();
}

}  // extern "C"
