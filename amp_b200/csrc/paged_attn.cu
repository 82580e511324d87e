// paged_attn.cu -- GQA attention decode over a paged KV cache.
//
// The reference keeps a per-sequence block table (Sequence::kv_page_ids,
// include/scheduler.hpp:61) of 16-token pages (SchedulerConfig::
// kv_page_size_tokens, include/scheduler.hpp:88; pages_needed_for,
// src/scheduler.cpp:64-67) but no kernel consumes it: its FlashAttention-2
// takes contiguous [B,H,S,D] tensors only (kernels/flash_attn.cuh:47-58).
// This file is the decode kernel for that format.
//
// Layout (defined here; AMP leaves page contents unspecified):
//   k_pool, v_pool  [num_pages][Hkv][16][D] bf16 -- one head's page is 4 KiB
//                   contiguous (D = 128)
//   block_table     int32 [B][max_pages_per_seq]; token t of sequence b is
//                   slot t % 16 of page block_table[b][t / 16]
//   ctx_lens        int32 [B]
//   q, out          [B][Hq][D] bf16 (one new token per sequence); lse [B][Hq]
//
// Decode is HBM-bound (4 KiB of K+V per context token for Hkv = 8, D = 128).
// One CTA per (chunk of 32 pages, kv head, sequence), 160 threads:
//   warp 4     producer: TMA (4-D page-gather map, 128-byte swizzle) of each
//              page's K and V blocks (2 x 4 KiB) into an 8-stage shared-memory
//              ring, so 64 KiB per CTA are in flight ahead of the math.
//   warps 0-3  consumers; warp w takes pages w, w+4, ... of the chunk.  Per
//              page, on the tensor cores (mma.sync m16n8k16, bf16 -> fp32):
//              S^T[16 tokens x 8 heads] = K Q^T (K by ldmatrix, Q held in
//              registers as B fragments; the GQA group's G <= 8 query heads
//              fill the 8 columns), online softmax per head down the token
//              rows (quad shuffles), P^T turned into B fragments by movmatrix,
//              O^T[128 x 8] += V^T P^T (V by ldmatrix.trans).
//   Warps merge in shared memory; chunks merge in k_paged_combine through
//   their log-sum-exp.
// A page id outside [0, num_pages) is never loaded: it is flagged in the device
// status word (AMP_DEV_ERR_BAD_PAGE) and its tokens are treated as masked.
// Slots past the context in the last page may hold anything: their scores are
// masked and their V rows zeroed in shared memory before the PV product.
#include <cuda.h>

#include <atomic>
#include <cmath>
#include <vector>

#include "common.cuh"
#include "runtime.h"
#include "tc_common.cuh"

namespace ampb {

int fa_make_tmap_pool(CUtensorMap* m, const void* base, int64_t d, int64_t hkv, int64_t pages);

namespace {

constexpr int kPage = 16;
constexpr int kChunkPages = 32;     // 512 tokens per split
constexpr int kCWarps = 4;          // consumer warps
constexpr int kThreads = (kCWarps + 1) * 32;
constexpr int kStages = 8;
constexpr int kSlab = kPage * 128;           // 16 rows x 128 B (64 bf16 of D), swizzled
constexpr int kStageBytes = 4 * kSlab;       // K d0-63 | K d64-127 | V d0-63 | V d64-127
constexpr int kDecodeSmem = kStages * kStageBytes + 1024 + 256;

struct DecodeParams {
    const __nv_bfloat16* q;
    const int* block_table;
    const int* ctx_lens;
    float* part_o;     // [B][Hq][max_chunks][D]
    float* part_ml;    // [B][Hq][max_chunks][2]  (m in log2 units, l)
    __nv_bfloat16* out;
    float* lse;
    int B, Hq, Hkv, num_pages, max_pages, max_chunks;
    float scale_log2;
    int* status;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// byte offset of (row, 16-byte chunk) in a [rows x 128 B] slab written by TMA with
// the 128-byte swizzle
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
    return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

template <int G>
__global__ void __launch_bounds__(kThreads) k_paged_decode(const __grid_constant__ CUtensorMap tmK,
                                                           const __grid_constant__ CUtensorMap tmV,
                                                           const DecodeParams p) {
    static_assert(G >= 1 && G <= 8, "one n8 tile holds the GQA group");
    constexpr int D = 128;
    const int chunk = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ctx = p.ctx_lens[b];
    const int n_pages = (ctx + kPage - 1) / kPage;
    const int pg0 = chunk * kChunkPages;
    if (pg0 >= n_pages || ctx <= 0) return;     // the combine kernel knows the chunk count
    const int np = min(n_pages - pg0, kChunkPages);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    int* page_ok = reinterpret_cast<int*>(empty + kStages);
    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        fence_barrier_init();
    }
    __syncthreads();

    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};
    float o[8][4];
#pragma unroll
    for (int mt = 0; mt < 8; ++mt)
#pragma unroll
        for (int j = 0; j < 4; ++j) o[mt][j] = 0.0f;

    if (warp == kCWarps) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            const int* bt = p.block_table + (int64_t)b * p.max_pages;
            int k = 0;
            for (; k < np; ++k) {
                const int s = k % kStages;
                if (!mbar_wait(&empty[s], ((k / kStages) & 1) ^ 1, p.status)) break;
                const int page = bt[pg0 + k];
                const bool ok = page >= 0 && page < p.num_pages;
                page_ok[s] = ok;
                if (ok) {
                    uint8_t* st = ring + s * kStageBytes;
                    mbar_arrive_expect_tx(&full[s], kStageBytes);
                    tma_load_4d(st, &tmK, &full[s], 0, 0, hk, page);
                    tma_load_4d(st + kSlab, &tmK, &full[s], 64, 0, hk, page);
                    tma_load_4d(st + 2 * kSlab, &tmV, &full[s], 0, 0, hk, page);
                    tma_load_4d(st + 3 * kSlab, &tmV, &full[s], 64, 0, hk, page);
                } else {
                    atomicExch(p.status, AMP_DEV_ERR_BAD_PAGE);
                    mbar_arrive(&full[s]);
                }
            }
            // every copy issued lands before the shared memory is reused or released
            for (int kk = max(0, k - kStages); kk < k; ++kk)
                mbar_wait(&full[kk % kStages], (kk / kStages) & 1, p.status);
        }
    } else {
        // ------------------------------------------------------------ consumers
        // Q^T as B fragments: lane holds head n = lane/4 at d = 16kk + 2(lane%4) (+8)
        const int n = lane >> 2, kq = 2 * (lane & 3);
        uint32_t qb[8][2];
        {
            const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
                p.q + ((int64_t)b * p.Hq + hk * G + (n < G ? n : 0)) * D);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                qb[kk][0] = n < G ? qrow[(16 * kk + kq) >> 1] : 0u;
                qb[kk][1] = n < G ? qrow[(16 * kk + 8 + kq) >> 1] : 0u;
            }
        }
        const float c = p.scale_log2;
        const int r = lane >> 2;              // token row of this lane's C elements (and r + 8)
        const int mi = lane >> 3, r8 = lane & 7;   // ldmatrix: matrix / row this lane addresses
        for (int k = warp; k < np; k += kCWarps) {
            const int s = k % kStages;
            if (!mbar_wait_warp(&full[s], (k / kStages) & 1, p.status)) break;
            const int vt = page_ok[s] ? min(kPage, ctx - (pg0 + k) * kPage) : 0;
            uint8_t* st = ring + s * kStageBytes;
            if (vt > 0) {
                if (vt < kPage) {
                    // zero V rows of the slots past the context (whole 128-byte rows,
                    // so the swizzle does not matter)
                    for (int i = lane; i < (kPage - vt) * 2 * 8; i += 32) {
                        const int row = vt + (i >> 4), sl = (i >> 3) & 1, ch = i & 7;
                        *reinterpret_cast<uint4*>(st + (2 + sl) * kSlab + row * 128 + ch * 16) =
                            make_uint4(0u, 0u, 0u, 0u);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                }
                // S^T = K Q^T: 8 k-steps of 16 along D
                float sc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                const uint32_t kbase = smem_u32(st);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const int row = r8 + 8 * (mi & 1);
                    const int chunk16 = 2 * (kk & 3) + (mi >> 1);
                    uint32_t a[4];
                    ldsm_x4(kbase + (kk >> 2) * kSlab + swz(row, chunk16), a);
                    mma16816(sc, a, qb[kk][0], qb[kk][1]);
                }
                // online softmax per head (column) down the 16 token rows
                float x[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int tok = r + 8 * (j >> 1);
                    x[j] = tok < vt ? sc[j] * c : -INFINITY;
                }
                float mx0 = fmaxf(x[0], x[2]), mx1 = fmaxf(x[1], x[3]);
#pragma unroll
                for (int off = 4; off < 32; off <<= 1) {
                    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
                }
                const float mn0 = fmaxf(m[0], mx0), mn1 = fmaxf(m[1], mx1);   // finite: token 0 valid
                const float al0 = ex2_approx(m[0] - mn0), al1 = ex2_approx(m[1] - mn1);
                const float p0 = ex2_approx(x[0] - mn0), p1 = ex2_approx(x[1] - mn1);
                const float p2 = ex2_approx(x[2] - mn0), p3 = ex2_approx(x[3] - mn1);
                float rs0 = p0 + p2, rs1 = p1 + p3;
#pragma unroll
                for (int off = 4; off < 32; off <<= 1) {
                    rs0 += __shfl_xor_sync(0xffffffffu, rs0, off);
                    rs1 += __shfl_xor_sync(0xffffffffu, rs1, off);
                }
                l[0] = l[0] * al0 + rs0;
                l[1] = l[1] * al1 + rs1;
                m[0] = mn0;
                m[1] = mn1;
                if (__any_sync(0xffffffffu, al0 != 1.0f || al1 != 1.0f)) {
#pragma unroll
                    for (int mt = 0; mt < 8; ++mt) {
                        o[mt][0] *= al0;
                        o[mt][1] *= al1;
                        o[mt][2] *= al0;
                        o[mt][3] *= al1;
                    }
                }
                // P^T as B fragments (tokens x heads), via an in-register transpose
                const uint32_t b01 = movm_t(f32x2_to_bf16x2(p0, p1));
                const uint32_t b23 = movm_t(f32x2_to_bf16x2(p2, p3));
                // O^T[d][head] += V^T P^T: 8 m-tiles of 16 along D
                const uint32_t vbase = kbase + 2 * kSlab;
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) {
                    const int tok = r8 + 8 * (mi >> 1);
                    const int dch = 2 * mt + (mi & 1);          // 16-byte chunk along D
                    uint32_t a[4];
                    ldsm_x4_t(vbase + (dch >> 3) * kSlab + swz(tok, dch & 7), a);
                    mma16816(o[mt], a, b01, b23);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
    }

    // merge the consumer warps (the ring is free: every copy has landed)
    __syncthreads();
    float* o_s = reinterpret_cast<float*>(ring);     // [kCWarps][8][D]
    float* m_s = o_s + kCWarps * 8 * D;              // [kCWarps][8]
    float* l_s = m_s + kCWarps * 8;                  // [kCWarps][8]
    if (warp < kCWarps) {
        const int h0 = 2 * (lane & 3), r = lane >> 2;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt)
#pragma unroll
            for (int j = 0; j < 4; ++j)
                o_s[(warp * 8 + h0 + (j & 1)) * D + 16 * mt + r + 8 * (j >> 1)] = o[mt][j];
        if (r == 0) {
            m_s[warp * 8 + h0] = m[0];
            m_s[warp * 8 + h0 + 1] = m[1];
            l_s[warp * 8 + h0] = l[0];
            l_s[warp * 8 + h0 + 1] = l[1];
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
        const int g = i / D, d = i % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kCWarps; ++w) M = fmaxf(M, m_s[w * 8 + g]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < kCWarps; ++w) {
            const float mw = m_s[w * 8 + g];
            const float a = (mw == -INFINITY) ? 0.0f : ex2_approx(mw - M);
            L += a * l_s[w * 8 + g];
            O += a * o_s[(w * 8 + g) * D + d];
        }
        const int64_t row = ((int64_t)b * p.Hq + hk * G + g) * p.max_chunks + chunk;
        p.part_o[row * D + d] = O;
        if (d == 0) {
            p.part_ml[row * 2] = M;
            p.part_ml[row * 2 + 1] = L;
        }
    }
}

template <int D>
__global__ void __launch_bounds__(D) k_paged_combine(const DecodeParams p) {
    const int bh = blockIdx.x;
    const int b = bh / p.Hq;
    const int d = threadIdx.x;
    const int ctx = p.ctx_lens[b];
    const int n_chunks = ctx > 0 ? ((ctx + kPage - 1) / kPage + kChunkPages - 1) / kChunkPages : 0;
    const int64_t row0 = (int64_t)bh * p.max_chunks;
    float M = -INFINITY;
    for (int c = 0; c < n_chunks; ++c) M = fmaxf(M, p.part_ml[(row0 + c) * 2]);
    float L = 0.0f, O = 0.0f;
    for (int c = 0; c < n_chunks; ++c) {
        const float mc = p.part_ml[(row0 + c) * 2];
        const float a = (mc == -INFINITY) ? 0.0f : ex2_approx(mc - M);
        L += a * p.part_ml[(row0 + c) * 2 + 1];
        O += a * p.part_o[(row0 + c) * D + d];
    }
    p.out[(int64_t)bh * D + d] = __float2bfloat16_rn(L > 0.0f ? O / L : 0.0f);
    if (d == 0 && p.lse) {
        float lg;
        asm("lg2.approx.f32 %0, %1;" : "=f"(lg) : "f"(L));
        p.lse[bh] = L > 0.0f ? (M + lg) * 0.69314718055994531f : -INFINITY;
    }
}

size_t decode_ws_bytes(int B, int Hq, int D, int max_ctx) {
    const int64_t max_chunks = ((int64_t)(max_ctx + kPage - 1) / kPage + kChunkPages - 1) / kChunkPages;
    const int64_t rows = (int64_t)B * Hq * (max_chunks > 0 ? max_chunks : 1);
    return (size_t)(rows * D * 4 + rows * 2 * 4 + 256);
}

}  // namespace

int paged_decode_dev(const void* q, const void* k_pool, const void* v_pool, const int* block_table,
                     const int* ctx_lens, void* out, float* lse, int B, int Hq, int Hkv, int D,
                     int num_pages, int max_pages, int max_ctx, float scale, void* ws,
                     size_t ws_bytes, cudaStream_t st) {
    AMPB_REQUIRE(B > 0 && Hq > 0 && Hkv > 0 && num_pages > 0 && max_pages > 0 && max_ctx > 0,
                 AMP_ERR_INVALID, "paged decode sizes must be positive");
    AMPB_REQUIRE(Hq % Hkv == 0, AMP_ERR_INVALID, "Hq (%d) must be a multiple of Hkv (%d)", Hq, Hkv);
    AMPB_REQUIRE(D == 128, AMP_ERR_UNSUPPORTED, "paged decode supports head_dim 128 (got %d)", D);
    AMPB_REQUIRE((int64_t)max_ctx <= (int64_t)max_pages * kPage, AMP_ERR_INVALID,
                 "max_context_len %d exceeds the block table's %d pages", max_ctx, max_pages);
    AMPB_REQUIRE(q && k_pool && v_pool && block_table && ctx_lens && out && ws, AMP_ERR_INVALID,
                 "NULL argument");
    AMPB_REQUIRE(aligned16(q) && aligned16(k_pool) && aligned16(v_pool), AMP_ERR_INVALID,
                 "q and the pools must be 16-byte aligned");
    const size_t need = decode_ws_bytes(B, Hq, D, max_ctx);
    AMPB_REQUIRE(ws_bytes >= need, AMP_ERR_INVALID, "workspace too small: %zu < %zu", ws_bytes, need);
    AMPB_REQUIRE(B <= 65535 && Hkv <= 65535, AMP_ERR_UNSUPPORTED, "grid limits exceeded");
    int* status = nullptr;
    int rc = device_status(&status);
    if (rc) return rc;
    CUtensorMap tmK, tmV;
    if ((rc = fa_make_tmap_pool(&tmK, k_pool, D, Hkv, num_pages))) return rc;
    if ((rc = fa_make_tmap_pool(&tmV, v_pool, D, Hkv, num_pages))) return rc;
    if (!(scale > 0.0f)) scale = 1.0f / sqrtf((float)D);
    DecodeParams p;
    p.q = static_cast<const __nv_bfloat16*>(q);
    p.block_table = block_table;
    p.ctx_lens = ctx_lens;
    p.max_chunks = ((max_ctx + kPage - 1) / kPage + kChunkPages - 1) / kChunkPages;
    p.part_o = static_cast<float*>(ws);
    p.part_ml = p.part_o + (int64_t)B * Hq * p.max_chunks * D;
    p.out = static_cast<__nv_bfloat16*>(out);
    p.lse = lse;
    p.B = B;
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.num_pages = num_pages;
    p.max_pages = max_pages;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.status = status;
    dim3 grid(p.max_chunks, Hkv, B);
    auto go = [&](auto kern, std::atomic<uint32_t>& attr_set) {
        int dev = 0;
        AMPB_CHECK_CUDA(cudaGetDevice(&dev));
        const uint32_t bit = 1u << (dev & 31);
        if (!(attr_set.load() & bit)) {
            AMPB_CHECK_CUDA(cudaFuncSetAttribute(
                kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kDecodeSmem));
            attr_set.fetch_or(bit);
        }
        kern<<<grid, kThreads, kDecodeSmem, st>>>(tmK, tmV, p);
        return AMP_OK;
    };
    static std::atomic<uint32_t> attr1{0}, attr2{0}, attr4{0}, attr8{0};
    switch (Hq / Hkv) {
        case 1: rc = go(k_paged_decode<1>, attr1); break;
        case 2: rc = go(k_paged_decode<2>, attr2); break;
        case 4: rc = go(k_paged_decode<4>, attr4); break;
        case 8: rc = go(k_paged_decode<8>, attr8); break;
        default:
            set_error(AMP_ERR_UNSUPPORTED, "GQA group size %d not supported (1, 2, 4, 8)", Hq / Hkv);
            return AMP_ERR_UNSUPPORTED;
    }
    if (rc) return rc;
    AMPB_CHECK_LAUNCH("k_paged_decode");
    k_paged_combine<128><<<B * Hq, 128, 0, st>>>(p);
    AMPB_CHECK_LAUNCH("k_paged_combine");
    return AMP_OK;
}

}  // namespace ampb

using namespace ampb;

extern "C" {

size_t amp_paged_decode_workspace_bytes(int B, int Hq, int head_dim, int max_context_len) {
    return decode_ws_bytes(B, Hq, head_dim, max_context_len);
}

int amp_paged_attn_decode_bf16_dev(const void* q, const void* k_pool, const void* v_pool,
                                   const int32_t* block_table, const int32_t* ctx_lens, void* out,
                                   float* lse, int B, int Hq, int Hkv, int head_dim, int num_pages,
                                   int max_pages_per_seq, int max_context_len, float scale,
                                   void* workspace, size_t workspace_bytes, void* stream) {
    return paged_decode_dev(q, k_pool, v_pool, block_table, ctx_lens, out, lse, B, Hq, Hkv,
                            head_dim, num_pages, max_pages_per_seq, max_context_len, scale,
                            workspace, workspace_bytes, as_stream(stream));
}

// Host-side check of a block table before it is uploaded: every page a
// sequence's context needs is in [0, num_pages) and no page is shared by two
// (sequence, slot) pairs.  Returns 0 or AMP_ERR_INVALID with the first fault.
int amp_paged_validate_block_table(const int32_t* block_table, const int32_t* ctx_lens, int B,
                                   int max_pages_per_seq, int num_pages) {
    AMPB_REQUIRE(block_table && ctx_lens && B > 0 && max_pages_per_seq > 0 && num_pages > 0,
                 AMP_ERR_INVALID, "bad block-table arguments");
    std::vector<int> owner(num_pages, -1);
    for (int b = 0; b < B; ++b) {
        AMPB_REQUIRE(ctx_lens[b] >= 0, AMP_ERR_INVALID, "sequence %d: negative context length", b);
        const int need = (ctx_lens[b] + kPage - 1) / kPage;
        AMPB_REQUIRE(need <= max_pages_per_seq, AMP_ERR_INVALID,
                     "sequence %d needs %d pages, table rows hold %d", b, need, max_pages_per_seq);
        for (int i = 0; i < need; ++i) {
            const int pg = block_table[(int64_t)b * max_pages_per_seq + i];
            AMPB_REQUIRE(pg >= 0 && pg < num_pages, AMP_ERR_INVALID,
                         "sequence %d slot %d: page id %d outside [0, %d)", b, i, pg, num_pages);
            AMPB_REQUIRE(owner[pg] < 0, AMP_ERR_INVALID,
                         "page %d used twice (sequence %d slot %d, and entry %d)", pg, b, i,
                         owner[pg]);
            owner[pg] = b * max_pages_per_seq + i;
        }
    }
    return AMP_OK;
}

}  // extern "C"
