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
// Decode is HBM-bound (4 KiB of K+V per context token for Hkv = 8, D = 128),
// and context lengths differ widely, so the work is balanced by pages, not by
// sequences: the pages of all (kv head, sequence) pairs form one list
// (kv head major, then sequence, then page) and each of the persistent CTAs
// (3 per SM) streams an equal contiguous slice of it, crossing sequence
// boundaries without draining its pipeline.  160 threads per CTA:
//   warp 4     producer: TMA (4-D page-gather map, 128-byte swizzle) of each
//              page's K and V blocks (2 x 4 KiB) into an 8-stage shared-memory
//              ring, so 64 KiB per CTA are in flight ahead of the math.
//   warps 0-3  consumers; the CTA's k-th page goes to warp k % 4.  Per page, on
//              the tensor cores (mma.sync m16n8k16, bf16 -> fp32):
//              S^T[16 tokens x 8 heads] = K Q^T (K by ldmatrix, Q held in
//              registers as B fragments; the GQA group's G <= 8 query heads
//              fill the 8 columns), online softmax per head down the token
//              rows (quad shuffles), P^T turned into B fragments by movmatrix,
//              O^T[128 x 8] += V^T P^T (V by ldmatrix.trans).
//              At the end of each (kv head, sequence) segment of its slice a
//              warp writes its partial (m, l, O) for that segment.
//   k_paged_plan (before) turns context lengths into page prefix sums;
//   k_paged_combine (after) merges each query head's partials through their
//   log-sum-exp.
// A page id outside [0, num_pages) is never loaded: it is flagged in the device
// status word (AMP_DEV_ERR_BAD_PAGE) and its tokens are treated as masked; so is
// a context longer than max_context_len (its extra pages are not read).
// Slots past the context in the last page may hold anything: their scores are
// masked and their V rows zeroed in shared memory before the PV product.
#include <cuda.h>

#include <algorithm>
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
constexpr int kCWarps = 4;          // consumer warps
constexpr int kThreads = (kCWarps + 1) * 32;
constexpr int kStages = 8;
constexpr int kSmemSeqs = 1024;     // up to this batch the decode CTAs build the page
                                    // prefix sums themselves (else k_paged_plan does)
constexpr int kSlab = kPage * 128;           // 16 rows x 128 B (64 bf16 of D), swizzled
constexpr int kStageBytes = 4 * kSlab;       // K d0-63 | K d64-127 | V d0-63 | V d64-127
constexpr int kDecodeSmem = kStages * kStageBytes + 1024 + 256 + (33 + kSmemSeqs + 1) * 4;
// Page k goes to stage k % kStages and to consumer warp k % kCWarps.  With
// kStages a multiple of kCWarps every stage has one consumer warp, which reaches
// fill n + 1 of its stage only after it has released fill n -- so a parity wait
// can never match a phase two fills back.
static_assert(kStages % kCWarps == 0, "each ring stage must belong to one consumer warp");

constexpr int kMinPages = 16;       // smallest slice a CTA streams

struct DecodeParams {
    const __nv_bfloat16* q;
    const int* block_table;
    const int* ctx_lens;
    int* pref;         // [B + 1] exclusive prefix sums of pages per sequence
    float* part_o;     // [B][Hq][rows][D]
    float* part_ml;    // [B][Hq][rows][2]  (m in log2 units, l)
    __nv_bfloat16* out;
    float* lse;
    int B, Hq, Hkv, num_pages, max_pages, max_ctx_pages;
    int rows;          // partial rows per query head = kCWarps * max CTAs per segment
    int n_cta;         // CTAs launched for k_paged_decode
    int plan_in_kernel;   // 1: B <= kSmemSeqs, prefix sums built in shared memory
    float scale_log2;
    int* status;
};

// Slice bookkeeping shared by the decode and combine kernels.
struct Slices {
    int64_t P_h, P;    // pages per kv head, pages in total
    int64_t n;         // CTAs that get a slice
    __device__ void init(const DecodeParams& p, const int* pref) {
        P_h = pref[p.B];
        P = P_h * p.Hkv;
        const int64_t by_size = P / kMinPages;
        n = min((int64_t)p.n_cta, by_size > 0 ? by_size : (int64_t)1);
    }
    __device__ int64_t begin(int64_t c) const { return c * P / n; }
    // the CTA whose slice holds flattened page f
    __device__ int64_t owner(int64_t f) const { return ((f + 1) * n - 1) / P; }
};

// largest b with pref[b] <= r (pref[B] > r)
__device__ __forceinline__ int seq_of(const int* pref, int B, int64_t r) {
    int lo = 0, hi = B - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (pref[mid] <= r) lo = mid; else hi = mid - 1;
    }
    return lo;
}

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

// Exclusive prefix sums of the pages each sequence needs, clamped to
// max_context_len (a longer context is flagged and cut there), written to
// out[0..B] by all NT threads of the block.  scratch: 33 ints of shared memory.
template <int NT>
__device__ void page_prefix(const DecodeParams& p, int* out, int* scratch, bool flag) {
    constexpr int NW = NT / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int* warp_tot = scratch;
    int& carry = scratch[32];
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int base = 0; base < p.B; base += NT) {
        const int b = base + threadIdx.x;
        int v = 0;
        if (b < p.B) {
            const int ctx = max(0, p.ctx_lens[b]);
            v = (ctx + kPage - 1) / kPage;
            if (v > p.max_ctx_pages) {
                if (flag) atomicExch(p.status, AMP_DEV_ERR_BAD_PAGE);
                v = p.max_ctx_pages;
            }
        }
        int incl = v;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += t;
        }
        if (lane == 31) warp_tot[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            int w = lane < NW ? warp_tot[lane] : 0;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, w, off);
                if (lane >= off) w += t;
            }
            if (lane < NW) warp_tot[lane] = w;   // inclusive over warps
        }
        __syncthreads();
        const int excl = carry + (warp > 0 ? warp_tot[warp - 1] : 0) + incl - v;
        if (b < p.B) out[b] = excl;
        __syncthreads();
        if (threadIdx.x == NT - 1) carry = excl + v;
        __syncthreads();
    }
    if (threadIdx.x == 0) out[p.B] = carry;
    __syncthreads();
}

// Large batches: the prefix sums once, in global memory, before the decode.
__global__ void __launch_bounds__(1024) k_paged_plan(const DecodeParams p) {
    pdl_wait();
    pdl_trigger();
    __shared__ int scratch[33];
    page_prefix<1024>(p, p.pref, scratch, true);
}

template <int G>
__global__ void __launch_bounds__(kThreads) k_paged_decode(const __grid_constant__ CUtensorMap tmK,
                                                           const __grid_constant__ CUtensorMap tmV,
                                                           const DecodeParams p) {
    static_assert(G >= 1 && G <= 8, "one n8 tile holds the GQA group");
    pdl_wait();
    pdl_trigger();
    constexpr int D = 128;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t c = blockIdx.x;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    int* page_ok = reinterpret_cast<int*>(empty + kStages);
    int* scratch = page_ok + kStages;             // 33 ints
    int* spref = scratch + 33;                    // [kSmemSeqs + 1]
    const int* pref = p.pref;
    if (p.plan_in_kernel) {
        // CTA 0 also leaves the sums in global memory for k_paged_combine
        page_prefix<kThreads>(p, spref, scratch, c == 0);
        if (c == 0)
            for (int i = threadIdx.x; i <= p.B; i += kThreads) p.pref[i] = spref[i];
        pref = spref;
    }
    Slices sl;
    sl.init(p, pref);
    if (sl.P == 0 || c >= sl.n) return;   // the combine kernel derives the same split
    const int64_t f0 = sl.begin(c), f1 = sl.begin(c + 1);
    // segment of the slice starting at flattened page f: kv head, sequence,
    // first page within the sequence, page count
    auto segment = [&](int64_t f, int& hk, int& b, int& page0, int& npg) {
        hk = (int)(f / sl.P_h);
        const int64_t r = f - (int64_t)hk * sl.P_h;
        b = seq_of(pref, p.B, r);
        page0 = (int)(r - pref[b]);
        npg = (int)min(f1 - f, (int64_t)pref[b + 1] - r);
    };

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kCWarps) {
        // ------------------------------------------------------------ producer
        // The whole warp walks the slice: it reads the block table 32 entries at
        // a time (one coalesced load instead of one dependent load per page);
        // lane 0 issues the copies.
        if (lane == 0) {
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
        }
        int k = 0;
        bool ok_run = true;
        for (int64_t f = f0; ok_run && f < f1;) {
            int hk, b, page0, npg;
            segment(f, hk, b, page0, npg);
            const int* bt = p.block_table + (int64_t)b * p.max_pages + page0;
            for (int base = 0; ok_run && base < npg; base += 32) {
                const int cnt = min(32, npg - base);
                const int my_page = lane < cnt ? bt[base + lane] : 0;
                for (int i = 0; i < cnt; ++i, ++k) {
                    const int page = __shfl_sync(0xffffffffu, my_page, i);
                    const int s = k % kStages;
                    if (!mbar_wait_warp(&empty[s], ((k / kStages) & 1) ^ 1, p.status)) {
                        ok_run = false;
                        break;
                    }
                    if (lane == 0) {
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
                    __syncwarp();
                }
            }
            f += npg;
        }
        // every copy issued lands before the shared memory is reused or released
        if (lane == 0)
            for (int kk = max(0, k - kStages); kk < k; ++kk)
                mbar_wait(&full[kk % kStages], (kk / kStages) & 1, p.status);
    } else {
        // ------------------------------------------------------------ consumers
        const int n = lane >> 2, kq = 2 * (lane & 3);
        const float c2 = p.scale_log2;
        const int r = lane >> 2;                   // token row of this lane's C elements (and r + 8)
        const int mi = lane >> 3, r8 = lane & 7;   // ldmatrix: matrix / row this lane addresses
        const int h0 = 2 * (lane & 3);             // heads of this lane's C columns: h0, h0 + 1
        int64_t kb = 0;                            // CTA-local index of the segment's first page
        bool ok_run = true;
        for (int64_t f = f0; ok_run && f < f1;) {
            int hk, b, page0, npg;
            segment(f, hk, b, page0, npg);
            const int ctx = p.ctx_lens[b];
            // Q^T as B fragments: lane holds head n at d = 16kk + 2(lane%4) (+8)
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
            float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};
            float o[8][4];
#pragma unroll
            for (int mt = 0; mt < 8; ++mt)
#pragma unroll
                for (int j = 0; j < 4; ++j) o[mt][j] = 0.0f;
            // this warp's pages of the segment: CTA-local index k = kb + i, k % 4 == warp
            for (int i = (int)((warp - kb % kCWarps + kCWarps) % kCWarps); i < npg; i += kCWarps) {
                const int64_t k = kb + i;
                const int s = (int)(k % kStages);
                if (!mbar_wait_warp(&full[s], (uint32_t)((k / kStages) & 1), p.status)) {
                    ok_run = false;
                    break;
                }
                const int vt = page_ok[s] ? min(kPage, ctx - (page0 + i) * kPage) : 0;
                uint8_t* st = ring + s * kStageBytes;
                if (vt > 0) {
                    if (vt < kPage) {
                        // zero V rows of the slots past the context (whole 128-byte
                        // rows, so the swizzle does not matter)
                        for (int e = lane; e < (kPage - vt) * 2 * 8; e += 32) {
                            const int row = vt + (e >> 4), half = (e >> 3) & 1, ch = e & 7;
                            *reinterpret_cast<uint4*>(st + (2 + half) * kSlab + row * 128 + ch * 16) =
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
                        x[j] = tok < vt ? sc[j] * c2 : -INFINITY;
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
            // this warp's partial for the segment (m = -inf if it saw no page)
            const int64_t fb = (int64_t)hk * sl.P_h + pref[b];
            const int64_t j = c - sl.owner(fb);
            if (j >= 0 && j * kCWarps + warp < p.rows) {
                const int64_t row0 = ((int64_t)b * p.Hq + hk * G) * p.rows + j * kCWarps + warp;
#pragma unroll
                for (int mt = 0; mt < 8; ++mt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int g = h0 + (e & 1);
                        if (g < G)
                            p.part_o[(row0 + (int64_t)g * p.rows) * D + 16 * mt + r + 8 * (e >> 1)] =
                                o[mt][e];
                    }
                if (r == 0) {
#pragma unroll
                    for (int e = 0; e < 2; ++e)
                        if (h0 + e < G) {
                            p.part_ml[(row0 + (int64_t)(h0 + e) * p.rows) * 2] = m[e];
                            p.part_ml[(row0 + (int64_t)(h0 + e) * p.rows) * 2 + 1] = l[e];
                        }
                }
            } else if (lane == 0) {
                atomicExch(p.status, AMP_DEV_ERR_BAD_PAGE);   // more slices than the workspace holds
            }
            kb += npg;
            f += npg;
        }
    }
    // every copy the producer issued has landed (it waited for them) before exit
    __syncthreads();
}

// One CTA per (sequence, query head): 8 warps share the partial rows, each lane
// four consecutive elements of D; the warps merge through shared memory.
constexpr int kCombineWarps = 8;
template <int D>
__global__ void __launch_bounds__(kCombineWarps * 32) k_paged_combine(const DecodeParams p) {
    static_assert(D == 128, "one float4 per lane covers D");
    pdl_wait();
    pdl_trigger();
    __shared__ float red[kCombineWarps];
    __shared__ float o_s[kCombineWarps][D];
    __shared__ float l_s[kCombineWarps];
    const int bh = blockIdx.x;
    const int b = bh / p.Hq, hq = bh % p.Hq;
    const int hk = hq / (p.Hq / p.Hkv);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    Slices sl;
    sl.init(p, p.pref);
    const int64_t pages = p.pref[b + 1] - p.pref[b];
    int n_rows = 0;
    if (pages > 0) {
        const int64_t fb = (int64_t)hk * sl.P_h + p.pref[b];
        n_rows = (int)min((int64_t)p.rows, (sl.owner(fb + pages - 1) - sl.owner(fb) + 1) * kCWarps);
    }
    const int64_t row0 = (int64_t)bh * p.rows;
    // One pass: each warp folds its rows (every kCombineWarps-th) into a running
    // (max, sum, O) with the online rescale, four rows loaded ahead; the warps'
    // states merge through shared memory.
    float Mw = -INFINITY, Lw = 0.0f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r0 = warp; r0 < n_rows; r0 += 4 * kCombineWarps) {
        float2 ml[4];
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int r = r0 + u * kCombineWarps;
            if (r < n_rows) {
                ml[u] = *reinterpret_cast<const float2*>(p.part_ml + (row0 + r) * 2);
                v[u] = *reinterpret_cast<const float4*>(p.part_o + (row0 + r) * D + 4 * lane);
            } else {
                ml[u] = make_float2(-INFINITY, 0.0f);
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (ml[u].x == -INFINITY) continue;   // warp-uniform: a row that saw no page
            if (ml[u].x > Mw) {
                const float sc = (Mw == -INFINITY) ? 0.0f : ex2_approx(Mw - ml[u].x);
                Lw *= sc;
                acc.x *= sc; acc.y *= sc; acc.z *= sc; acc.w *= sc;
                Mw = ml[u].x;
            }
            const float a = ex2_approx(ml[u].x - Mw);
            Lw += a * ml[u].y;
            acc.x += a * v[u].x;
            acc.y += a * v[u].y;
            acc.z += a * v[u].z;
            acc.w += a * v[u].w;
        }
    }
    *reinterpret_cast<float4*>(&o_s[warp][4 * lane]) = acc;
    if (lane == 0) {
        l_s[warp] = Lw;
        red[warp] = Mw;
    }
    __syncthreads();
    if (threadIdx.x < D) {
        const int d = threadIdx.x;
        float M = red[0];
#pragma unroll
        for (int w = 1; w < kCombineWarps; ++w) M = fmaxf(M, red[w]);
        float O = 0.0f, Lt = 0.0f;
#pragma unroll
        for (int w = 0; w < kCombineWarps; ++w) {
            const float sc = (red[w] == -INFINITY) ? 0.0f : ex2_approx(red[w] - M);
            O += sc * o_s[w][d];
            Lt += sc * l_s[w];
        }
        p.out[(int64_t)bh * D + d] = __float2bfloat16_rn(Lt > 0.0f ? O / Lt : 0.0f);
        if (d == 0 && p.lse) {
            float lg;
            asm("lg2.approx.f32 %0, %1;" : "=f"(lg) : "f"(Lt));
            p.lse[bh] = Lt > 0.0f ? (M + lg) * 0.69314718055994531f : -INFINITY;
        }
    }
}

// partial rows per query head: kCWarps for every CTA a sequence's pages can span
int decode_rows(int max_ctx) {
    const int64_t max_pages = ((int64_t)max_ctx + kPage - 1) / kPage;
    return (int)(kCWarps * ((max_pages + kMinPages - 1) / kMinPages + 1));
}

size_t decode_ws_bytes(int B, int Hq, int D, int max_ctx) {
    const int64_t rows = (int64_t)B * Hq * decode_rows(max_ctx > 0 ? max_ctx : 1);
    const int64_t pref = ((int64_t)B + 1 + 63) / 64 * 64;   // int32, 256-byte multiple
    return (size_t)(pref * 4 + rows * D * 4 + rows * 2 * 4 + 256);
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
    p.rows = decode_rows(max_ctx);
    p.pref = static_cast<int*>(ws);
    const int64_t pref_words = ((int64_t)B + 1 + 63) / 64 * 64;
    p.part_o = reinterpret_cast<float*>(p.pref + pref_words);
    p.part_ml = p.part_o + (int64_t)B * Hq * p.rows * D;
    p.out = static_cast<__nv_bfloat16*>(out);
    p.lse = lse;
    p.B = B;
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.num_pages = num_pages;
    p.max_pages = max_pages;
    p.max_ctx_pages = (max_ctx + kPage - 1) / kPage;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.status = status;
    p.n_cta = 0;   // set per kernel below, from its occupancy
    p.plan_in_kernel = B <= kSmemSeqs;
    if (!p.plan_in_kernel) {
        AMPB_CHECK_CUDA(launch_pdl(k_paged_plan, dim3(1), dim3(1024), 0, st, p));
    }
    // persistent grid: as many CTAs as are resident at once (per device and
    // group size, from the occupancy calculator), never more than the pages need
    auto go = [&](auto kern, std::atomic<int>* per_dev) {
        int dev = 0;
        AMPB_CHECK_CUDA(cudaGetDevice(&dev));
        std::atomic<int>& resident = per_dev[dev & 31];
        if (resident.load() == 0) {
            AMPB_CHECK_CUDA(cudaFuncSetAttribute(
                kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kDecodeSmem));
            int per_sm = 0;
            AMPB_CHECK_CUDA(
                cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, kDecodeSmem));
            resident.store(std::max(1, per_sm) * sm_count());
        }
        const int64_t total_pages = (int64_t)Hkv * B * p.max_ctx_pages;
        const int64_t by_size = (total_pages + kMinPages - 1) / kMinPages;
        p.n_cta = (int)std::max<int64_t>(1, std::min<int64_t>(resident.load(), by_size));
        AMPB_CHECK_CUDA(launch_pdl(kern, dim3(p.n_cta), dim3(kThreads), kDecodeSmem, st, tmK, tmV, p));
        return AMP_OK;
    };
    static std::atomic<int> res1[32], res2[32], res4[32], res8[32];
    switch (Hq / Hkv) {
        case 1: rc = go(k_paged_decode<1>, res1); break;
        case 2: rc = go(k_paged_decode<2>, res2); break;
        case 4: rc = go(k_paged_decode<4>, res4); break;
        case 8: rc = go(k_paged_decode<8>, res8); break;
        default:
            set_error(AMP_ERR_UNSUPPORTED, "GQA group size %d not supported (1, 2, 4, 8)", Hq / Hkv);
            return AMP_ERR_UNSUPPORTED;
    }
    if (rc) return rc;
    AMPB_CHECK_LAUNCH("k_paged_decode");
    AMPB_CHECK_CUDA(launch_pdl(k_paged_combine<128>, dim3(B * Hq), dim3(kCombineWarps * 32), 0, st, p));
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

// Padded block table from per-sequence page lists: the shape AMP's scheduler
// keeps (Sequence::kv_page_ids, include/scheduler.hpp:61), concatenated --
// sequence b's pages are page_ids[seq_start[b] .. seq_start[b + 1]) in token
// order.  block_table[b][i] = its i-th page, -1 past the list.  A list longer
// than a table row, or shorter than the sequence's context needs, is an error.
int amp_paged_pack_block_table(const int32_t* page_ids, const int32_t* seq_start,
                               const int32_t* ctx_lens, int B, int max_pages_per_seq,
                               int32_t* block_table) {
    AMPB_REQUIRE(page_ids && seq_start && ctx_lens && block_table && B > 0 &&
                     max_pages_per_seq > 0,
                 AMP_ERR_INVALID, "bad block-table arguments");
    for (int b = 0; b < B; ++b) {
        const int n = seq_start[b + 1] - seq_start[b];
        AMPB_REQUIRE(n >= 0 && n <= max_pages_per_seq, AMP_ERR_INVALID,
                     "sequence %d holds %d pages, table rows hold %d", b, n, max_pages_per_seq);
        AMPB_REQUIRE(ctx_lens[b] >= 0 && (ctx_lens[b] + kPage - 1) / kPage <= n, AMP_ERR_INVALID,
                     "sequence %d: context %d needs %d pages, it holds %d", b, ctx_lens[b],
                     (ctx_lens[b] + kPage - 1) / kPage, n);
        int32_t* row = block_table + (int64_t)b * max_pages_per_seq;
        for (int i = 0; i < max_pages_per_seq; ++i) row[i] = i < n ? page_ids[seq_start[b] + i] : -1;
    }
    return AMP_OK;
}

// Bytes of one contiguous K (or V) pool [num_pages][Hkv][16][head_dim] bf16.  A
// page id handed out by a page allocator (AMP's PagePoolFast ids are 0..n-1,
// src/pool_fast.cpp:31-60) is the pool's row, so one allocation replaces the
// allocator's per-page cudaMalloc (src/pool_fast.cpp:11-13).
size_t amp_paged_pool_bytes(int num_pages, int Hkv, int head_dim) {
    if (num_pages <= 0 || Hkv <= 0 || head_dim <= 0) return 0;
    return (size_t)num_pages * Hkv * kPage * head_dim * 2;
}

}  // extern "C"
