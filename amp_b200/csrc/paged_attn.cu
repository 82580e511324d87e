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
// so it runs on the CUDA cores with split-KV: one CTA per (chunk of 32 pages,
// kv head, sequence); each of its 4 warps takes every 4th page -- lane pair
// (2t, 2t+1) holds token t of the page, each lane half of D, so the 4 KiB
// page row is read fully coalesced -- and keeps an online softmax for the
// GQA group's query heads that share the kv head.  Warps merge in shared
// memory, chunks merge in k_paged_combine through their log-sum-exp.
// A page id outside [0, num_pages) is skipped and flagged in the device
// status word (AMP_DEV_ERR_BAD_PAGE); it never becomes a memory access.
#include <cmath>
#include <vector>

#include "common.cuh"
#include "runtime.h"
#include "tc_common.cuh"

namespace ampb {
namespace {

constexpr int kPage = 16;
constexpr int kChunkPages = 32;     // 512 tokens per split
constexpr int kWarps = 4;

struct DecodeParams {
    const __nv_bfloat16* q;
    const __nv_bfloat16* k_pool;
    const __nv_bfloat16* v_pool;
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

__device__ __forceinline__ void bf16x8_to_f32(uint4 w, float* f) {
    f[0] = bf16_lo(w.x); f[1] = bf16_hi(w.x); f[2] = bf16_lo(w.y); f[3] = bf16_hi(w.y);
    f[4] = bf16_lo(w.z); f[5] = bf16_hi(w.z); f[6] = bf16_lo(w.w); f[7] = bf16_hi(w.w);
}

template <int D, int G>
__global__ void __launch_bounds__(kWarps * 32) k_paged_decode(const DecodeParams p) {
    static_assert(D == 128, "decode kernel is written for head_dim 128");
    constexpr int HALF = D / 2;                 // elements of D per lane in the QK stage
    constexpr int DPL = D / 32;                 // elements of D per lane in the PV stage
    const int chunk = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ctx = p.ctx_lens[b];
    const int n_pages = (ctx + kPage - 1) / kPage;
    const int pg0 = chunk * kChunkPages;
    if (pg0 >= n_pages || ctx <= 0) return;     // the combine kernel knows the chunk count
    const int pg1 = min(n_pages, pg0 + kChunkPages);

    __shared__ float q_s[G][D];
    __shared__ float m_s[kWarps][G], l_s[kWarps][G];
    __shared__ float o_s[kWarps][G][D];
    for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
        const int g = i / D, d = i % D;
        q_s[g][d] = __bfloat162float(p.q[((int64_t)b * p.Hq + hk * G + g) * D + d]);
    }
    __syncthreads();

    const int t = lane >> 1, half = lane & 1;
    float m[G], l[G], o[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) o[g][j] = 0.0f;
    }
    const int* bt = p.block_table + (int64_t)b * p.max_pages;
    for (int pi = pg0 + warp; pi < pg1; pi += kWarps) {
        const int page = bt[pi];
        if (page < 0 || page >= p.num_pages) {
            if (lane == 0) atomicExch(p.status, AMP_DEV_ERR_BAD_PAGE);
            continue;
        }
        const int64_t base = ((int64_t)page * p.Hkv + hk) * kPage * D;
        // K: lane pair (2t, 2t+1) reads token t's row, one half each (8 x 16 B)
        const uint4* kp = reinterpret_cast<const uint4*>(p.k_pool + base + t * D + half * HALF);
        uint4 kw[HALF / 8];
#pragma unroll
        for (int i = 0; i < HALF / 8; ++i) kw[i] = ldg_stream_v4(kp + i);
        // V: lane reads DPL consecutive elements of every token row (8 B each)
        const uint2* vp = reinterpret_cast<const uint2*>(p.v_pool + base + lane * DPL);
        uint2 vw[kPage];
#pragma unroll
        for (int tt = 0; tt < kPage; ++tt) vw[tt] = *(vp + tt * (D / DPL));
        float s[G];
#pragma unroll
        for (int g = 0; g < G; ++g) s[g] = 0.0f;
#pragma unroll
        for (int i = 0; i < HALF / 8; ++i) {
            float kf[8];
            bf16x8_to_f32(kw[i], kf);
#pragma unroll
            for (int e = 0; e < 8; ++e)
#pragma unroll
                for (int g = 0; g < G; ++g) s[g] = fmaf(q_s[g][half * HALF + i * 8 + e], kf[e], s[g]);
        }
        const bool tok_ok = pi * kPage + t < ctx;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            s[g] += __shfl_xor_sync(0xffffffffu, s[g], 1);
            s[g] = tok_ok ? s[g] * p.scale_log2 : -INFINITY;
            float mt = s[g];
#pragma unroll
            for (int off = 2; off < 32; off <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
            const float m_new = fmaxf(m[g], mt);              // finite: token 0 of a page is valid
            const float alpha = ex2_approx(m[g] - m_new);     // 0 when m[g] = -inf
            const float pr = ex2_approx(s[g] - m_new);
            float ps = half ? 0.0f : pr;                      // count each token once
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
            l[g] = l[g] * alpha + ps;
            m[g] = m_new;
#pragma unroll
            for (int j = 0; j < DPL; ++j) o[g][j] *= alpha;
            s[g] = pr;
        }
        // slots past the context in the last page may hold anything: zero their V
        const int valid_tok = ctx - pi * kPage;
#pragma unroll
        for (int tt = 0; tt < kPage; ++tt)
            if (tt >= valid_tok) vw[tt] = make_uint2(0u, 0u);
#pragma unroll
        for (int tt = 0; tt < kPage; ++tt) {
            const float v0 = bf16_lo(vw[tt].x), v1 = bf16_hi(vw[tt].x);
            const float v2 = bf16_lo(vw[tt].y), v3 = bf16_hi(vw[tt].y);
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float pt = __shfl_sync(0xffffffffu, s[g], 2 * tt);
                o[g][0] = fmaf(pt, v0, o[g][0]);
                o[g][1] = fmaf(pt, v1, o[g][1]);
                o[g][2] = fmaf(pt, v2, o[g][2]);
                o[g][3] = fmaf(pt, v3, o[g][3]);
            }
        }
    }
    // merge the 4 warps of this chunk
#pragma unroll
    for (int g = 0; g < G; ++g) {
        if (lane == 0) {
            m_s[warp][g] = m[g];
            l_s[warp][g] = l[g];
        }
#pragma unroll
        for (int j = 0; j < DPL; ++j) o_s[warp][g][lane * DPL + j] = o[g][j];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
        const int g = i / D, d = i % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, m_s[w][g]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const float a = (m_s[w][g] == -INFINITY) ? 0.0f : ex2_approx(m_s[w][g] - M);
            L += a * l_s[w][g];
            O += a * o_s[w][g][d];
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
    if (!(scale > 0.0f)) scale = 1.0f / sqrtf((float)D);
    DecodeParams p;
    p.q = static_cast<const __nv_bfloat16*>(q);
    p.k_pool = static_cast<const __nv_bfloat16*>(k_pool);
    p.v_pool = static_cast<const __nv_bfloat16*>(v_pool);
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
    switch (Hq / Hkv) {
        case 1: k_paged_decode<128, 1><<<grid, kWarps * 32, 0, st>>>(p); break;
        case 2: k_paged_decode<128, 2><<<grid, kWarps * 32, 0, st>>>(p); break;
        case 4: k_paged_decode<128, 4><<<grid, kWarps * 32, 0, st>>>(p); break;
        case 8: k_paged_decode<128, 8><<<grid, kWarps * 32, 0, st>>>(p); break;
        default:
            set_error(AMP_ERR_UNSUPPORTED, "GQA group size %d not supported (1, 2, 4, 8)", Hq / Hkv);
            return AMP_ERR_UNSUPPORTED;
    }
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
