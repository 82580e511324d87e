// flash_attn_bwd.cu -- FlashAttention-2 backward on tcgen05: the lse consumer.
//
// The reference has no backward; its forward documents lse as "required for
// the backward pass" (kernels/flash_attn.cuh:48).  Given Q, K, V, O, dO and the
// forward's lse (natural log):
//   Delta = rowsum(dO * O)                                   k_fa_bwd_delta
//   P = exp(scale Q K^T - lse),  dP = dO V^T,  dS = P * (dP - Delta)
//   dV = P^T dO,  dK = scale dS^T Q,  dQ = scale dS K
// in two passes shaped like the forward, so every product is one of its MMA
// forms (SS, K-major x K-major; TS with P / dS in TMEM and an MN-major B):
//   k_fa_bwd_dkdv  per (batch * kv head, 128-key tile), on persistent CTAs (one
//                  per SM) that walk pairs of such tiles.  S^T = K Q^T and
//                  dP^T = V dO^T put keys on the TMEM lanes; P^T and dS^T go
//                  back over them as bf16; dV += P^T dO and dK += dS^T Q
//                  accumulate in TMEM over every query tile of every query head
//                  that shares the kv head (GQA).
//   k_fa_bwd_dq    per (batch * query head, 128-query tile), on persistent
//                  CTAs (one per SM) that walk pairs of such tiles.  S = Q K^T,
//                  dP = dO V^T with queries on the lanes; dS back over dP;
//                  dQ += dS K over the visible key tiles.
// Steps overlap: the element-wise warps write P (or P^T) first and dS after, so
// the tensor core takes the next step's S^T while dS^T is computed (dK/dV pass:
// dV_t, S^T_{t+1}, dK_t, dP^T_{t+1}); the dQ pass keeps two S buffers in TMEM
// (S_{j+1}, dQ_j, dP_{j+1}).
// Each pass recomputes P from lse, so there are no atomics and no fp32 dQ
// accumulator in global memory.  Both kernels: 384 threads; warp 0 TMA, warp 1
// TMEM + MMA issue (warps 2-3 only lend their registers, setmaxnreg 72 / 216);
// warps 4-11 the element-wise work, two warps per TMEM lane quadrant (one row
// per thread), each taking one 64-column half of the 128-column tile.
#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <cmath>

#include "common.cuh"
#include "runtime.h"
#include "tc_common.cuh"

namespace ampb {

int fa_make_tmap_3d(CUtensorMap* m, const void* base, int64_t d, int64_t s, int64_t bh);

namespace {

constexpr int BT = 128;                 // rows per query / key tile
constexpr int kThreads = 384;      // 3 warpgroups
// Register split: 128 * 72 + 256 * 216 == 384 * 168, the launch's allocation
// (__launch_bounds__(384, 1) compiles for exactly 168).
constexpr int kRegCtl = 72, kRegEw = 216;
constexpr int SLAB_BYTES = 128 * 128;   // [128 rows x 128 bytes] swizzled slab
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct BwdCfg {
    static constexpr int SLABS = D / 64;
    static constexpr int TILE = SLABS * SLAB_BYTES;          // 128 rows x D bf16
    static constexpr uint32_t IDESC_SS = make_idesc(1, 1, 0, 0, BT, BT);
    static constexpr uint32_t IDESC_TS = make_idesc(1, 1, 0, 1, BT, D);
};

struct BwdParams {
    int B, Hq, Hkv, S_q, S_kv;
    int causal, causal_offset;   // key j visible for query i iff j <= i + causal_offset
    float scale, scale_log2;
    const float* lse;            // [B*Hq][S_q], natural log (forward output)
    const float* delta;          // [B*Hq][S_q]
    void* dq;                    // [B*Hq][S_q][D] bf16
    void* dk;                    // [B*Hkv][S_kv][D] bf16
    void* dv;
    int* status;
};

// SS product of two 128-row K-major tiles over D: acc[128 x 128] (+)= A B^T
template <int D>
__device__ __forceinline__ void mma_ss(uint32_t acc, uint32_t a_addr, uint32_t b_addr) {
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = (kk >> 2) * SLAB_BYTES + (kk & 3) * 32;
        tc_mma_f16(acc, smem_desc_sw128(a_addr + off, 16, 1024),
                   smem_desc_sw128(b_addr + off, 16, 1024), BwdCfg<D>::IDESC_SS, kk != 0);
    }
}
// TS product: acc[128 x D] (+)= T[128 x 128] (bf16 in TMEM) x B[128 rows x D] (MN-major).
// T is packed two bf16 per column in two halves: its columns 0-63 at TMEM
// columns [t_col, t_col + 32), 64-127 at [t_col + 96, t_col + 128) -- where the
// two element-wise warps of a lane quadrant write them (see the element-wise code).
template <int D>
__device__ __forceinline__ void mma_ts(uint32_t acc, uint32_t t_col, uint32_t b_addr,
                                       bool accumulate) {
#pragma unroll
    for (int kk = 0; kk < BT / 16; ++kk)
        tc_mma_f16_ts(acc, t_col + kk * 8 + (kk >= BT / 32 ? BT / 2 : 0),
                      smem_desc_sw128(b_addr + kk * 16 * 128, SLAB_BYTES, 1024),
                      BwdCfg<D>::IDESC_TS, (accumulate || kk != 0) ? 1u : 0u);
}

// ---------------------------------------------------------------- Delta
// Delta[row] = sum_d dO[row][d] * O[row][d] in fp32.  HBM-bound (reads O and dO
// once): D/8 lanes per row with 16-byte loads, kDeltaLoads rows per lane group in
// flight, and the row's partial sums reduced within its lane group.
constexpr int kDeltaLoads = 4;
template <int D>
__global__ void __launch_bounds__(256) k_fa_bwd_delta(const __nv_bfloat16* __restrict__ O,
                                                      const __nv_bfloat16* __restrict__ dO,
                                                      float* __restrict__ delta, int64_t rows) {
    pdl_wait();
    pdl_trigger();
    constexpr int LPR = D / 8;            // lanes per row, 8 bf16 (16 bytes) each
    constexpr int RPW = 32 / LPR;         // rows per warp-wide load
    constexpr int ROWS = RPW * kDeltaLoads;
    static_assert(LPR >= 1 && LPR <= 32 && (LPR & (LPR - 1)) == 0, "D/8 lanes per row");
    const int lane = threadIdx.x & 31;
    const int sub = lane / LPR, col = (lane % LPR) * 8;
    const int64_t nwarps = (int64_t)gridDim.x * 8;
    for (int64_t r0 = ((int64_t)blockIdx.x * 8 + (threadIdx.x >> 5)) * ROWS; r0 < rows;
         r0 += nwarps * ROWS) {
        uint4 o[kDeltaLoads], g[kDeltaLoads];
#pragma unroll
        for (int u = 0; u < kDeltaLoads; ++u) {
            const int64_t r = r0 + u * RPW + sub;
            if (r < rows) {
                o[u] = *reinterpret_cast<const uint4*>(O + r * D + col);
                g[u] = *reinterpret_cast<const uint4*>(dO + r * D + col);
            } else {
                o[u] = make_uint4(0u, 0u, 0u, 0u);
                g[u] = o[u];
            }
        }
#pragma unroll
        for (int u = 0; u < kDeltaLoads; ++u) {
            const uint32_t ow[4] = {o[u].x, o[u].y, o[u].z, o[u].w};
            const uint32_t gw[4] = {g[u].x, g[u].y, g[u].z, g[u].w};
            float acc = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                acc = fmaf(bf16_lo(ow[i]), bf16_lo(gw[i]), acc);
                acc = fmaf(bf16_hi(ow[i]), bf16_hi(gw[i]), acc);
            }
#pragma unroll
            for (int m = LPR / 2; m > 0; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
            const int64_t r = r0 + u * RPW + sub;
            if (lane % LPR == 0 && r < rows) delta[r] = acc;
        }
    }
}

// store columns [half * D/2, half * D/2 + D/2) of one 128 x D fp32 TMEM
// accumulator row (this thread's lane) as bf16 * mul
template <int D>
__device__ __forceinline__ void store_row(uint32_t lane_addr, float mul, __nv_bfloat16* row,
                                          bool ok, int half) {
    __syncwarp();
#pragma unroll
    for (int ocl = 0; ocl < D / 64; ++ocl) {
        const int oc = half * (D / 64) + ocl;
        uint32_t v[32];
        tmem_ld_32x32b_x32(lane_addr + oc * 32, v);
        tmem_ld_wait();
        if (ok) {
#pragma unroll
            for (int e = 0; e < 32; e += 8) {
                uint4 w;
                w.x = f32x2_to_bf16x2(__uint_as_float(v[e]) * mul, __uint_as_float(v[e + 1]) * mul);
                w.y = f32x2_to_bf16x2(__uint_as_float(v[e + 2]) * mul, __uint_as_float(v[e + 3]) * mul);
                w.z = f32x2_to_bf16x2(__uint_as_float(v[e + 4]) * mul, __uint_as_float(v[e + 5]) * mul);
                w.w = f32x2_to_bf16x2(__uint_as_float(v[e + 6]) * mul, __uint_as_float(v[e + 7]) * mul);
                *reinterpret_cast<uint4*>(row + oc * 32 + e) = w;
            }
        }
    }
}

template <int D>
__device__ __forceinline__ void store_zero_row(__nv_bfloat16* row, int half) {
#pragma unroll
    for (int e = half * (D / 2); e < (half + 1) * (D / 2); e += 8)
        *reinterpret_cast<uint4*>(row + e) = make_uint4(0u, 0u, 0u, 0u);
}

// ---------------------------------------------------------------- dK, dV
template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    k_fa_bwd_dkdv(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                  const BwdParams p) {
    pdl_wait();
    pdl_trigger();
    using CF = BwdCfg<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint8_t* k_s = smem;                          // K_j
    uint8_t* v_s = k_s + CF::TILE;                // V_j
    uint8_t* q_s = v_s + CF::TILE;                // [2][Q_i]
    uint8_t* o_s = q_s + 2 * CF::TILE;            // [2][dO_i]
    float* cols = reinterpret_cast<float*>(o_s + 2 * CF::TILE);   // [2][2][128] lse2, Delta
    uint64_t* bars = reinterpret_cast<uint64_t*>(cols + 2 * 2 * BT);
    uint64_t* kv_full = bars;
    uint64_t* qs_full = bars + 1;     // [2]
    uint64_t* qs_empty = bars + 3;    // [2]
    uint64_t* s_full = bars + 5;      // S^T of the step in TMEM
    uint64_t* dp_full = bars + 6;     // dP^T of the step in TMEM
    uint64_t* p_full = bars + 7;      // P^T written back (8 warps)
    uint64_t* ds_full = bars + 8;     // dS^T written back (8 warps)
    // bars + 9: unused (S^T_{t+1} follows dV_t in MMA issue order, no barrier between)
    uint64_t* dk_done = bars + 10;    // dK has read dS^T: dP^T may be rewritten
    uint64_t* drain = bars + 11;
    uint64_t* cols_ready = bars + 12; // [2]: the 256 element-wise threads posted the step
    uint64_t* kv_empty = bars + 14;   // the item's last MMA reading K / V has completed
    uint64_t* dkv_free = bars + 15;   // the item's epilogue has read dK, dV out of TMEM
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = p.Hq / p.Hkv;
    const int n_qt = (p.S_q + BT - 1) / BT;
    const int n_kt = (p.S_kv + BT - 1) / BT;
    // Persistent: unit u = blockIdx.x + (k/2) * gridDim.x pairs key tile n_kt-1-q with
    // key tile q of one kv head (under a causal mask they see the fewest and the most
    // query tiles), so the units of a causal square problem carry the same work.
    const int half_units = (n_kt + 1) / 2;
    const int units = p.B * p.Hkv * half_units;
    // k-th item of this CTA: 0 = no more, 1 = item (bh_kv, jt), 2 = empty slot
    auto item_at = [&](int k, int& bh_kv, int& jt) -> int {
        const int u = (int)blockIdx.x + (k >> 1) * (int)gridDim.x;
        if (u >= units) return 0;
        bh_kv = u / half_units;
        const int q = u % half_units;
        jt = (k & 1) ? q : n_kt - 1 - q;
        return ((k & 1) && q == n_kt - 1 - q) ? 2 : 1;
    };
    // first query tile with a query that sees a key of tile jt
    auto first_tile = [&](int jt) {
        int i_lo = 0;
        if (p.causal) {
            const int first_q = jt * BT - p.causal_offset;
            i_lo = first_q <= 0 ? 0 : first_q / BT;
        }
        return i_lo;
    };

    if (threadIdx.x == 0) {
        mbar_init(kv_full, 1);
        mbar_init(kv_empty, 1);
        mbar_init(dkv_free, 8);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&qs_full[s], 1);
            mbar_init(&qs_empty[s], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(dp_full, 1);
        mbar_init(p_full, 8);
        mbar_init(ds_full, 8);
        mbar_init(dk_done, 1);
        mbar_init(drain, 1);
        mbar_init(&cols_ready[0], 256);
        mbar_init(&cols_ready[1], 256);
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t T_S = tmem, T_dP = tmem + BT, T_dV = tmem + 2 * BT, T_dK = tmem + 2 * BT + D;

    if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegCtl));
    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmdO);
            int g = 0, li = 0;   // Q/dO tiles loaded (ring stage g & 1); items with work
            bool ok = true;
            for (int k = 0; ok; ++k) {
                int bh_kv, jt;
                const int st = item_at(k, bh_kv, jt);
                if (st == 0) break;
                if (st == 2) continue;
                const int i_lo = first_tile(jt);
                const int per_head = max(0, n_qt - i_lo);
                const int steps = G * per_head;
                if (steps == 0) continue;
                const int b = bh_kv / p.Hkv, hk = bh_kv % p.Hkv;
                // K_j / V_j once the previous item's last MMA reading them has completed
                if (li > 0 && !mbar_wait(kv_empty, (li - 1) & 1, p.status)) break;
                mbar_arrive_expect_tx(kv_full, 2 * CF::TILE);
#pragma unroll
                for (int sl = 0; sl < CF::SLABS; ++sl) {
                    tma_load_3d(k_s + sl * SLAB_BYTES, &tmK, kv_full, sl * 64, jt * BT, bh_kv);
                    tma_load_3d(v_s + sl * SLAB_BYTES, &tmV, kv_full, sl * 64, jt * BT, bh_kv);
                }
                for (int t = 0; t < steps; ++t, ++g) {
                    const int s = g & 1;
                    if (!mbar_wait(&qs_empty[s], ((g >> 1) & 1) ^ 1, p.status)) { ok = false; break; }
                    const int gq = t / per_head, it = i_lo + t % per_head;
                    const int bh_q = b * p.Hq + hk * G + gq;
                    mbar_arrive_expect_tx(&qs_full[s], 2 * CF::TILE);
#pragma unroll
                    for (int sl = 0; sl < CF::SLABS; ++sl) {
                        tma_load_3d(q_s + s * CF::TILE + sl * SLAB_BYTES, &tmQ, &qs_full[s],
                                    sl * 64, it * BT, bh_q);
                        tma_load_3d(o_s + s * CF::TILE + sl * SLAB_BYTES, &tmdO, &qs_full[s],
                                    sl * 64, it * BT, bh_q);
                    }
                }
                ++li;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // tensor-core order per step t:  dV_t, S^T_{t+1}, dK_t, dP^T_{t+1} -- so the
            // next step's S^T runs while the element-wise warps compute dS^T_t
            const uint32_t ka0 = smem_u32(k_s), va0 = smem_u32(v_s);
            auto qa = [&](int g) { return opaque_u32(smem_u32(q_s + (g & 1) * CF::TILE)); };
            auto oa = [&](int g) { return opaque_u32(smem_u32(o_s + (g & 1) * CF::TILE)); };
            int g = 0, li = 0;   // steps before this item; items with work before it
            bool ok = true;
            for (int k = 0; ok; ++k) {
                int bh_kv, jt;
                const int st = item_at(k, bh_kv, jt);
                if (st == 0) break;
                if (st == 2) continue;
                const int steps = G * max(0, n_qt - first_tile(jt));
                if (steps == 0) continue;
                const uint32_t ka = opaque_u32(ka0), va = opaque_u32(va0);
                if (!(mbar_wait(kv_full, li & 1, p.status) &&
                      mbar_wait(&qs_full[g & 1], (g >> 1) & 1, p.status)))
                    break;
                // S^T held the previous item's last P^T, read by its dV; dP^T its last
                // dS^T, read by its dK: both were issued before
                tc_fence_after();
                mma_ss<D>(T_S, ka, qa(g));     // S^T_0 = K Q_0^T
                tc_commit(s_full);
                mma_ss<D>(T_dP, va, oa(g));    // dP^T_0 = V dO_0^T
                tc_commit(dp_full);
                if (steps == 1) tc_commit(kv_empty);
                for (int t = 0; ok && t < steps; ++t) {
                    const int gt = g + t;
                    const bool more = t + 1 < steps;
                    if (!mbar_wait(p_full, gt & 1, p.status)) { ok = false; break; }
                    // the item's first dV / dK overwrite the accumulators: the previous
                    // item's epilogue must have read them
                    if (t == 0 && li > 0 && !mbar_wait(dkv_free, (li - 1) & 1, p.status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    mma_ts<D>(T_dV, T_S, oa(gt), t != 0);    // dV += P^T dO
                    if (more) {
                        // S^T_{t+1} overwrites P^T_t, which dV_t reads: tcgen05.mma operations
                        // issued by one thread execute in issue order, so no wait is needed
                        if (!mbar_wait(&qs_full[(gt + 1) & 1], ((gt + 1) >> 1) & 1, p.status)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        mma_ss<D>(T_S, ka, qa(gt + 1));
                        tc_commit(s_full);
                    }
                    if (!mbar_wait(ds_full, gt & 1, p.status)) { ok = false; break; }
                    tc_fence_after();
                    mma_ts<D>(T_dK, T_dP, qa(gt), t != 0);   // dK += dS^T Q
                    tc_commit(dk_done);
                    tc_commit(&qs_empty[gt & 1]);
                    if (more) {   // dP^T_{t+1} over dS^T_t, after dK_t in issue order
                        mma_ss<D>(T_dP, va, oa(gt + 1));
                        tc_commit(dp_full);
                        if (t + 2 == steps) tc_commit(kv_empty);   // the item's last S^T / dP^T
                    }
                }
                g += steps;
                ++li;
            }
            tc_commit(drain);
            mbar_wait(drain, 0, p.status);
        }
    }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegEw));
        // ---------------------------------------------------- element-wise
        // Two warps per lane quadrant: `half` takes query columns [64 half, 64 half + 64)
        // of the tile.  P^T / dS^T of half 0 are packed into TMEM columns [0, 32) of
        // their region, of half 1 into [96, 128), so each half overwrites only columns
        // it has already read itself (mma_ts reads that layout).
        const int quad = warp & 3, half = (warp - 4) >> 2;
        const int tid = threadIdx.x - 128;            // 0..255
        const int kr = quad * 32 + lane;              // key row == TMEM lane
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        const uint32_t src_col = half * 64, dst_col = half ? 96 : 0;
        const uint64_t c2 = f2pack(p.scale_log2, p.scale_log2);
        int gs = 0;   // steps before this item
        bool ok = true;
        for (int k = 0; ok; ++k) {
        int bh_kv, jt;
        const int st = item_at(k, bh_kv, jt);
        if (st == 0) break;
        if (st == 2) continue;
        const int b = bh_kv / p.Hkv, hk = bh_kv % p.Hkv;
        const int kj = jt * BT + kr;
        const int i_lo = first_tile(jt);
        const int per_head = max(0, n_qt - i_lo);
        const int steps = G * per_head;
        __nv_bfloat16* dk_row = static_cast<__nv_bfloat16*>(p.dk) + ((int64_t)bh_kv * p.S_kv + (kj < p.S_kv ? kj : 0)) * D;
        __nv_bfloat16* dv_row = static_cast<__nv_bfloat16*>(p.dv) + ((int64_t)bh_kv * p.S_kv + (kj < p.S_kv ? kj : 0)) * D;
        if (steps == 0) {   // no query sees these keys: dK = dV = 0, no barriers
            if (kj < p.S_kv) {
                store_zero_row<D>(dk_row, half);
                store_zero_row<D>(dv_row, half);
            }
            continue;
        }
        // -lse2 / -Delta of query `tid` of step t's tile (threads tid < 128)
        auto fetch = [&](int t, float& nl2, float& ndl) {
            const int gq = t / per_head, it = i_lo + t % per_head;
            const int q = it * BT + tid;
            const int64_t row = (int64_t)(b * p.Hq + hk * G + gq) * p.S_q + q;
            const float lse = q < p.S_q ? p.lse[row] : -INFINITY;
            nl2 = lse == -INFINITY ? -INFINITY : -lse * kLog2e;   // -inf: the column's P is 0
            ndl = q < p.S_q ? -p.delta[row] : 0.0f;
        };
        float nl2 = 0.0f, ndl = 0.0f;
        if (tid < BT) fetch(0, nl2, ndl);
        for (int t = 0; t < steps; ++t) {
            const int gt = gs + t;
            // [-lse2 | -Delta] of this step's query tile; a buffer is rewritten two
            // steps later, after all 256 threads have posted the step in between (so
            // every thread has finished reading this one)
            float* cl = cols + (gt & 1) * 2 * BT;
            if (tid < BT) {
                cl[tid] = nl2;
                cl[BT + tid] = ndl;
            }
            mbar_arrive(&cols_ready[gt & 1]);
            if (!mbar_wait_warp(&cols_ready[gt & 1], (gt >> 1) & 1, p.status)) { ok = false; break; }
            if (t + 1 < steps && tid < BT) fetch(t + 1, nl2, ndl);
            // key kj sees query q iff kj <= q + causal_offset: this half's columns
            // e < lo are masked (q = q0 + e)
            const int q0 = (i_lo + t % per_head) * BT + half * 64;
            int lo = 0;
            if (kj >= p.S_kv) lo = 64;
            else if (p.causal) lo = min(64, max(0, kj - p.causal_offset - q0));
            const bool dense = __all_sync(0xffffffffu, lo == 0);
            const float* hcl = cl + half * 64;
            // phase P (needs S^T only): P^T = exp2(S^T c - lse2), kept as bf16 pairs
            if (!mbar_wait_warp(s_full, gt & 1, p.status)) { ok = false; break; }
            tc_fence_after();
            uint32_t sv[2][32];
            __syncwarp();
            tmem_ld_32x32b_x32(T_S + lane_base + src_col, sv[0]);
            tmem_ld_32x32b_x32(T_S + lane_base + src_col + 32, sv[1]);
            tmem_ld_wait();
            uint32_t pw[32];
#pragma unroll
            for (int e = 0; e < 64; e += 4) {
                const float4 l4 = *reinterpret_cast<const float4*>(hcl + e);
#pragma unroll
                for (int u = 0; u < 4; u += 2) {
                    const int ee = e + u;
                    const uint64_t x2 = ffma2(f2pack(__uint_as_float(sv[ee >> 5][ee & 31]),
                                                     __uint_as_float(sv[ee >> 5][(ee & 31) + 1])),
                                              c2, u ? f2pack(l4.z, l4.w) : f2pack(l4.x, l4.y));
                    float x0, x1;
                    f2unpack(x2, x0, x1);
                    if (!dense) {
                        x0 = ee >= lo ? x0 : -INFINITY;
                        x1 = ee + 1 >= lo ? x1 : -INFINITY;
                    }
                    pw[ee >> 1] = f32x2_to_bf16x2(ex2_approx(x0), ex2_approx(x1));
                }
            }
            tmem_st_32x32b_x32(T_S + lane_base + dst_col, pw);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
            // phase dS (needs dP^T): dS^T = P^T (dP^T - Delta) back over dP^T
            if (!mbar_wait_warp(dp_full, gt & 1, p.status)) { ok = false; break; }
            tc_fence_after();
            __syncwarp();
            tmem_ld_32x32b_x32(T_dP + lane_base + src_col, sv[0]);
            tmem_ld_32x32b_x32(T_dP + lane_base + src_col + 32, sv[1]);
            tmem_ld_wait();
            uint32_t dw[32];
#pragma unroll
            for (int e = 0; e < 64; e += 4) {
                const float4 d4 = *reinterpret_cast<const float4*>(hcl + BT + e);
#pragma unroll
                for (int u = 0; u < 4; u += 2) {
                    const int ee = e + u;
                    const uint32_t pp = pw[ee >> 1];
                    const uint64_t g2 = fadd2(f2pack(__uint_as_float(sv[ee >> 5][ee & 31]),
                                                     __uint_as_float(sv[ee >> 5][(ee & 31) + 1])),
                                              u ? f2pack(d4.z, d4.w) : f2pack(d4.x, d4.y));
                    float d0, d1;
                    f2unpack(fmul2(f2pack(bf16_lo(pp), bf16_hi(pp)), g2), d0, d1);
                    dw[ee >> 1] = f32x2_to_bf16x2(d0, d1);
                }
            }
            tmem_st_32x32b_x32(T_dP + lane_base + dst_col, dw);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(ds_full);
        }

        // epilogue: dK = scale * acc, dV = acc (each half stores half of the columns)
        if (ok && !mbar_wait_warp(dk_done, (gs + steps - 1) & 1, p.status)) ok = false;
        if (!ok) break;
        tc_fence_after();
        store_row<D>(T_dK + lane_base, p.scale, dk_row, kj < p.S_kv, half);
        store_row<D>(T_dV + lane_base, 1.0f, dv_row, kj < p.S_kv, half);
        // both accumulators are read out of TMEM: the next item's dV / dK may run
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dkv_free);
        gs += steps;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------- dQ
// One persistent CTA per SM walks units of two (batch * query head, 128-query tile)
// items of one head: tile n_qt-1-q (the heaviest under a causal mask) and tile q, so
// units of a causal square problem carry the same work.  K/V tiles, S buffers and
// the per-step barriers count on across items (step g of the CTA: ring stage and
// S buffer g & 1); Q/dO reload once the item's last dP has been issued (q_empty),
// and an item's first dQ MMA waits for the previous item's epilogue to have read
// dQ out of TMEM (dq_free).
template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    k_fa_bwd_dq(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                const BwdParams p) {
    pdl_wait();
    pdl_trigger();
    using CF = BwdCfg<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint8_t* q_s = smem;                          // Q_i
    uint8_t* o_s = q_s + CF::TILE;                // dO_i
    uint8_t* k_s = o_s + CF::TILE;                // [2][K_j]
    uint8_t* v_s = k_s + 2 * CF::TILE;            // [2][V_j]
    uint64_t* bars = reinterpret_cast<uint64_t*>(v_s + 2 * CF::TILE);
    uint64_t* q_full = bars;
    uint64_t* k_full = bars + 1;      // [2]
    uint64_t* k_empty = bars + 3;     // [2]
    uint64_t* v_full = bars + 5;      // [2]
    uint64_t* v_empty = bars + 7;     // [2]
    uint64_t* s_full = bars + 9;      // [2]: S of step g in TMEM buffer g & 1
    uint64_t* dp_full = bars + 11;
    uint64_t* ds_full = bars + 12;
    uint64_t* dq_done = bars + 13;    // dQ has read dS: dP may be rewritten
    uint64_t* drain = bars + 14;
    uint64_t* q_empty = bars + 15;    // the item's last MMA reading Q / dO has completed
    uint64_t* dq_free = bars + 16;    // the item's epilogue has read dQ out of TMEM
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_qt = (p.S_q + BT - 1) / BT;
    const int half_units = (n_qt + 1) / 2;
    const int units = p.B * p.Hq * half_units;
    // k-th item of this CTA: 0 = no more, 1 = item (bh, it), 2 = empty slot
    auto item_at = [&](int k, int& bh, int& it) -> int {
        const int u = (int)blockIdx.x + (k >> 1) * (int)gridDim.x;
        if (u >= units) return 0;
        bh = u / half_units;
        const int q = u % half_units;
        it = (k & 1) ? q : n_qt - 1 - q;
        return ((k & 1) && q == n_qt - 1 - q) ? 2 : 1;
    };
    auto kv_tiles = [&](int it) {
        int n_kv = (p.S_kv + BT - 1) / BT;
        if (p.causal) {
            const int last = it * BT + BT - 1 + p.causal_offset;
            n_kv = min(n_kv, last < 0 ? 0 : last / BT + 1);
        }
        return n_kv;
    };

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        mbar_init(dq_free, 8);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        mbar_init(&s_full[0], 1);
        mbar_init(&s_full[1], 1);
        mbar_init(dp_full, 1);
        mbar_init(ds_full, 8);
        mbar_init(dq_done, 1);
        mbar_init(drain, 1);
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // two S buffers, so that the next step's S = Q K^T runs during this step
    const uint32_t T_S = tmem, T_dP = tmem + 2 * BT, T_dQ = tmem + 3 * BT;

    if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegCtl));
    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            int g = 0, li = 0;   // K/V tiles loaded; items with work loaded
            bool ok = true;
            for (int k = 0; ok; ++k) {
                int bh, it;
                const int st = item_at(k, bh, it);
                if (st == 0) break;
                const int n_kv = st == 1 ? kv_tiles(it) : 0;
                if (n_kv == 0) continue;
                const int b = bh / p.Hq, h = bh % p.Hq;
                const int bh_kv = b * p.Hkv + h / (p.Hq / p.Hkv);
                if (li > 0 && !mbar_wait(q_empty, (li - 1) & 1, p.status)) break;
                mbar_arrive_expect_tx(q_full, 2 * CF::TILE);
#pragma unroll
                for (int sl = 0; sl < CF::SLABS; ++sl) {
                    tma_load_3d(q_s + sl * SLAB_BYTES, &tmQ, q_full, sl * 64, it * BT, bh);
                    tma_load_3d(o_s + sl * SLAB_BYTES, &tmdO, q_full, sl * 64, it * BT, bh);
                }
                for (int j = 0; j < n_kv; ++j, ++g) {
                    const int s = g & 1;
                    const uint32_t ph = ((g >> 1) & 1) ^ 1;
                    if (!mbar_wait(&k_empty[s], ph, p.status)) { ok = false; break; }
                    mbar_arrive_expect_tx(&k_full[s], CF::TILE);
#pragma unroll
                    for (int sl = 0; sl < CF::SLABS; ++sl)
                        tma_load_3d(k_s + s * CF::TILE + sl * SLAB_BYTES, &tmK, &k_full[s],
                                    sl * 64, j * BT, bh_kv);
                    if (!mbar_wait(&v_empty[s], ph, p.status)) { ok = false; break; }
                    mbar_arrive_expect_tx(&v_full[s], CF::TILE);
#pragma unroll
                    for (int sl = 0; sl < CF::SLABS; ++sl)
                        tma_load_3d(v_s + s * CF::TILE + sl * SLAB_BYTES, &tmV, &v_full[s],
                                    sl * 64, j * BT, bh_kv);
                }
                ++li;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // tensor-core order per step j:  S_{j+1}, dQ_j, dP_{j+1}
            const uint32_t qa0 = smem_u32(q_s), oa0 = smem_u32(o_s);
            auto ka = [&](int g) { return opaque_u32(smem_u32(k_s + (g & 1) * CF::TILE)); };
            auto va = [&](int g) { return opaque_u32(smem_u32(v_s + (g & 1) * CF::TILE)); };
            int g = 0, li = 0;   // steps before this item; items with work before it
            bool ok = true;
            for (int k = 0; ok; ++k) {
                int bh, it;
                const int st = item_at(k, bh, it);
                if (st == 0) break;
                const int n_kv = st == 1 ? kv_tiles(it) : 0;
                if (n_kv == 0) continue;
                const uint32_t qa = opaque_u32(qa0), oa = opaque_u32(oa0);
                const int s0 = g & 1;
                const uint32_t ph0 = (g >> 1) & 1;
                if (!(mbar_wait(q_full, li & 1, p.status) && mbar_wait(&k_full[s0], ph0, p.status) &&
                      mbar_wait(&v_full[s0], ph0, p.status)))
                    break;
                // S buffer s0 held S of step g-2, read before ds_full(g-2); dP held the
                // previous item's last dS, read by its dQ, issued before
                tc_fence_after();
                mma_ss<D>(T_S + s0 * BT, qa, ka(g));     // S_0 = Q K_0^T
                tc_commit(&s_full[s0]);
                mma_ss<D>(T_dP, oa, va(g));              // dP_0 = dO V_0^T
                tc_commit(&v_empty[s0]);
                tc_commit(dp_full);
                if (n_kv == 1) tc_commit(q_empty);
                for (int j = 0; ok && j < n_kv; ++j) {
                    const int gj = g + j;
                    const bool more = j + 1 < n_kv;
                    const int n1 = (gj + 1) & 1;
                    const uint32_t ph1 = ((gj + 1) >> 1) & 1;
                    if (more) {   // S buffer n1 held S of step gj-1, read before ds_full(gj-1)
                        if (!mbar_wait(&k_full[n1], ph1, p.status)) { ok = false; break; }
                        tc_fence_after();
                        mma_ss<D>(T_S + n1 * BT, qa, ka(gj + 1));
                        tc_commit(&s_full[n1]);
                    }
                    if (!mbar_wait(ds_full, gj & 1, p.status)) { ok = false; break; }
                    // the item's first dQ overwrites the accumulator: the previous
                    // item's epilogue must have read it
                    if (j == 0 && li > 0 && !mbar_wait(dq_free, (li - 1) & 1, p.status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    mma_ts<D>(T_dQ, T_dP, ka(gj), j != 0);   // dQ += dS K
                    tc_commit(dq_done);
                    tc_commit(&k_empty[gj & 1]);
                    if (more) {   // dP_{j+1} over dS_j, after dQ_j in issue order
                        if (!mbar_wait(&v_full[n1], ph1, p.status)) { ok = false; break; }
                        tc_fence_after();
                        mma_ss<D>(T_dP, oa, va(gj + 1));
                        tc_commit(&v_empty[n1]);
                        tc_commit(dp_full);
                        if (j + 2 == n_kv) tc_commit(q_empty);   // the item's last dP
                    }
                }
                g += n_kv;
                ++li;
            }
            tc_commit(drain);
            mbar_wait(drain, 0, p.status);
        }
    }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegEw));
        // ---------------------------------------------------- element-wise
        // Two warps per lane quadrant: `half` takes key columns [64 half, 64 half + 64);
        // dS of half 0 is packed into TMEM columns [0, 32) of the dP region, of half 1
        // into [96, 128) (the layout mma_ts reads).
        const int quad = warp & 3, half = (warp - 4) >> 2;
        const int r = quad * 32 + lane;               // query row == TMEM lane
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        const uint32_t src_col = half * 64, dst_col = half ? 96 : 0;
        const uint64_t c2 = f2pack(p.scale_log2, p.scale_log2);
        int g = 0;   // steps before this item
        bool ok = true;
        for (int k = 0; ok; ++k) {
        int bh, it;
        const int st = item_at(k, bh, it);
        if (st == 0) break;
        if (st == 2) continue;
        const int n_kv = kv_tiles(it);
        const int qi = it * BT + r;
        const int64_t row = (int64_t)bh * p.S_q + qi;
        __nv_bfloat16* dq_row = static_cast<__nv_bfloat16*>(p.dq) + ((int64_t)bh * p.S_q + (qi < p.S_q ? qi : 0)) * D;
        if (n_kv == 0) {   // no visible key: dQ = 0, no barriers
            if (qi < p.S_q) store_zero_row<D>(dq_row, half);
            continue;
        }
        const float lse = qi < p.S_q ? p.lse[row] : -INFINITY;
        const float nl2 = lse == -INFINITY ? -INFINITY : -lse * kLog2e;   // -inf: P = 0
        const float ndl = qi < p.S_q ? -p.delta[row] : 0.0f;
        const uint64_t nl2x2 = f2pack(nl2, nl2), ndlx2 = f2pack(ndl, ndl);
        const int vis_hi = p.causal ? min(p.S_kv - 1, qi + p.causal_offset) : p.S_kv - 1;
        for (int j = 0; j < n_kv; ++j) {
            const int gj = g + j;
            // this half's key columns e > hi are masked
            const int hi = vis_hi - (j * BT + half * 64);
            const bool dense = __all_sync(0xffffffffu, hi >= 63);
            // phase P (needs S only), kept in registers as bf16 pairs
            if (!mbar_wait_warp(&s_full[gj & 1], (gj >> 1) & 1, p.status)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sb = T_S + (gj & 1) * BT;
            uint32_t sv[2][32];
            __syncwarp();
            tmem_ld_32x32b_x32(sb + lane_base + src_col, sv[0]);
            tmem_ld_32x32b_x32(sb + lane_base + src_col + 32, sv[1]);
            tmem_ld_wait();
            uint32_t pw[32];
#pragma unroll
            for (int e = 0; e < 64; e += 2) {
                const uint64_t x2 = ffma2(f2pack(__uint_as_float(sv[e >> 5][e & 31]),
                                                 __uint_as_float(sv[e >> 5][(e & 31) + 1])),
                                          c2, nl2x2);
                float x0, x1;
                f2unpack(x2, x0, x1);
                if (!dense) {
                    x0 = e <= hi ? x0 : -INFINITY;
                    x1 = e + 1 <= hi ? x1 : -INFINITY;
                }
                pw[e >> 1] = f32x2_to_bf16x2(ex2_approx(x0), ex2_approx(x1));
            }
            // phase dS (needs dP): dS = P (dP - Delta) back over dP
            if (!mbar_wait_warp(dp_full, gj & 1, p.status)) { ok = false; break; }
            tc_fence_after();
            __syncwarp();
            tmem_ld_32x32b_x32(T_dP + lane_base + src_col, sv[0]);
            tmem_ld_32x32b_x32(T_dP + lane_base + src_col + 32, sv[1]);
            tmem_ld_wait();
            uint32_t dw[32];
#pragma unroll
            for (int e = 0; e < 64; e += 2) {
                const uint32_t pp = pw[e >> 1];
                const uint64_t g2 = fadd2(f2pack(__uint_as_float(sv[e >> 5][e & 31]),
                                                 __uint_as_float(sv[e >> 5][(e & 31) + 1])),
                                          ndlx2);
                float d0, d1;
                f2unpack(fmul2(f2pack(bf16_lo(pp), bf16_hi(pp)), g2), d0, d1);
                dw[e >> 1] = f32x2_to_bf16x2(d0, d1);
            }
            tmem_st_32x32b_x32(T_dP + lane_base + dst_col, dw);   // dS over dP
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(ds_full);
        }
        if (ok && !mbar_wait_warp(dq_done, (g + n_kv - 1) & 1, p.status)) ok = false;
        if (!ok) break;
        tc_fence_after();
        store_row<D>(T_dQ + lane_base, p.scale, dq_row, qi < p.S_q, half);
        // store_row has read this half of dQ out of TMEM: the next item's dQ may run
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dq_free);
        g += n_kv;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

template <int D>
int launch_bwd(const void* Q, const void* K, const void* V, const void* O, const void* dO,
               const float* lse, void* dQ, void* dK, void* dV, float* delta, int B, int Hq,
               int Hkv, int S_q, int S_kv, int causal, float scale, cudaStream_t st) {
    using CF = BwdCfg<D>;
    CUtensorMap tq, tk, tv, to;
    int rc;
    if ((rc = fa_make_tmap_3d(&tq, Q, D, S_q, (int64_t)B * Hq))) return rc;
    if ((rc = fa_make_tmap_3d(&to, dO, D, S_q, (int64_t)B * Hq))) return rc;
    if ((rc = fa_make_tmap_3d(&tk, K, D, S_kv, (int64_t)B * Hkv))) return rc;
    if ((rc = fa_make_tmap_3d(&tv, V, D, S_kv, (int64_t)B * Hkv))) return rc;
    int* status = nullptr;
    if ((rc = device_status(&status))) return rc;
    BwdParams p;
    p.B = B;
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.S_q = S_q;
    p.S_kv = S_kv;
    p.causal = causal;
    p.causal_offset = 0;
    p.scale = scale;
    p.scale_log2 = scale * kLog2e;
    p.lse = lse;
    p.delta = delta;
    p.dq = dQ;
    p.dk = dK;
    p.dv = dV;
    p.status = status;
    const int64_t rows = (int64_t)B * Hq * S_q;
    const int64_t delta_rows_per_block = 8 * (32 / (D / 8)) * kDeltaLoads;
    const int dgrid = (int)std::min<int64_t>((rows + delta_rows_per_block - 1) / delta_rows_per_block,
                                             (int64_t)sm_count() * 8);
    AMPB_CHECK_CUDA(launch_pdl(k_fa_bwd_delta<D>, dim3(dgrid), dim3(256), 0, st,
                               static_cast<const __nv_bfloat16*>(O),
                               static_cast<const __nv_bfloat16*>(dO), delta, rows));
    constexpr int SMEM_KV = 6 * CF::TILE + 2 * 2 * BT * 4 + 1024 + 256;
    constexpr int SMEM_Q = 6 * CF::TILE + 1024 + 256;
    static std::atomic<uint64_t> attr_done{0};
    int dev = 0;
    AMPB_CHECK_CUDA(cudaGetDevice(&dev));
    if (dev >= 64 || !(attr_done.load() >> dev & 1)) {
        AMPB_CHECK_CUDA(cudaFuncSetAttribute(k_fa_bwd_dkdv<D>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_KV));
        AMPB_CHECK_CUDA(cudaFuncSetAttribute(k_fa_bwd_dq<D>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_Q));
        if (dev < 64) attr_done.fetch_or(1ull << dev);
    }
    // dK/dV: one persistent CTA per SM over units of two key tiles (k_fa_bwd_dkdv)
    const int64_t kv_units = (int64_t)B * Hkv * (((S_kv + BT - 1) / BT + 1) / 2);
    AMPB_REQUIRE(kv_units <= INT32_MAX / 2, AMP_ERR_UNSUPPORTED, "attention too large");
    AMPB_CHECK_CUDA(launch_pdl(k_fa_bwd_dkdv<D>, dim3((unsigned)std::min<int64_t>(kv_units, sm_count())),
                               dim3(kThreads), SMEM_KV, st, tq, tk, tv, to, p));
    // dQ: one persistent CTA per SM over units of two query tiles (k_fa_bwd_dq)
    const int64_t dq_units = (int64_t)B * Hq * (((S_q + BT - 1) / BT + 1) / 2);
    AMPB_REQUIRE(dq_units <= INT32_MAX / 2, AMP_ERR_UNSUPPORTED, "attention too large");
    AMPB_CHECK_CUDA(launch_pdl(k_fa_bwd_dq<D>, dim3((unsigned)std::min<int64_t>(dq_units, sm_count())),
                               dim3(kThreads), SMEM_Q, st, tq, tk, tv, to, p));
    return AMP_OK;
}

}  // namespace

size_t fa_bwd_ws_bytes(int B, int Hq, int S_q) { return (size_t)B * Hq * S_q * 4 + 256; }

int flash_attn_bwd_dev(const void* Q, const void* K, const void* V, const void* O, const void* dO,
                       const float* lse, void* dQ, void* dK, void* dV, int B, int Hq, int Hkv,
                       int S_q, int S_kv, int D, int causal, float scale, void* ws,
                       size_t ws_bytes, cudaStream_t st) {
    AMPB_REQUIRE(B > 0 && Hq > 0 && Hkv > 0 && S_q > 0 && S_kv > 0, AMP_ERR_INVALID,
                 "attention sizes must be positive");
    AMPB_REQUIRE(Hq % Hkv == 0, AMP_ERR_INVALID, "num_q_heads (%d) must be a multiple of "
                 "num_kv_heads (%d)", Hq, Hkv);
    AMPB_REQUIRE(Q && K && V && O && dO && lse && dQ && dK && dV && ws, AMP_ERR_INVALID,
                 "NULL tensor");
    AMPB_REQUIRE(aligned16(Q) && aligned16(K) && aligned16(V) && aligned16(O) && aligned16(dO) &&
                     aligned16(dQ) && aligned16(dK) && aligned16(dV),
                 AMP_ERR_INVALID, "tensors must be 16-byte aligned");
    AMPB_REQUIRE(!causal || S_q == S_kv, AMP_ERR_UNSUPPORTED,
                 "causal backward needs S_q == S_kv (top-left aligned mask)");
    AMPB_REQUIRE((int64_t)B * Hq <= 65535, AMP_ERR_UNSUPPORTED, "B*Hq must be <= 65535");
    AMPB_REQUIRE(ws_bytes >= fa_bwd_ws_bytes(B, Hq, S_q), AMP_ERR_INVALID,
                 "workspace too small: %zu < %zu", ws_bytes, fa_bwd_ws_bytes(B, Hq, S_q));
    AMPB_REQUIRE((reinterpret_cast<uintptr_t>(ws) & 15u) == 0, AMP_ERR_INVALID,
                 "workspace must be 16-byte aligned");
    if (!(scale > 0.0f)) scale = 1.0f / sqrtf((float)D);
    float* delta = static_cast<float*>(ws);
    switch (D) {
        case 128:
            return launch_bwd<128>(Q, K, V, O, dO, lse, dQ, dK, dV, delta, B, Hq, Hkv, S_q, S_kv,
                                   causal, scale, st);
        case 64:
            return launch_bwd<64>(Q, K, V, O, dO, lse, dQ, dK, dV, delta, B, Hq, Hkv, S_q, S_kv,
                                  causal, scale, st);
        default:
            set_error(AMP_ERR_UNSUPPORTED, "flash_attn backward: head_dim %d not supported (64, 128)", D);
            return AMP_ERR_UNSUPPORTED;
    }
}

}  // namespace ampb

using namespace ampb;

extern "C" {

size_t amp_flash_attn_bwd_workspace_bytes(int B, int Hq, int S_q) {
    return fa_bwd_ws_bytes(B, Hq, S_q);
}

int amp_flash_attn_bwd_bf16_dev(const void* Q, const void* K, const void* V, const void* O,
                                const void* dO, const float* lse, void* dQ, void* dK, void* dV,
                                int B, int Hq, int Hkv, int S_q, int S_kv, int head_dim,
                                int causal, float scale, void* workspace, size_t workspace_bytes,
                                void* stream) {
    return flash_attn_bwd_dev(Q, K, V, O, dO, lse, dQ, dK, dV, B, Hq, Hkv, S_q, S_kv, head_dim,
                              causal, scale, workspace, workspace_bytes, as_stream(stream));
}

}  // extern "C"
