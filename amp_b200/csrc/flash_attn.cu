// flash_attn.cu -- FlashAttention-2 forward (causal / full, GQA) on tcgen05.
//
// Replaces flash_attn_fwd_kernel<Br,Bc,D> and dispatch_flash_attn
// (kernels/flash_attn.cu:73-283 of the reference: one warp per query row,
// scalar fp32 dot products repeated by every lane, fp32 shared-memory tiles).
// Same contract: Q,O [B,Hq,S_q,D] bf16, K,V [B,Hkv,S_kv,D] bf16, lse [B,Hq,S_q]
// fp32 = ln(sum_j exp(scale * q.k_j)); kv head = hq / (Hq/Hkv)
// (flash_attn.cu:90); causal masks key j > query i (top-left aligned,
// flash_attn.cu:134,152) -- generalised here by an offset so that paged
// prefill can use bottom-right alignment (key j visible iff j <= i + offset).
//
// Work items are (batch*head, pair of 128-row query tiles).  The dense forward
// runs one persistent CTA per SM over units of two items of one head (the
// heaviest and the lightest pair left under a causal mask, so units weigh the
// same); the barriers' phases run on across items, the load warp fetches the
// next item's Q and K/V while the current one finishes, and the next item's first
// QK_0 is issued as soon as query tile 0 has finished.  The paged and all-gather
// forms run one CTA per item.  384 threads in three warpgroups (setmaxnreg: 72
// registers for the first, 216 for the softmax ones):
//   warp 0     TMA: both Q tiles of each item; K and V tiles (128 rows) into separate
//              2-stage rings (128-byte swizzle, 3-D maps so each head's tail is
//              zero-filled; 4-D page-gather maps for paged K/V).
//   warp 1     TMEM (512 columns: S0 | S1 | O0 | O1) and one MMA-issuing lane.
//              Per K/V tile j and query tile t: O_t += P_t,j V_j (TS form: P
//              read from TMEM, V MN-major from shared memory), then at once
//              S_t = Q_t K_{j+1}^T (SS form) into the columns P_t,j occupies:
//              MMAs issued by one thread execute in issue order, so the PV has
//              read P before the QK overwrites it.  The two tiles' chains S -> softmax -> P -> PV -> S are
//              offset by half a step, so the tensor core works on one tile
//              while the other tile's softmax runs.
//   warps 2-3  idle (they only hand their registers to the softmax warps).
//   warps 4-7  softmax of query tile 0, warps 8-11 of query tile 1; one query
//              row per thread: tcgen05.ld the S row, mask, online max in the
//              log2 domain (scale * log2(e) folded into one packed f32x2 FMA
//              per two scores), ex2, row sum in fp32 (independent accumulator
//              chains), P packed to bf16 and tcgen05.st back over S.  O is
//              rescaled (tcgen05.ld/st) only when a row maximum grows by more
//              than 2^8; otherwise the stale maximum is kept.
//              Epilogue: O / l to bf16, lse = (m + log2 l) * ln 2.
//
// All-gather mode ((batch*head)-sharded attention on the GPUs of one node: the
// reference's launch + ncclAllGather of O / lse, include/collective.hpp:87-89):
// each softmax warp stages its 32 output rows in the tile's Q buffer (free once
// the tile's last MMA has completed) and writes them -- contiguous in O -- to
// every rank's O, then its lse values; when all softmax warps on the GPU are
// done (system-scope fence + counter), the last one exchanges this launch's
// sequence number with every rank through the peer mailboxes (bounded wait).
#include <cuda.h>

#include <cmath>

#include "common.cuh"
#include "peer.cuh"
#include "runtime.h"
#include "tc_common.cuh"

namespace ampb {

int fa_make_tmap_3d(CUtensorMap* m, const void* base, int64_t d, int64_t s, int64_t bh);
int fa_make_tmap_pool(CUtensorMap* m, const void* base, int64_t d, int64_t hkv, int64_t pages);

namespace {

constexpr int BQ = 128;            // query rows per tile (two tiles per CTA)
constexpr int BKV = 128;           // key/value rows per tile
constexpr int KV_STAGES = 2;
constexpr int kThreads = 384;      // 3 warpgroups
// Register split between the control warpgroup and the two softmax warpgroups;
// it must not exceed what the launch holds: 128*72 + 256*216 == 384*168, and the
// kernel is compiled for exactly 168 registers a thread (__launch_bounds__(384, 1)).
constexpr int kRegCtl = 72, kRegSoftmax = 216;
constexpr int SLAB_BYTES = 128 * 128;  // [128 rows x 128 bytes] swizzled slab
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct FaParams {
    int B, Hq, Hkv, S_q, S_kv;
    int causal;
    int causal_offset;   // key j visible for query i iff j <= i + causal_offset
    float scale_log2;    // softmax scale * log2(e)
    void* O;
    float* lse;
    int* status;
    // paged K/V (prefill): pools [num_pages][Hkv][16][D], table [B][max_pages]
    const int* block_table;
    const int* ctx_lens;
    int max_pages, num_pages;
    // all-gather mode: every rank's O ([bh_total][S_q][D] bf16) and lse; this
    // launch's (batch*head) 0 is global index bh_base
    void* const* o_peers;
    float* const* lse_peers;
    int world, rank, bh_base;
    unsigned long long* const* mbox;
    unsigned seq;
    unsigned* done;
};

// Softmax warps of the all-gather attention that have stored their rows; one
// counter per device (one all-gather attention launch in flight per device).
__device__ unsigned g_fa_allgather_done;

constexpr int kPageTokens = 16;

__device__ __forceinline__ float lg2_approx(float x) {
    float y;
    asm("lg2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

template <int D>
struct FaCfg {
    static constexpr int SLABS = D / 64;
    static constexpr int TILE = SLABS * SLAB_BYTES;
    static constexpr int SMEM = 2 * TILE + KV_STAGES * 2 * TILE + 1024 + 256;
    static constexpr uint32_t IDESC_QK = make_idesc(1, 1, 0, 0, BQ, BKV);
    static constexpr uint32_t IDESC_PV = make_idesc(1, 1, 0, 1, BQ, D);
    static constexpr uint32_t O_COL = 2 * BKV;            // S0 | S1 | O0 | O1
};

// kPersist: one CTA per SM walks a list of (batch*head, query-tile pair) items
// (see item_at below) instead of one CTA per item, so that the next item's Q and
// K/V loads and its first QK overlap the current item's last steps and epilogue.
template <int D, bool kPaged, bool kAllGather = false, bool kPersist = false>
__global__ void __launch_bounds__(kThreads, 1)
    k_flash_fwd(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
           const __grid_constant__ CUtensorMap tmV, const FaParams p) {
    static_assert(!(kPersist && kAllGather), "the all-gather epilogue stages in Q: one item per CTA");
    using CF = FaCfg<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint8_t* q_s = smem;                        // [2][TILE]
    uint8_t* k_s = q_s + 2 * CF::TILE;          // [KV_STAGES][TILE]
    uint8_t* v_s = k_s + KV_STAGES * CF::TILE;        // [KV_STAGES][TILE]
    uint64_t* bars = reinterpret_cast<uint64_t*>(v_s + KV_STAGES * CF::TILE);
    uint64_t* q_full = bars;             // [2] per query tile
    uint64_t* q_empty = q_full + 2;      // [2] the item's last QK_t has read Q_t
    uint64_t* k_full = q_empty + 2;
    uint64_t* k_empty = k_full + KV_STAGES;
    uint64_t* v_full = k_empty + KV_STAGES;
    uint64_t* v_empty = v_full + KV_STAGES;
    uint64_t* s_full = v_empty + KV_STAGES;   // [2] per query tile
    uint64_t* p_full = s_full + 2;      // [2]
    uint64_t* pv_done = p_full + 2;     // [2]
    uint64_t* o_free = pv_done + 2;     // [2] the epilogue has read O_t out of TMEM
    uint64_t* drain = o_free + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_qb = (p.S_q + 2 * BQ - 1) / (2 * BQ);
    // Items of this CTA, k = 0, 1, ...: 0 = no more, 1 = item (bh, qb), 2 = empty slot.
    // Persistent: unit u = blockIdx.x + (k/2) * gridDim.x pairs query-tile pair
    // n_qb-1-q (heaviest under a causal mask) with pair q of the same head, so every
    // unit of a causal square problem carries the same work and consecutive units
    // share a head (K/V stay in L2).  Otherwise the one item of the grid cell.
    const int half = (n_qb + 1) / 2;
    const int units = p.B * p.Hq * half;
    auto item_at = [&](int k, int& bh, int& qb) -> int {
        if constexpr (!kPersist) {
            if (k > 0) return 0;
            bh = blockIdx.y;
            qb = n_qb - 1 - (int)blockIdx.x;
            return 1;
        } else {
            const int u = (int)blockIdx.x + (k >> 1) * (int)gridDim.x;
            if (u >= units) return 0;
            bh = u / half;
            const int q = u % half;
            qb = (k & 1) ? q : n_qb - 1 - q;
            return ((k & 1) && q == n_qb - 1 - q) ? 2 : 1;
        }
    };
    struct Geo {
        int b, h, bh_kv, q0, S_kv, coff, n0, n1;
    };
    auto geo = [&](int bh, int qb) {
        Geo g;
        g.b = bh / p.Hq;
        g.h = bh % p.Hq;
        g.bh_kv = g.b * p.Hkv + g.h / (p.Hq / p.Hkv);
        g.q0 = qb * 2 * BQ;
        g.S_kv = p.S_kv;
        g.coff = p.causal_offset;
        if constexpr (kPaged) {
            g.S_kv = max(0, p.ctx_lens[g.b]);
            g.coff = g.S_kv - p.S_q;
        }
        const int n_all = (g.S_kv + BKV - 1) / BKV;
        auto nblk = [&](int row0) {
            int n = n_all;
            if (p.causal) {
                const int last = row0 + BQ - 1 + g.coff;
                n = min(n, last < 0 ? 0 : last / BKV + 1);
            }
            return max(n, 1);
        };
        g.n0 = nblk(g.q0);
        g.n1 = max(nblk(g.q0 + BQ), g.n0);
        return g;
    };

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&q_full[i], 1);
            mbar_init(&q_empty[i], 1);
            mbar_init(&o_free[i], 4);
        }
        for (int s = 0; s < KV_STAGES; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 4);
            mbar_init(&pv_done[i], 1);
        }
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

    if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegCtl));
    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            // K/V tiles run through the rings continuously across items: tile g of
            // this CTA uses stage g % KV_STAGES in phase (g / KV_STAGES) & 1
            int gkv = 0, li = 0;
            bool ok = true;
            for (int k = 0; ok; ++k) {
                int bh, qb;
                const int st = item_at(k, bh, qb);
                if (st == 0) break;
                if (st == 2) continue;
                const Geo g = geo(bh, qb);
                // Q_t of this item once the previous item's last QK_t has read Q_t.
                // Persistent order: Q_0, K/V 0, Q_1, K/V 1.. -- Q_1 is freed last
                // (tile 1 runs the previous item's last step), and the next item's
                // first QK_0 is issued while it does.  One item: Q_0, Q_1, K/V 0, ...
                auto load_q = [&](int t) {
                    if (li > 0 && !mbar_wait(&q_empty[t], (li - 1) & 1, p.status)) return false;
                    mbar_arrive_expect_tx(&q_full[t], CF::TILE);
#pragma unroll
                    for (int sl = 0; sl < CF::SLABS; ++sl)
                        tma_load_3d(q_s + t * CF::TILE + sl * SLAB_BYTES, &tmQ, &q_full[t],
                                    sl * 64, g.q0 + t * BQ, bh);
                    return true;
                };
                if (!load_q(0)) break;
                if (!kPersist && !load_q(1)) break;
                const int last_page = max(0, (g.S_kv + kPageTokens - 1) / kPageTokens - 1);
                const int hk = g.h / (p.Hq / p.Hkv);
                for (int j = 0; j < g.n1; ++j) {
                    const int s = (gkv + j) % KV_STAGES;
                    const uint32_t ph = ((gkv + j) / KV_STAGES) & 1;
                    int pages[BKV / kPageTokens];
                    if constexpr (kPaged) {
                        const int* bt = p.block_table + (int64_t)g.b * p.max_pages;
#pragma unroll
                        for (int i = 0; i < BKV / kPageTokens; ++i) {
                            const int pg = bt[min(j * (BKV / kPageTokens) + i, last_page)];
                            const bool bad = pg < 0 || pg >= p.num_pages;
                            if (bad && g.S_kv > 0) atomicExch(p.status, AMP_DEV_ERR_BAD_PAGE);
                            pages[i] = bad ? 0 : pg;
                        }
                    }
                    if (!mbar_wait(&k_empty[s], ph ^ 1, p.status)) { ok = false; break; }
                    mbar_arrive_expect_tx(&k_full[s], CF::TILE);
#pragma unroll
                    for (int sl = 0; sl < CF::SLABS; ++sl) {
                        uint8_t* dst = k_s + s * CF::TILE + sl * SLAB_BYTES;
                        if constexpr (kPaged) {
#pragma unroll
                            for (int i = 0; i < BKV / kPageTokens; ++i)
                                tma_load_4d(dst + i * kPageTokens * 128, &tmK, &k_full[s], sl * 64,
                                            0, hk, pages[i]);
                        } else {
                            tma_load_3d(dst, &tmK, &k_full[s], sl * 64, j * BKV, g.bh_kv);
                        }
                    }
                    if (!mbar_wait(&v_empty[s], ph ^ 1, p.status)) { ok = false; break; }
                    mbar_arrive_expect_tx(&v_full[s], CF::TILE);
#pragma unroll
                    for (int sl = 0; sl < CF::SLABS; ++sl) {
                        uint8_t* dst = v_s + s * CF::TILE + sl * SLAB_BYTES;
                        if constexpr (kPaged) {
#pragma unroll
                            for (int i = 0; i < BKV / kPageTokens; ++i)
                                tma_load_4d(dst + i * kPageTokens * 128, &tmV, &v_full[s], sl * 64,
                                            0, hk, pages[i]);
                        } else {
                            tma_load_3d(dst, &tmV, &v_full[s], sl * 64, j * BKV, g.bh_kv);
                        }
                    }
                    if (kPersist && j == 0 && !load_q(1)) { ok = false; break; }
                }
                gkv += g.n1;
                ++li;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t q_addr = smem_u32(q_s);
            // S_t = Q_t K^T (K-major x K-major, 16-deep steps along the head dim)
            auto qk = [&](int t, uint32_t k_addr) {
                const uint32_t qa = opaque_u32(q_addr + t * CF::TILE);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * SLAB_BYTES + (kk & 3) * 32;
                    tc_mma_f16(tmem + t * BKV, smem_desc_sw128(qa + off, 16, 1024),
                               smem_desc_sw128(k_addr + off, 16, 1024), CF::IDESC_QK, kk != 0);
                }
            };
            // gkv: K/V tiles consumed before this item (ring stage / phase as in the
            // load warp); c[t]: query tile t's steps before this item (phase of
            // s_full / p_full / pv_done); li: items before this one (q_full, q_empty,
            // o_free)
            int gkv = 0, li = 0, c[2] = {0, 0};
            bool ok = true, pre0 = false;   // pre0: this item's QK_0 was issued early
            for (int k = 0; ok; ++k) {
                int bh, qb;
                const int st = item_at(k, bh, qb);
                if (st == 0) break;
                if (st == 2) continue;
                const Geo g = geo(bh, qb);
                const int n0 = g.n0, n1 = g.n1;
                // S_t = Q_t K_0^T of this item.  S_t may still hold P_t of the previous
                // item's last step: its PV was issued earlier, and runs first.
                {
                    const int s0 = gkv % KV_STAGES;
                    if (!mbar_wait(&k_full[s0], (gkv / KV_STAGES) & 1, p.status)) break;
                    const uint32_t k_addr = opaque_u32(smem_u32(k_s + s0 * CF::TILE));
#pragma unroll
                    for (int t = 0; t < 2; ++t) {
                        if (t == 0 && pre0) continue;
                        if (!mbar_wait(&q_full[t], li & 1, p.status)) { ok = false; break; }
                        tc_fence_after();
                        qk(t, k_addr);
                        tc_commit(&s_full[t]);
                        if ((t ? n1 : n0) == 1) tc_commit(&q_empty[t]);
                    }
                    if (!ok) break;
                    tc_commit(&k_empty[s0]);
                    pre0 = false;
                }
                for (int j = 0; ok && j < n1; ++j) {
                    const int gj = gkv + j;
                    const int s = gj % KV_STAGES, s1 = (gj + 1) % KV_STAGES;
                    if (!mbar_wait(&v_full[s], (gj / KV_STAGES) & 1, p.status)) { ok = false; break; }
                    const uint32_t v_addr = opaque_u32(smem_u32(v_s + s * CF::TILE));
                    const uint32_t k1_addr = opaque_u32(smem_u32(k_s + s1 * CF::TILE));
                    bool k1_ready = false;
#pragma unroll
                    for (int t = 0; t < 2; ++t) {
                        const int nt = t ? n1 : n0;
                        if (j >= nt) continue;
                        if (t == 1 && j == n1 - 1 && j >= n0) {
                            // Tile 0 is done with this item: S_0 of the next item now,
                            // while tile 1 runs its last step (S_0 held P_0 of this
                            // item's last tile-0 step, whose PV was issued before).
                            int kn = k + 1, bh2, qb2, st2;
                            while ((st2 = item_at(kn, bh2, qb2)) == 2) ++kn;
                            if (st2 == 1) {
                                const int n0n = geo(bh2, qb2).n0;
                                const int gn = gkv + n1, sn = gn % KV_STAGES;
                                if (!mbar_wait(&k_full[sn], (gn / KV_STAGES) & 1, p.status) ||
                                    !mbar_wait(&q_full[0], (li + 1) & 1, p.status)) {
                                    ok = false;
                                    break;
                                }
                                tc_fence_after();
                                qk(0, opaque_u32(smem_u32(k_s + sn * CF::TILE)));
                                tc_commit(&s_full[0]);
                                if (n0n == 1) tc_commit(&q_empty[0]);
                                pre0 = true;
                            }
                        }
                        // the first PV_t of an item overwrites O_t: the previous item's
                        // epilogue must have read it
                        if (j == 0 && li > 0 && !mbar_wait(&o_free[t], (li - 1) & 1, p.status)) {
                            ok = false;
                            break;
                        }
                        if (!mbar_wait(&p_full[t], (c[t] + j) & 1, p.status)) { ok = false; break; }
                        tc_fence_after();
#pragma unroll
                        for (int kk = 0; kk < BKV / 16; ++kk)
                            tc_mma_f16_ts(tmem + CF::O_COL + t * D, tmem + t * BKV + kk * 8,
                                          smem_desc_sw128(v_addr + kk * 16 * 128, SLAB_BYTES, 1024),
                                          CF::IDESC_PV, (j | kk) != 0);
                        tc_commit(&pv_done[t]);
                        if (t == 1) tc_commit(&v_empty[s]);
                        if (j + 1 < nt) {
                            if (!k1_ready) {
                                if (!mbar_wait(&k_full[s1], ((gj + 1) / KV_STAGES) & 1, p.status)) {
                                    ok = false;
                                    break;
                                }
                                tc_fence_after();
                                k1_ready = true;
                            }
                            // P_t,j sits in S_t, which this QK overwrites: tcgen05.mma
                            // operations issued by one thread execute in issue order, so
                            // PV_t,j has read P before QK_t,j+1 writes S_t -- no wait here.
                            qk(t, k1_addr);
                            tc_commit(&s_full[t]);
                            if (j + 2 == nt) tc_commit(&q_empty[t]);   // the item's last QK_t
                            if (t == 1) tc_commit(&k_empty[s1]);
                        }
                    }
                }
                gkv += n1;
                c[0] += n0;
                c[1] += n1;
                ++li;
            }
            tc_commit(drain);
            mbar_wait(drain, 0, p.status);
        }
    }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegSoftmax));
        // ---------------------------------------------------------- softmax
        const int t = (warp - 4) >> 2;
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
        const uint32_t s_col = t * BKV, o_col = CF::O_COL + t * D;
        const float c = p.scale_log2;
        // c_t: this tile's steps before the current item (phase of s_full / pv_done)
        int c_t = 0;
        bool ok = true;
        for (int it = 0; ok; ++it) {
        int bh, qb;
        const int st_item = item_at(it, bh, qb);
        if (st_item == 0) break;
        if (st_item == 2) continue;
        const Geo g = geo(bh, qb);
        const int q0 = g.q0, S_kv = g.S_kv, coff = g.coff;
        const int qi = q0 + t * BQ + r;
        const int nt = t ? g.n1 : g.n0;
        const int vis_hi = p.causal ? min(S_kv - 1, qi + coff) : S_kv - 1;
        float m_run = -INFINITY, l_run = 0.0f;
        for (int j = 0; j < nt; ++j) {
            if (!mbar_wait_warp(&s_full[t], (c_t + j) & 1, p.status)) { ok = false; break; }
            tc_fence_after();
            uint32_t sr[BKV / 32][32];
            __syncwarp();
#pragma unroll
            for (int cch = 0; cch < BKV / 32; ++cch)
                tmem_ld_32x32b_x32(lane_base + s_col + cch * 32, sr[cch]);
            tmem_ld_wait();
            const int k0 = j * BKV;
            if (k0 + BKV - 1 > vis_hi) {
#pragma unroll
                for (int cch = 0; cch < BKV / 32; ++cch)
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        if (k0 + cch * 32 + e > vis_hi) sr[cch][e] = __float_as_uint(-INFINITY);
            }
            float mx[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) mx[i] = -INFINITY;
#pragma unroll
            for (int cch = 0; cch < BKV / 32; ++cch)
#pragma unroll
                for (int e = 0; e < 32; e += 16)
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        mx[i] = fmax3(mx[i], __uint_as_float(sr[cch][e + 2 * i]),
                                      __uint_as_float(sr[cch][e + 2 * i + 1]));
            const float mt = fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]),
                                   fmaxf(mx[6], mx[7]));
            const float m_new = fmaxf(m_run, mt * c);
            const bool need = (j == 0) || (m_new > m_run + kRescaleThreshold);
            if (__any_sync(0xffffffffu, need)) {
                const float alpha = (m_run == -INFINITY) ? 0.0f : ex2_approx(m_run - m_new);
                if (j > 0) {
                    if (!mbar_wait_warp(&pv_done[t], (c_t + j - 1) & 1, p.status)) { ok = false; break; }
                    tc_fence_after();
                    __syncwarp();
#pragma unroll
                    for (int oc = 0; oc < D / 32; ++oc) {
                        uint32_t o[32];
                        tmem_ld_32x32b_x32(lane_base + o_col + oc * 32, o);
                        tmem_ld_wait();
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                        tmem_st_32x32b_x32(lane_base + o_col + oc * 32, o);
                    }
                }
                l_run *= alpha;
                m_run = m_new;
            }
            const float m_use = (m_run == -INFINITY) ? 0.0f : m_run;
            const uint64_t c2 = f2pack(c, c), nm2 = f2pack(-m_use, -m_use);
            uint64_t rs4[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) rs4[i] = f2pack(0.0f, 0.0f);
#pragma unroll
            for (int cch = 0; cch < BKV / 32; ++cch) {
                uint32_t pk[16];
#pragma unroll
                for (int e = 0; e < 32; e += 2) {
                    const uint64_t x2 = ffma2(f2pack(__uint_as_float(sr[cch][e]), __uint_as_float(sr[cch][e + 1])), c2, nm2);
                    float x0, x1;
                    f2unpack(x2, x0, x1);
                    const uint64_t p2 = f2pack(ex2_approx(x0), ex2_approx(x1));
                    rs4[(e >> 1) & 3] = fadd2(rs4[(e >> 1) & 3], p2);
                    float p0, p1;
                    f2unpack(p2, p0, p1);
                    pk[e >> 1] = f32x2_to_bf16x2(p0, p1);
                }
#pragma unroll
                for (int e = 0; e < 16; ++e) sr[cch >> 1][(cch & 1) * 16 + e] = pk[e];
                if (cch & 1) tmem_st_32x32b_x32(lane_base + s_col + (cch >> 1) * 32, sr[cch >> 1]);
            }
            float rs_lo, rs_hi;
            f2unpack(fadd2(fadd2(rs4[0], rs4[1]), fadd2(rs4[2], rs4[3])), rs_lo, rs_hi);
            l_run += rs_lo + rs_hi;
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[t]);
        }
        if (ok && !mbar_wait_warp(&pv_done[t], (c_t + nt - 1) & 1, p.status)) ok = false;
        if (ok) {
            tc_fence_after();
            const float inv_l = l_run > 0.0f ? 1.0f / l_run : 0.0f;
            const bool row_ok = qi < p.S_q;
            const float lse_v =
                l_run > 0.0f ? (m_run + lg2_approx(l_run)) * 0.69314718055994531f : -INFINITY;
            if constexpr (!kAllGather) {
                __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.O) +
                                      ((int64_t)bh * p.S_q + (row_ok ? qi : 0)) * D;
                __syncwarp();
                // all of O_t into registers (one wait), then O_t is free for the next
                // item's first PV while this warp normalises and stores
                uint32_t o[D / 32][32];
#pragma unroll
                for (int oc = 0; oc < D / 32; ++oc)
                    tmem_ld_32x32b_x32(lane_base + o_col + oc * 32, o[oc]);
                tmem_ld_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&o_free[t]);
                if (row_ok) {
#pragma unroll
                    for (int oc = 0; oc < D / 32; ++oc)
#pragma unroll
                        for (int e = 0; e < 32; e += 8) {
                            uint4 w;
                            w.x = f32x2_to_bf16x2(__uint_as_float(o[oc][e]) * inv_l, __uint_as_float(o[oc][e + 1]) * inv_l);
                            w.y = f32x2_to_bf16x2(__uint_as_float(o[oc][e + 2]) * inv_l, __uint_as_float(o[oc][e + 3]) * inv_l);
                            w.z = f32x2_to_bf16x2(__uint_as_float(o[oc][e + 4]) * inv_l, __uint_as_float(o[oc][e + 5]) * inv_l);
                            w.w = f32x2_to_bf16x2(__uint_as_float(o[oc][e + 6]) * inv_l, __uint_as_float(o[oc][e + 7]) * inv_l);
                            *reinterpret_cast<uint4*>(orow + oc * 32 + e) = w;
                        }
                }
                if (row_ok && p.lse) p.lse[(int64_t)bh * p.S_q + qi] = lse_v;
            } else {
                // stage this warp's 32 rows (D * 2 bytes each, 16-byte slots swizzled by
                // row) in the tile's Q buffer: every MMA that read it has completed
                constexpr int SLOTS = D * 2 / 16;
                uint4* st = reinterpret_cast<uint4*>(q_s + t * CF::TILE) + quad * 32 * SLOTS;
                fence_proxy_async_smem();
                __syncwarp();
#pragma unroll
                for (int oc = 0; oc < D / 32; ++oc) {
                    uint32_t o[32];
                    tmem_ld_32x32b_x32(lane_base + o_col + oc * 32, o);
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 32; e += 8) {
                        uint4 w;
                        w.x = f32x2_to_bf16x2(__uint_as_float(o[e]) * inv_l, __uint_as_float(o[e + 1]) * inv_l);
                        w.y = f32x2_to_bf16x2(__uint_as_float(o[e + 2]) * inv_l, __uint_as_float(o[e + 3]) * inv_l);
                        w.z = f32x2_to_bf16x2(__uint_as_float(o[e + 4]) * inv_l, __uint_as_float(o[e + 5]) * inv_l);
                        w.w = f32x2_to_bf16x2(__uint_as_float(o[e + 6]) * inv_l, __uint_as_float(o[e + 7]) * inv_l);
                        const int slot = oc * 4 + (e >> 3);
                        st[lane * SLOTS + ((slot & ~7) | ((slot ^ lane) & 7))] = w;
                    }
                }
                __syncwarp();
                // the warp's rows are contiguous in O: whole 512-byte stores to every rank
                const int row0 = q0 + t * BQ + quad * 32;
                const int nrows = max(0, min(32, p.S_q - row0));
                const int64_t grow = (int64_t)(p.bh_base + bh) * p.S_q + row0;
                for (int i = 1; i <= p.world; ++i) {
                    const int d = (p.rank + i) % p.world;
                    uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.o_peers[d]) +
                                                          grow * D);
                    for (int idx = lane; idx < nrows * SLOTS; idx += 32) {
                        const int rr = idx / SLOTS, slot = idx % SLOTS;
                        dst[idx] = st[rr * SLOTS + ((slot & ~7) | ((slot ^ rr) & 7))];
                    }
                    if (row_ok && p.lse_peers) p.lse_peers[d][grow + lane] = lse_v;
                }
            }
        }
        c_t += nt;
        }
    }
    if constexpr (kAllGather) {
        if (warp >= 4) {
            // this warp's stores are visible system-wide before it counts itself done;
            // the last of the 8 softmax warps of every CTA signals the other ranks
            __threadfence_system();
            __syncwarp();
            unsigned last = 0;
            if (lane == 0)
                last = atomicAdd(p.done, 1u) == 8u * gridDim.x * gridDim.y - 1u;
            if (__shfl_sync(0xffffffffu, last, 0)) {
                __shared__ unsigned got[kMaxPeers];
                __threadfence_system();
                mailbox_exchange(p.mbox, p.rank, p.world, p.seq, 1u, got, p.status);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

struct PagedKV {
    const int* block_table = nullptr;
    const int* ctx_lens = nullptr;
    int max_pages = 0, num_pages = 0;
};

struct FaAllGather {
    void* const* o_peers = nullptr;
    float* const* lse_peers = nullptr;
    int world = 1, rank = 0, bh_base = 0;
    unsigned long long* const* mbox = nullptr;
    unsigned seq = 0;
};

template <int D, bool kPaged>
int launch_fa(const void* Q, const void* K, const void* V, void* O, float* lse, int B, int Hq,
              int Hkv, int S_q, int S_kv, int causal, int causal_offset, float scale,
              const PagedKV& pkv, cudaStream_t st, const FaAllGather* ag = nullptr) {
    CUtensorMap tq, tk, tv;
    int rc;
    if ((rc = fa_make_tmap_3d(&tq, Q, D, S_q, (int64_t)B * Hq))) return rc;
    if constexpr (kPaged) {
        if ((rc = fa_make_tmap_pool(&tk, K, D, Hkv, pkv.num_pages))) return rc;
        if ((rc = fa_make_tmap_pool(&tv, V, D, Hkv, pkv.num_pages))) return rc;
    } else {
        if ((rc = fa_make_tmap_3d(&tk, K, D, S_kv, (int64_t)B * Hkv))) return rc;
        if ((rc = fa_make_tmap_3d(&tv, V, D, S_kv, (int64_t)B * Hkv))) return rc;
    }
    int* status = nullptr;
    if ((rc = device_status(&status))) return rc;
    FaParams p;
    p.B = B;
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.S_q = S_q;
    p.S_kv = S_kv;
    p.causal = causal;
    p.causal_offset = causal_offset;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.O = O;
    p.lse = lse;
    p.status = status;
    p.block_table = pkv.block_table;
    p.ctx_lens = pkv.ctx_lens;
    p.max_pages = pkv.max_pages;
    p.num_pages = pkv.num_pages;
    p.o_peers = nullptr;
    p.lse_peers = nullptr;
    p.world = 1;
    p.rank = 0;
    p.bh_base = 0;
    p.mbox = nullptr;
    p.seq = 0;
    p.done = nullptr;
    auto kern = k_flash_fwd<D, kPaged, false>;
    if constexpr (!kPaged) {
        if (ag) {
            void* done = nullptr;
            AMPB_CHECK_CUDA(cudaGetSymbolAddress(&done, g_fa_allgather_done));
            AMPB_CHECK_CUDA(cudaMemsetAsync(done, 0, sizeof(unsigned), st));
            p.o_peers = ag->o_peers;
            p.lse_peers = ag->lse_peers;
            p.world = ag->world;
            p.rank = ag->rank;
            p.bh_base = ag->bh_base;
            p.mbox = ag->mbox;
            p.seq = ag->seq;
            p.done = static_cast<unsigned*>(done);
            kern = k_flash_fwd<D, kPaged, true>;
        }
    }
    const int n_qb = (S_q + 2 * BQ - 1) / (2 * BQ);
    dim3 grid(n_qb, B * Hq);
    if constexpr (!kPaged) {
        const int64_t units = (int64_t)B * Hq * ((n_qb + 1) / 2);
        if (!ag && units <= INT32_MAX / 2) {
            // dense, one GPU's output: one persistent CTA per SM over units of two
            // query-tile pairs (k_flash_fwd's item_at)
            kern = k_flash_fwd<D, kPaged, false, true>;
            grid = dim3((unsigned)std::min<int64_t>(units, sm_count()), 1);
        }
    }
    AMPB_CHECK_CUDA(
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, FaCfg<D>::SMEM));
    kern<<<grid, kThreads, FaCfg<D>::SMEM, st>>>(tq, tk, tv, p);
    AMPB_CHECK_LAUNCH("k_flash_fwd");
    return AMP_OK;
}

}  // namespace


// [bh][s][d] bf16 tensor as a 3-D TMA map, box [1][128][64], 128-byte swizzle.
int fa_make_tmap_3d(CUtensorMap* m, const void* base, int64_t d, int64_t s, int64_t bh) {
    cuuint64_t dims[3] = {(cuuint64_t)d, (cuuint64_t)s, (cuuint64_t)bh};
    cuuint64_t strides[2] = {(cuuint64_t)(d * 2), (cuuint64_t)(s * d * 2)};
    cuuint32_t box[3] = {64, 128, 1};
    return encode_tmap(m, base, 2, 3, dims, strides, box);
}

// Paged pool [pages][hkv][16][d] bf16 as a 4-D TMA map, box = one page of one
// head (16 rows x 64 columns), 128-byte swizzle.
int fa_make_tmap_pool(CUtensorMap* m, const void* base, int64_t d, int64_t hkv, int64_t pages) {
    cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)kPageTokens, (cuuint64_t)hkv,
                          (cuuint64_t)pages};
    cuuint64_t strides[3] = {(cuuint64_t)(d * 2), (cuuint64_t)(kPageTokens * d * 2),
                             (cuuint64_t)(hkv * kPageTokens * d * 2)};
    cuuint32_t box[4] = {64, (cuuint32_t)kPageTokens, 1, 1};
    return encode_tmap(m, base, 2, 4, dims, strides, box);
}


int flash_attn_fwd_dev(const void* Q, const void* K, const void* V, void* O, float* lse, int B,
                       int Hq, int Hkv, int S_q, int S_kv, int D, int causal, int causal_offset,
                       float scale, cudaStream_t st, const FaAllGather* ag = nullptr) {
    AMPB_REQUIRE(B > 0 && Hq > 0 && Hkv > 0 && S_q > 0 && S_kv > 0, AMP_ERR_INVALID,
                 "attention sizes must be positive");
    AMPB_REQUIRE(Hq % Hkv == 0, AMP_ERR_INVALID, "num_q_heads (%d) must be a multiple of "
                 "num_kv_heads (%d)", Hq, Hkv);
    AMPB_REQUIRE(Q && K && V && (O || ag), AMP_ERR_INVALID, "NULL tensor");
    AMPB_REQUIRE(aligned16(Q) && aligned16(K) && aligned16(V) && (ag || aligned16(O)),
                 AMP_ERR_INVALID, "Q, K, V, O must be 16-byte aligned");
    AMPB_REQUIRE((int64_t)B * Hq <= 65535, AMP_ERR_UNSUPPORTED, "B*Hq must be <= 65535");
    if (!(scale > 0.0f)) scale = 1.0f / sqrtf((float)D);
    const PagedKV none;
    switch (D) {
        case 128:
            return launch_fa<128, false>(Q, K, V, O, lse, B, Hq, Hkv, S_q, S_kv, causal,
                                         causal_offset, scale, none, st, ag);
        case 64:
            return launch_fa<64, false>(Q, K, V, O, lse, B, Hq, Hkv, S_q, S_kv, causal,
                                        causal_offset, scale, none, st, ag);
        default:
            set_error(AMP_ERR_UNSUPPORTED, "flash_attn: head_dim %d not supported (64, 128)", D);
            return AMP_ERR_UNSUPPORTED;
    }
}

int paged_prefill_dev(const void* q, const void* k_pool, const void* v_pool,
                      const int* block_table, const int* ctx_lens, void* out, float* lse, int B,
                      int Hq, int Hkv, int Lq, int D, int num_pages, int max_pages, float scale,
                      cudaStream_t st) {
    AMPB_REQUIRE(B > 0 && Hq > 0 && Hkv > 0 && Lq > 0 && num_pages > 0 && max_pages > 0,
                 AMP_ERR_INVALID, "paged prefill sizes must be positive");
    AMPB_REQUIRE(Hq % Hkv == 0, AMP_ERR_INVALID, "Hq (%d) must be a multiple of Hkv (%d)", Hq, Hkv);
    AMPB_REQUIRE(q && k_pool && v_pool && block_table && ctx_lens && out, AMP_ERR_INVALID,
                 "NULL argument");
    AMPB_REQUIRE(aligned16(q) && aligned16(k_pool) && aligned16(v_pool) && aligned16(out),
                 AMP_ERR_INVALID, "q, out and the pools must be 16-byte aligned");
    AMPB_REQUIRE((int64_t)B * Hq <= 65535, AMP_ERR_UNSUPPORTED, "B*Hq must be <= 65535");
    if (!(scale > 0.0f)) scale = 1.0f / sqrtf((float)D);
    PagedKV pkv;
    pkv.block_table = block_table;
    pkv.ctx_lens = ctx_lens;
    pkv.max_pages = max_pages;
    pkv.num_pages = num_pages;
    switch (D) {
        case 128:
            return launch_fa<128, true>(q, k_pool, v_pool, out, lse, B, Hq, Hkv, Lq, 0, 1, 0, scale,
                                        pkv, st);
        case 64:
            return launch_fa<64, true>(q, k_pool, v_pool, out, lse, B, Hq, Hkv, Lq, 0, 1, 0, scale,
                                       pkv, st);
        default:
            set_error(AMP_ERR_UNSUPPORTED, "paged prefill: head_dim %d not supported (64, 128)", D);
            return AMP_ERR_UNSUPPORTED;
    }
}

}  // namespace ampb

using namespace ampb;

extern "C" int amp_paged_attn_prefill_bf16_dev(const void* q, const void* k_pool,
                                               const void* v_pool, const int32_t* block_table,
                                               const int32_t* ctx_lens, void* out, float* lse,
                                               int B, int Hq, int Hkv, int Lq, int head_dim,
                                               int num_pages, int max_pages_per_seq, float scale,
                                               void* stream) {
    return paged_prefill_dev(q, k_pool, v_pool, block_table, ctx_lens, out, lse, B, Hq, Hkv, Lq,
                             head_dim, num_pages, max_pages_per_seq, scale, as_stream(stream));
}

extern "C" int amp_flash_attn_fwd_bf16_dev(const void* Q, const void* K, const void* V, void* O,
                                           float* lse, int B, int Hq, int Hkv, int S_q, int S_kv,
                                           int head_dim, int causal, float scale, void* stream) {
    return flash_attn_fwd_dev(Q, K, V, O, lse, B, Hq, Hkv, S_q, S_kv, head_dim, causal, 0, scale,
                              as_stream(stream));
}

// (batch*head)-sharded attention with the all-gather of O and lse fused into the
// epilogue.  Q, K, V hold this rank's B*Hq (B*Hkv) slice; O_peers / lse_peers
// are DEVICE arrays of `world` pointers to every rank's full O [bh_total][S_q][D]
// and lse [bh_total][S_q] (lse_peers may be NULL); this rank's batch*head 0 is
// global index bh_base.  Mailboxes and seq as for amp_gemm_bf16_allgather_dev.
extern "C" int amp_flash_attn_fwd_allgather_dev(const void* Q, const void* K, const void* V,
                                                void* const* O_peers, float* const* lse_peers,
                                                int rank, int world, int bh_base,
                                                void* const* mailboxes, unsigned seq, int B,
                                                int Hq, int Hkv, int S_q, int S_kv, int head_dim,
                                                int causal, float scale, void* stream) {
    AMPB_REQUIRE(O_peers && mailboxes, AMP_ERR_INVALID, "all-gather needs O and mailbox tables");
    AMPB_REQUIRE(world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world, AMP_ERR_INVALID,
                 "rank %d / world %d outside [0, %d)", rank, world, kMaxPeers);
    AMPB_REQUIRE(seq != 0, AMP_ERR_INVALID, "sequence numbers start at 1");
    AMPB_REQUIRE(bh_base >= 0, AMP_ERR_INVALID, "bh_base must be >= 0");
    FaAllGather ag;
    ag.o_peers = O_peers;
    ag.lse_peers = lse_peers;
    ag.world = world;
    ag.rank = rank;
    ag.bh_base = bh_base;
    ag.mbox = reinterpret_cast<unsigned long long* const*>(mailboxes);
    ag.seq = seq;
    return flash_attn_fwd_dev(Q, K, V, nullptr, nullptr, B, Hq, Hkv, S_q, S_kv, head_dim, causal,
                              0, scale, as_stream(stream), &ag);
}

// Host-pointer form (plugin convention): all tensors in host memory; device
// staging, launch and copy-back are done before returning.
extern "C" int amp_user_flash_attn_fwd_bf16(const uint16_t* Q, const uint16_t* K,
                                            const uint16_t* V, uint16_t* O, float* lse, int B,
                                            int Hq, int Hkv, int S_q, int S_kv, int head_dim,
                                            int causal, float scale) {
    AMPB_REQUIRE(B > 0 && Hq > 0 && Hkv > 0 && S_q > 0 && S_kv > 0 && head_dim > 0,
                 AMP_ERR_INVALID, "attention sizes must be positive");
    AMPB_REQUIRE(Q && K && V && O, AMP_ERR_INVALID, "NULL tensor");
    const size_t q = (size_t)B * Hq * S_q * head_dim * 2, kv = (size_t)B * Hkv * S_kv * head_dim * 2;
    const size_t l = (size_t)B * Hq * S_q * 4;
    void *dq, *dk, *dv, *dout, *dl;
    int rc;
    if ((rc = staging_get(0, q, &dq)) || (rc = staging_get(1, kv, &dk)) ||
        (rc = staging_get(2, kv, &dv)) || (rc = staging_get(3, q, &dout)) ||
        (rc = staging_get(4, l, &dl)))
        return rc;
    cudaStream_t st = 0;
    AMPB_CHECK_CUDA(cudaMemcpyAsync(dq, Q, q, cudaMemcpyHostToDevice, st));
    AMPB_CHECK_CUDA(cudaMemcpyAsync(dk, K, kv, cudaMemcpyHostToDevice, st));
    AMPB_CHECK_CUDA(cudaMemcpyAsync(dv, V, kv, cudaMemcpyHostToDevice, st));
    if ((rc = flash_attn_fwd_dev(dq, dk, dv, dout, static_cast<float*>(dl), B, Hq, Hkv, S_q, S_kv,
                                 head_dim, causal, 0, scale, st)))
        return rc;
    AMPB_CHECK_CUDA(cudaMemcpyAsync(O, dout, q, cudaMemcpyDeviceToHost, st));
    if (lse) AMPB_CHECK_CUDA(cudaMemcpyAsync(lse, dl, l, cudaMemcpyDeviceToHost, st));
    AMPB_CHECK_CUDA(cudaStreamSynchronize(st));
    const int status = amp_device_status(1);
    if (status) return status;
    return staging_end_of_call();
}
