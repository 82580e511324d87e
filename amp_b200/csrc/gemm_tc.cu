// gemm_tc.cu -- bf16 and FP8 E4M3 GEMM on the 5th-generation tensor cores.
//
// Replaces the reference's bf16 WMMA kernel (kernels/matmul.cu:47-110: one
// warp per 16x16 tile, operands staged through shared memory every k-step,
// fp32 C) and its FP8 route (kernels/matmul.cu:235-270 -> cuBLASLt in
// src/gemm_vendor.cpp:154-237, per-tensor scales, fp32 C).
//
// Layout is AMP's: A [M,K] row-major (K-major operand), B [K,N] row-major
// (N-major operand, consumed as an MN-major UMMA operand, no transpose), C
// [M,N] row-major in fp32 or bf16 -- and, for FP8 inputs, E4M3 with a caller
// scale and/or the amax of C computed in the epilogue (what AMP's GemmDesc
// carries as d_scale_c / d_amax_c for cuBLASLt, include/gemm_vendor.hpp:55-56).
//
// Kernel structure (persistent, one 128x256 output tile per iteration, one
// CTA per SM, 192 threads):
//   warp 0      TMA producer: per 128-byte k-slab, one A box [128 rows x 128 B]
//               and 256*es/128 B boxes [BK rows x 128 B], 128-byte swizzle,
//               into a 4-stage ring guarded by full/empty mbarriers.
//   warp 1      allocates 512 TMEM columns (two 128x256 fp32 accumulators);
//               one lane issues tcgen05.mma (M=128, N=256, K=16 bf16 / 32 fp8,
//               4 per k-slab) and commits each stage back to its empty barrier
//               and each finished tile to the accumulator's full barrier.
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time from their TMEM lane
//               quadrant, apply the FP8 scales, convert, store to global; the
//               accumulator is released as soon as it has been read, so the
//               next tile's MMAs overlap this tile's stores.
// Tiles are visited in groups of 16 M-tiles (a ~2K-row band) so that the
// CTAs running at the same time share A rows and B columns in L2.
//
// All-gather mode (N-sharded GEMM on the GPUs of one node, the reference's
// launch + ncclAllGather of C, include/collective.hpp:87-89): rank r computes
// its column block C[:, r*N : (r+1)*N] and the epilogue stores every chunk
// straight into the replicated C of every rank -- its own and, over NVLink,
// each peer's (CUDA IPC mappings) -- so the exchange overlaps the MMAs of the
// next tiles.  When a CTA's epilogue warps have stored their last tile they
// fence at system scope and count themselves done; the last warp on the GPU
// posts this launch's sequence number to every rank's mailbox and waits
// (bounded) until every rank has posted it, so the kernel ends only once
// every peer's stores into this rank's C are visible.
#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <cfloat>
#include <mutex>

#include "common.cuh"
#include "peer.cuh"
#include "runtime.h"
#include "tc_common.cuh"

namespace ampb {
namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int SLAB = 128;        // bytes of K per stage (one 128-byte swizzle row)
constexpr int STAGES = 4;
constexpr int kThreads = 192;
constexpr int kGroupM = 16;
constexpr int A_STAGE_BYTES = BM * SLAB;           // 16 KiB
constexpr int B_STAGE_BYTES = BN * SLAB;           // 32 KiB (BK rows x 256 cols x es)
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
// all-gather mode: per epilogue warp a [32 rows x 128 B] staging tile, so that
// the stores to the other ranks go out as whole 128-byte row segments
// Staged rows are AG_GROUP = 128 bytes plus 16 of padding, so that the
// epilogue lanes' 16-byte writes of their own rows spread over the banks while
// every row stays contiguous for the bulk copy that sends it.  (Whole 512-byte
// tile rows, with the pair kernel's ring cut to 4 stages to make room, measured
// slower at 2 GPUs: bf16 1490 -> 1390, E4M3 2707 -> 2471 TFLOP/s a rank.)
constexpr int AG_GROUP = 128;
constexpr int AG_ROW_PITCH = AG_GROUP + 16;
constexpr int AG_STAGE_BYTES = 4 * 32 * AG_ROW_PITCH;
constexpr int SMEM_BYTES_AG = SMEM_BYTES + AG_STAGE_BYTES;
constexpr uint32_t TMEM_COLS = 512;

enum ScaleMode : int { kNoScale = 0, kTensorScale = 1, kRowColScale = 2 };

struct TcParams {
    int M, N, K;
    int num_m, num_n, num_kb;
    void* C;
    const float* scale_a;   // per-tensor: [1]; row/col: [M]
    const float* scale_b;   // per-tensor: [1]; row/col: [N]
    int scale_mode;
    const float* scale_c;   // E4M3 output: dequantisation scale of C (device float)
    float* amax;            // optional: max |C| before output conversion (device float)
    int* status;
    // all-gather mode (peers != nullptr): C of every rank, [M][ldc] each; this
    // rank's block starts at column col_base
    void* const* peers;
    int world, rank, ldc, col_base;
    unsigned long long* const* mbox;
    unsigned seq;
    unsigned* done;         // epilogue warps finished (zeroed before the launch)
};

// Epilogue warps of the all-gather GEMM that have stored their last tile; one
// counter per device (one all-gather GEMM in flight per device).
__device__ unsigned g_allgather_done;

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& tm, int& tn) {
    const int per_group = kGroupM * num_n;
    const int g = t / per_group;
    const int first_m = g * kGroupM;
    const int gm = min(kGroupM, num_m - first_m);
    const int local = t - g * per_group;
    tm = first_m + local % gm;
    tn = local / gm;
}

// ---- epilogue steps on one 32-column chunk of a C row (both GEMM kernels)

// Scales a row takes: sa multiplies every accumulator (per-tensor product, or
// scale_a[row] per row); inv_c is the E4M3 output's RN(1/scale_c), as the quantiser.
template <typename OutT>
__device__ __forceinline__ void row_scales(const TcParams& p, int row, bool row_ok, float& sa,
                                           float& inv_c) {
    inv_c = 1.0f;
    if constexpr (sizeof(OutT) == 1) {
        inv_c = __frcp_rn(p.scale_c[0]);
        inv_c = inv_c > FLT_MAX ? FLT_MAX : inv_c;
    }
    sa = 1.0f;
    if (p.scale_mode == kTensorScale) sa = p.scale_a[0] * p.scale_b[0];
    else if (p.scale_mode == kRowColScale && row_ok) sa = p.scale_a[row];
}

// v = accumulators x sa (x scale_b[col] per column: all lanes take part in the shuffles)
__device__ __forceinline__ void scale_chunk(const uint32_t (&r)[32], float (&v)[32], float sa,
                                            const TcParams& p, int col0, int lane) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * sa;
    if (p.scale_mode == kRowColScale) {
        const float sbv = (col0 + lane < p.N) ? p.scale_b[col0 + lane] : 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] *= __shfl_sync(0xffffffffu, sbv, j);
    }
}

// amx = max(amx, |v[j]|) over the nv columns inside C (NaN ignored by fmaxf)
__device__ __forceinline__ void amax_chunk(float& amx, const float (&v)[32], int nv) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
        if (j < nv) amx = fmaxf(amx, fabsf(v[j]));
}

// Stores the first min(nv, 32) values of v at `out` as OutT (E4M3 codes of v * inv_c
// for 1-byte C).  Every loop has constant indices, so v stays in registers.
template <typename OutT>
__device__ __forceinline__ void store_chunk(OutT* out, const float (&v)[32], int nv, float inv_c) {
    const bool full_chunk = nv >= 32 && ((reinterpret_cast<uintptr_t>(out) & 15u) == 0);
    if constexpr (sizeof(OutT) == 1) {
        uint32_t w8[8];
#pragma unroll
        for (int j = 0; j < 32; j += 4)
            w8[j >> 2] = f32x2_to_e4m3x2(__fmul_rn(v[j], inv_c), __fmul_rn(v[j + 1], inv_c)) |
                         (f32x2_to_e4m3x2(__fmul_rn(v[j + 2], inv_c), __fmul_rn(v[j + 3], inv_c))
                          << 16);
        if (full_chunk) {
            reinterpret_cast<uint4*>(out)[0] = make_uint4(w8[0], w8[1], w8[2], w8[3]);
            reinterpret_cast<uint4*>(out)[1] = make_uint4(w8[4], w8[5], w8[6], w8[7]);
        } else {
            uint8_t* o8 = reinterpret_cast<uint8_t*>(out);
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < nv) o8[j] = (uint8_t)(w8[j >> 2] >> (8 * (j & 3)));
        }
    } else if constexpr (sizeof(OutT) == 4) {
        if (full_chunk) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
                *reinterpret_cast<float4*>(out + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < nv) out[j] = v[j];
        }
    } else {
        if (full_chunk) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
                uint4 w;
                w.x = f32x2_to_bf16x2(v[j], v[j + 1]);
                w.y = f32x2_to_bf16x2(v[j + 2], v[j + 3]);
                w.z = f32x2_to_bf16x2(v[j + 4], v[j + 5]);
                w.w = f32x2_to_bf16x2(v[j + 6], v[j + 7]);
                *reinterpret_cast<uint4*>(out + j) = w;
            }
        } else {
            uint16_t* o16 = reinterpret_cast<uint16_t*>(out);
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < nv) o16[j] = (uint16_t)(f32x2_to_bf16x2(v[j], 0.0f) & 0xffffu);
        }
    }
}

// All-gather mode, one 32-value chunk of this thread's row: chunk groups of 128
// bytes a row that lie inside N go through the warp's [32 rows x 128 B] staging
// tile (all lanes, rows past M included); after a group's last chunk every lane
// hands its row's 128 bytes to the bulk-copy (TMA) engine, one asynchronous
// shared -> global copy per rank's C (this rank last), so the NVLink traffic is
// streamed by the copy engine instead of by the epilogue's store instructions.
// Before a lane rewrites its staging row it waits until its earlier copies have
// read it.  Returns false for a chunk outside such a group, which the caller
// stores row by row.  row0: the warp's first row of C; stage: the warp's tile.
template <typename OutT>
__device__ __forceinline__ bool ag_stage_chunk(const float (&v)[32], int c, int tn, int row0,
                                               int lane, uint8_t* stage, const TcParams& p) {
    static_assert(sizeof(OutT) != 1, "E4M3 output is stored row by row");
    constexpr int CPG = AG_GROUP / (32 * (int)sizeof(OutT));   // chunks per group
    if (tn * BN + (c / CPG + 1) * CPG * 32 > p.N) return false;
    constexpr int Q = 32 * (int)sizeof(OutT) / 16;         // 16-byte slots of a chunk
    uint4* row = reinterpret_cast<uint4*>(stage + lane * AG_ROW_PITCH);
    if (c % CPG == 0)   // this lane's copies of the previous group have read its row
        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
#pragma unroll
    for (int k = 0; k < Q; ++k) {
        uint4 w;
        if constexpr (sizeof(OutT) == 4) {
            w = make_uint4(__float_as_uint(v[4 * k]), __float_as_uint(v[4 * k + 1]),
                           __float_as_uint(v[4 * k + 2]), __float_as_uint(v[4 * k + 3]));
        } else {
            w.x = f32x2_to_bf16x2(v[8 * k], v[8 * k + 1]);
            w.y = f32x2_to_bf16x2(v[8 * k + 2], v[8 * k + 3]);
            w.z = f32x2_to_bf16x2(v[8 * k + 4], v[8 * k + 5]);
            w.w = f32x2_to_bf16x2(v[8 * k + 6], v[8 * k + 7]);
        }
        row[(c % CPG) * Q + k] = w;
    }
    if (c % CPG == CPG - 1 && row0 + lane < p.M) {
        fence_proxy_async_smem();   // the row's generic-proxy writes, seen by the copies
        const int gcol = p.col_base + tn * BN + (c - CPG + 1) * 32;
        const int64_t off = ((int64_t)(row0 + lane) * p.ldc + gcol) * sizeof(OutT);
        for (int i = 1; i <= p.world; ++i) {
            uint8_t* dst = static_cast<uint8_t*>(p.peers[(p.rank + i) % p.world]) + off;
            asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
                         "r"(smem_u32(row)), "n"(AG_GROUP)
                         : "memory");
        }
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
    return true;
}

// All-gather mode: a chunk outside the staged groups, row by row into every
// rank's C (this rank last).
template <typename OutT>
__device__ __forceinline__ void ag_store_row_chunk(const float (&v)[32], int row, int col0,
                                                   float inv_c, const TcParams& p) {
    for (int i = 1; i <= p.world; ++i) {
        const int d = (p.rank + i) % p.world;
        store_chunk(static_cast<OutT*>(p.peers[d]) + (int64_t)row * p.ldc + p.col_base + col0, v,
                    p.N - col0, inv_c);
    }
}

// All-gather mode, after an epilogue warp's last tile: its stores and bulk copies
// (local and remote) are made visible system-wide before it counts itself done; the last
// of the launch's 4 * gridDim.x epilogue warps exchanges the call's sequence
// number with every rank, so the kernel ends only once every rank's C is whole.
__device__ __forceinline__ void ag_finish(int lane, const TcParams& p) {
    // this lane's bulk copies have completed their writes
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __threadfence_system();
    __syncwarp();
    unsigned last = 0;
    if (lane == 0) last = atomicAdd(p.done, 1u) == 4u * gridDim.x - 1u;
    if (__shfl_sync(0xffffffffu, last, 0)) {
        __shared__ unsigned got[kMaxPeers];
        __threadfence_system();
        mailbox_exchange(p.mbox, p.rank, p.world, p.seq, 1u, got, p.status);
    }
}

template <bool kFP8, typename OutT, bool kAllGather>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const TcParams p) {
    constexpr int ES = kFP8 ? 1 : 2;                 // element size
    constexpr int BK = SLAB / ES;                    // K elements per stage
    constexpr int UMMA_K = 32 / ES;                  // K per MMA (32 bytes)
    constexpr int B_BOX_COLS = SLAB / ES;            // N columns per B box
    constexpr int B_BOXES = BN / B_BOX_COLS;         // 4 (bf16) or 2 (fp8)
    constexpr int B_BOX_BYTES = BK * SLAB;           // 8 KiB or 16 KiB
    constexpr uint32_t IDESC = make_idesc(kFP8 ? 0 : 1, kFP8 ? 0 : 1, 0, 1, BM, BN);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int total = p.num_m * p.num_n;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                int tm, tn;
                tile_coords(t, p.num_m, p.num_n, tm, tn);
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(&empty[s], ph ^ 1, p.status)) { ok = false; break; }
                    uint8_t* sa = smem + s * STAGE_BYTES;
                    uint8_t* sb = sa + A_STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
                    tma_load_2d(sa, &tmA, &full[s], kb * BK, tm * BM);
#pragma unroll
                    for (int j = 0; j < B_BOXES; ++j)
                        tma_load_2d(sb + j * B_BOX_BYTES, &tmB, &full[s],
                                    tn * BN + j * B_BOX_COLS, kb * BK);
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            int i = 0;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++i) {
                const int acc = i & 1;
                const uint32_t acc_ph = (i >> 1) & 1;
                if (!mbar_wait(&tempty[acc], acc_ph ^ 1, p.status)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(&full[s], ph, p.status)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
                    const uint32_t sb = sa + A_STAGE_BYTES;
#pragma unroll
                    for (int k = 0; k < SLAB / 32; ++k) {
                        const uint64_t ad = smem_desc_sw128(sa + k * 32, 16, 1024);
                        const uint64_t bd = smem_desc_sw128(sb + k * UMMA_K * SLAB, B_BOX_BYTES, 1024);
                        if constexpr (kFP8)
                            tc_mma_f8(d_tmem, ad, bd, IDESC, (kb | k) != 0);
                        else
                            tc_mma_f16(d_tmem, ad, bd, IDESC, (kb | k) != 0);
                    }
                    tc_commit(&empty[s]);
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                }
                if (ok) tc_commit(&tfull[acc]);
            }
            // Every MMA this thread issued has finished before TMEM is freed.
            tc_commit(drain);
            mbar_wait(drain, 0, p.status);
        }
    } else {
        const int quad = warp & 3;             // TMEM lanes [32*quad, 32*quad + 32)
        const int row_in_tile = quad * 32 + lane;
        uint8_t* ag_stage = smem + STAGES * STAGE_BYTES + 256 +
                            (warp - 2) * 32 * AG_ROW_PITCH;   // all-gather mode only
        float amx = 0.0f;                      // this thread's max |C| (NaN ignored)
        int i = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x, ++i) {
            const int acc = i & 1;
            const uint32_t acc_ph = (i >> 1) & 1;
            int tm, tn;
            tile_coords(t, p.num_m, p.num_n, tm, tn);
            if (!mbar_wait_warp(&tfull[acc], acc_ph, p.status)) break;
            tc_fence_after();
            const int row = tm * BM + row_in_tile;
            const bool row_ok = row < p.M;
            float sa, inv_c;
            row_scales<OutT>(p, row, row_ok, sa, inv_c);
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                __syncwarp();  // tcgen05.ld is warp-collective: reconverge first
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + c * 32, r);
                tmem_ld_wait();
                if (c == BN / 32 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[acc]);
                }
                const int col0 = tn * BN + c * 32;
                if (col0 >= p.N) continue;  // warp-uniform
                float v[32];
                scale_chunk(r, v, sa, p, col0, lane);
                if (p.amax && row_ok) amax_chunk(amx, v, p.N - col0);
                if constexpr (kAllGather && sizeof(OutT) != 1) {
                    if (ag_stage_chunk<OutT>(v, c, tn, tm * BM + quad * 32, lane, ag_stage, p))
                        continue;
                }
                if (!row_ok) continue;
                if constexpr (!kAllGather)
                    store_chunk(static_cast<OutT*>(p.C) + (int64_t)row * p.N + col0, v, p.N - col0,
                                inv_c);
                else
                    ag_store_row_chunk<OutT>(v, row, col0, inv_c, p);
            }
        }
        if (p.amax) {   // non-negative floats order like their bit patterns
            const float m = warp_max(amx);
            if (lane == 0) atomicMax(reinterpret_cast<unsigned*>(p.amax), __float_as_uint(m));
        }
        if constexpr (kAllGather) ag_finish(lane, p);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ------------------------------------------------------------------ 2-SM tiles
// A cluster of two CTAs (a pair) computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2: each CTA loads its 128 rows of A and its 128 columns
// of B, and holds its 128 rows of the accumulator in its own TMEM, so each SM
// streams two thirds of the operand bytes of a 128 x 256 single-SM tile.  Only
// the leader (cluster rank 0) issues MMAs; both CTAs' TMA loads count on the
// leader's full barriers; each of the leader's commits arrives on the same
// barrier in both CTAs (CTA mask 0b11); the peer's epilogue releases the
// accumulator on the leader's barrier.  Every operand copy lands only in the
// shared memory of the CTA that issues it.
constexpr int STAGES2 = 6;
constexpr int STAGE2_BYTES = A_STAGE_BYTES + (BN / 2) * SLAB;   // 16 KiB A + 16 KiB B
constexpr int SMEM2_BYTES = STAGES2 * STAGE2_BYTES + 1024 + 256;
constexpr int SMEM2_BYTES_AG = SMEM2_BYTES + AG_STAGE_BYTES;   // + the all-gather staging
static_assert(SMEM2_BYTES_AG <= 227 * 1024 && SMEM_BYTES_AG <= 227 * 1024,
              "dynamic shared memory above the 227 KiB a CTA can have");

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
}
// shared::cluster address of this CTA's object `p` in the CTA of cluster rank `r`
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t r) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(r));
    return a;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
                 : "memory");
}
// bounded wait with cluster-scope acquire (arrivals come from the other CTA too)
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* status) {
    const uint64_t t0 = globaltimer_ns();
    uint32_t n = 0;
    while (true) {
        uint32_t ok;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;"
            " selp.u32 %0, 1, 0, p; }"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
        if (ok) return true;
        if ((++n & 1023u) == 0) {
            if (wait_expired(globaltimer_ns() - t0, status)) {
                atomicExch(status, AMP_DEV_ERR_TIMEOUT);
                return false;
            }
            if (*reinterpret_cast<volatile int*>(status) != AMP_DEV_OK) return false;
        }
    }
}
// this CTA's box, completion counted on the barrier at cluster address `bar`
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* m, uint32_t bar,
                                                 int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}
template <bool kFP8>
__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
    if constexpr (kFP8)
        asm volatile(
            "{ .reg .pred p; setp.ne.b32 p, %4, 0;"
            " tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    else
        asm volatile(
            "{ .reg .pred p; setp.ne.b32 p, %4, 0;"
            " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
}
// arrive on the barrier at this offset in both CTAs of the pair once the pair's
// MMAs issued so far have completed
__device__ __forceinline__ void tc_commit_pair_mc(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;" ::"r"(smem_u32(bar)), "h"((uint16_t)3)
        : "memory");
}
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

template <bool kFP8, typename OutT, bool kAllGather = false>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const TcParams p) {
    constexpr int ES = kFP8 ? 1 : 2;                 // element size
    constexpr int BK = SLAB / ES;                    // K elements per stage
    constexpr int UMMA_K = 32 / ES;                  // K per MMA (32 bytes)
    constexpr int B_BOX_COLS = SLAB / ES;            // N columns per B box
    constexpr int B_BOXES = (BN / 2) / B_BOX_COLS;   // this CTA's half of N: 2 (bf16) or 1 (fp8)
    constexpr int B_BOX_BYTES = BK * SLAB;           // 8 KiB or 16 KiB
    // the pair's MMA: M = 256 (128 rows from each CTA), N = 256 (128 columns from each)
    constexpr uint32_t IDESC = make_idesc(kFP8 ? 0 : 1, kFP8 ? 0 : 1, 0, 1, 2 * BM, BN);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    constexpr int ST = STAGES2;   // operand ring depth
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + ST * STAGE2_BYTES);
    uint64_t* empty = full + ST;
    uint64_t* tfull = empty + ST;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();        // 0: the pair's leader, 1: its peer
    const bool leader = rank == 0;
    const int pair = (int)blockIdx.x >> 1, n_pairs = (int)gridDim.x >> 1;
    const int total = p.num_m * p.num_n;            // 256 x 256 tiles

    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(&full[s], 1);      // leader: its producer's expect_tx, both CTAs' bytes
            mbar_init(&empty[s], 1);     // each CTA: the leader's commit (CTA mask 0b11)
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);     // each CTA: the leader's commit (CTA mask 0b11)
            mbar_init(&tempty[b], 8);    // leader: the epilogue warps of both CTAs
        }
        mbar_init(drain, 1);
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();   // both CTAs' barriers initialised and TMEM allocated
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = pair; t < total && ok; t += n_pairs) {
                int tm, tn;
                tile_coords(t, p.num_m, p.num_n, tm, tn);
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(&empty[s], ph ^ 1, p.status)) { ok = false; break; }
                    uint8_t* sa = smem + s * STAGE2_BYTES;
                    uint8_t* sb = sa + A_STAGE_BYTES;
                    // the leader's full barrier counts the bytes of both CTAs' loads
                    if (leader) mbar_arrive_expect_tx(&full[s], 2 * STAGE2_BYTES);
                    const uint32_t fb = cluster_addr(&full[s], 0);
                    tma_load_2d_pair(sa, &tmA, fb, kb * BK, tm * 2 * BM + (int)rank * BM);
#pragma unroll
                    for (int j = 0; j < B_BOXES; ++j)
                        tma_load_2d_pair(sb + j * B_BOX_BYTES, &tmB, fb,
                                         tn * BN + (int)rank * (BN / 2) + j * B_BOX_COLS, kb * BK);
                    if (++s == ST) { s = 0; ph ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            int i = 0;
            for (int t = pair; t < total && ok; t += n_pairs, ++i) {
                const int acc = i & 1;
                const uint32_t acc_ph = (i >> 1) & 1;
                if (!mbar_wait_cluster(&tempty[acc], acc_ph ^ 1, p.status)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait_cluster(&full[s], ph, p.status)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + s * STAGE2_BYTES);
                    const uint32_t sb = sa + A_STAGE_BYTES;
#pragma unroll
                    for (int k = 0; k < SLAB / 32; ++k) {
                        const uint64_t ad = smem_desc_sw128(sa + k * 32, 16, 1024);
                        const uint64_t bd = smem_desc_sw128(sb + k * UMMA_K * SLAB, B_BOX_BYTES, 1024);
                        tc_mma_pair<kFP8>(d_tmem, ad, bd, IDESC, (kb | k) != 0);
                    }
                    tc_commit_pair_mc(&empty[s]);
                    if (++s == ST) { s = 0; ph ^= 1; }
                }
                if (ok) tc_commit_pair_mc(&tfull[acc]);
            }
            // Every MMA of the pair has finished before TMEM is freed or the peer exits.
            tc_commit_pair(drain);
            mbar_wait(drain, 0, p.status);
        }
    } else {
        const int quad = warp & 3;             // TMEM lanes [32*quad, 32*quad + 32)
        const int row_in_tile = quad * 32 + lane;
        const uint32_t tempty0 = cluster_addr(&tempty[0], 0), tempty1 = cluster_addr(&tempty[1], 0);
        uint8_t* ag_stage = smem + ST * STAGE2_BYTES + 256 +
                            (warp - 2) * 32 * AG_ROW_PITCH;   // all-gather mode only
        float amx = 0.0f;                      // this thread's max |C| (NaN ignored)
        int i = 0;
        for (int t = pair; t < total; t += n_pairs, ++i) {
            const int acc = i & 1;
            const uint32_t acc_ph = (i >> 1) & 1;
            int tm, tn;
            tile_coords(t, p.num_m, p.num_n, tm, tn);
            if (!mbar_wait_warp(&tfull[acc], acc_ph, p.status)) break;
            tc_fence_after();
            const int row = tm * 2 * BM + (int)rank * BM + row_in_tile;
            const bool row_ok = row < p.M;
            float sa, inv_c;
            row_scales<OutT>(p, row, row_ok, sa, inv_c);
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                __syncwarp();  // tcgen05.ld is warp-collective: reconverge first
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + c * 32, r);
                tmem_ld_wait();
                if (c == BN / 32 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(acc ? tempty1 : tempty0);
                }
                const int col0 = tn * BN + c * 32;
                if (col0 >= p.N) continue;  // warp-uniform
                float v[32];
                scale_chunk(r, v, sa, p, col0, lane);
                if (p.amax && row_ok) amax_chunk(amx, v, p.N - col0);
                if constexpr (kAllGather && sizeof(OutT) != 1) {
                    if (ag_stage_chunk<OutT>(v, c, tn, tm * 2 * BM + (int)rank * BM + quad * 32,
                                             lane, ag_stage, p))
                        continue;
                }
                if (!row_ok) continue;
                if constexpr (!kAllGather)
                    store_chunk(static_cast<OutT*>(p.C) + (int64_t)row * p.N + col0, v, p.N - col0,
                                inv_c);
                else
                    ag_store_row_chunk<OutT>(v, row, col0, inv_c, p);
            }
        }
        if (p.amax) {   // non-negative floats order like their bit patterns
            const float m = warp_max(amx);
            if (lane == 0) atomicMax(reinterpret_cast<unsigned*>(p.amax), __float_as_uint(m));
        }
        if constexpr (kAllGather) ag_finish(lane, p);
    }

    tc_fence_before();
    cluster_sync();   // the leader's MMAs (which read this CTA's shared memory) are done
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, TMEM_COLS);
    }
}

// ------------------------------------------------------------------ fp32 as 3 x TF32
// C = A B in fp32 on the tensor cores (kind::tf32).  Each operand is split as
// x = hi + lo with hi = x with its low 13 mantissa bits cleared (exactly a TF32
// value) and lo = x - hi (exact in fp32, |lo| < 2^-10 |x|), and
//   A B ~= hi(A) hi(B) + hi(A) lo(B) + lo(A) hi(B)
// -- the dropped lo(A) lo(B) term and the TF32 reading of lo are ~2^-20 of
// each product, so the result keeps fp32-level accuracy (the plugin's bound is
// 1e-3 relative).  k_tf32_split writes hi and lo of A; k_tf32_split_t those of
// B transposed to [N, K], so both operands are K-major (for MN-major 32-bit
// operands the MMA wants a different shared-memory swizzle).  The GEMM streams
// hi and lo tiles of A and B through one ring and issues three MMAs per K=8 step.
constexpr uint32_t kTf32HiMask = 0xFFFFE000u;

__global__ void __launch_bounds__(256) k_tf32_split(const float* __restrict__ x, int64_t n,
                                                    float* __restrict__ hi, float* __restrict__ lo) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n / 4; i += stride) {
        const float4 v = reinterpret_cast<const float4*>(x)[i];
        float4 h, l;
        h.x = __uint_as_float(__float_as_uint(v.x) & kTf32HiMask); l.x = v.x - h.x;
        h.y = __uint_as_float(__float_as_uint(v.y) & kTf32HiMask); l.y = v.y - h.y;
        h.z = __uint_as_float(__float_as_uint(v.z) & kTf32HiMask); l.z = v.z - h.z;
        h.w = __uint_as_float(__float_as_uint(v.w) & kTf32HiMask); l.w = v.w - h.w;
        reinterpret_cast<float4*>(hi)[i] = h;
        reinterpret_cast<float4*>(lo)[i] = l;
    }
    for (int64_t i = n / 4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const float h = __uint_as_float(__float_as_uint(x[i]) & kTf32HiMask);
        hi[i] = h;
        lo[i] = x[i] - h;
    }
}

// B [K, N] -> hi(B)^T, lo(B)^T [N, K]: 32 x 32 tiles through shared memory
__global__ void __launch_bounds__(256) k_tf32_split_t(const float* __restrict__ b, int K, int N,
                                                      float* __restrict__ hi_t,
                                                      float* __restrict__ lo_t) {
    __shared__ float tile[32][33];
    const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 32 x 8 threads
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
        const int k = k0 + ty + i, n = n0 + tx;
        tile[ty + i][tx] = (k < K && n < N) ? b[(int64_t)k * N + n] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
        const int n = n0 + ty + i, k = k0 + tx;
        if (n < N && k < K) {
            const float v = tile[tx][ty + i];
            const float h = __uint_as_float(__float_as_uint(v) & kTf32HiMask);
            hi_t[(int64_t)n * K + k] = h;
            lo_t[(int64_t)n * K + k] = v - h;
        }
    }
}

__device__ __forceinline__ void tc_mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

template <int TBN>
struct Tf32Cfg {
    static constexpr int BK = SLAB / 4;                    // 32 K elements a stage
    static constexpr int A_BYTES = BM * SLAB;              // [128 rows x 32 K] 16 KiB
    static constexpr int B_BYTES = TBN * SLAB;             // [TBN rows x 32 K]
    static constexpr int STAGE = 2 * A_BYTES + 2 * B_BYTES;
    static constexpr int STAGES = (200 * 1024) / STAGE;
    static constexpr int SMEM = STAGES * STAGE + 1024 + 256;
    static constexpr uint32_t IDESC = make_idesc(2, 2, 0, 0, BM, TBN);   // TF32, both K-major
};

template <int TBN>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tf32x3(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
                  const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmBl,
                  float* __restrict__ C, int M, int N, int K, int* status) {
    using CF = Tf32Cfg<TBN>;
    constexpr int ST = CF::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + ST * CF::STAGE);
    uint64_t* empty = full + ST;
    uint64_t* tfull = empty + ST;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_m = (M + BM - 1) / BM, num_n = (N + TBN - 1) / TBN;
    const int num_kb = (K + CF::BK - 1) / CF::BK;
    const int total = num_m * num_n;

    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 2 * TBN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                int tm, tn;
                tile_coords(t, num_m, num_n, tm, tn);
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&empty[s], ph ^ 1, status)) { ok = false; break; }
                    uint8_t* st = smem + s * CF::STAGE;
                    mbar_arrive_expect_tx(&full[s], CF::STAGE);
                    tma_load_2d(st, &tmAh, &full[s], kb * CF::BK, tm * BM);
                    tma_load_2d(st + CF::A_BYTES, &tmAl, &full[s], kb * CF::BK, tm * BM);
                    tma_load_2d(st + 2 * CF::A_BYTES, &tmBh, &full[s], kb * CF::BK, tn * TBN);
                    tma_load_2d(st + 2 * CF::A_BYTES + CF::B_BYTES, &tmBl, &full[s], kb * CF::BK,
                                tn * TBN);
                    if (++s == ST) { s = 0; ph ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            int i = 0;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++i) {
                const int acc = i & 1;
                if (!mbar_wait(&tempty[acc], ((i >> 1) & 1) ^ 1, status)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * TBN;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&full[s], ph, status)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t ah = smem_u32(smem + s * CF::STAGE), al = ah + CF::A_BYTES;
                    const uint32_t bh = ah + 2 * CF::A_BYTES, bl = bh + CF::B_BYTES;
#pragma unroll
                    for (int k = 0; k < SLAB / 32; ++k) {   // K = 8 (32 bytes) per MMA
                        const uint64_t dah = smem_desc_sw128(ah + k * 32, 16, 1024);
                        const uint64_t dal = smem_desc_sw128(al + k * 32, 16, 1024);
                        const uint64_t dbh = smem_desc_sw128(bh + k * 32, 16, 1024);
                        const uint64_t dbl = smem_desc_sw128(bl + k * 32, 16, 1024);
                        // the two small cross terms first, then the large one
                        tc_mma_tf32(d_tmem, dal, dbh, CF::IDESC, (kb | k) != 0);
                        tc_mma_tf32(d_tmem, dah, dbl, CF::IDESC, 1);
                        tc_mma_tf32(d_tmem, dah, dbh, CF::IDESC, 1);
                    }
                    tc_commit(&empty[s]);
                    if (++s == ST) { s = 0; ph ^= 1; }
                }
                if (ok) tc_commit(&tfull[acc]);
            }
            tc_commit(drain);
            mbar_wait(drain, 0, status);
        }
    } else {
        const int quad = warp & 3;
        const int row_in_tile = quad * 32 + lane;
        int i = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x, ++i) {
            const int acc = i & 1;
            int tm, tn;
            tile_coords(t, num_m, num_n, tm, tn);
            if (!mbar_wait_warp(&tfull[acc], (i >> 1) & 1, status)) break;
            tc_fence_after();
            const int row = tm * BM + row_in_tile;
            const bool row_ok = row < M;
            for (int c = 0; c < TBN / 32; ++c) {
                uint32_t r[32];
                __syncwarp();
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * TBN + c * 32, r);
                tmem_ld_wait();
                if (c == TBN / 32 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[acc]);
                }
                const int col0 = tn * TBN + c * 32;
                if (col0 >= N || !row_ok) continue;
                float* out = C + (int64_t)row * N + col0;
                if (col0 + 32 <= N && (reinterpret_cast<uintptr_t>(out) & 15u) == 0) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *reinterpret_cast<float4*>(out + j) =
                            make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                        __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)   // constant indices: r stays in registers
                        if (col0 + j < N) out[j] = __uint_as_float(r[j]);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 2 * TBN);
    }
}

// ------------------------------------------------------------------ host side
// Row-major [rows, cols] matrix of `es`-byte elements, box [box_rows, 128 bytes], 128B swizzle.
int make_tmap(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int es,
              int box_rows) {
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(cols * es)};
    cuuint32_t box[2] = {(cuuint32_t)(128 / es), (cuuint32_t)box_rows};
    return encode_tmap(m, base, es, 2, dims, strides, box);
}

struct AllGather {
    void* const* peers = nullptr;              // device array of `world` C pointers
    int world = 1, rank = 0;
    unsigned long long* const* mbox = nullptr; // device array of `world` mailboxes
    unsigned seq = 0;
};

// How many SM pairs can hold a k_gemm_tc2 cluster at once on this device (0 if
// none), with the kernel's shared-memory attribute set on first use.
template <bool kFP8, typename OutT, bool kAG = false>
int pair_slots() {
    static std::atomic<int> slots[64];   // per device ordinal: 0 unknown, -1 none, else count
    constexpr int smem = kAG ? SMEM2_BYTES_AG : SMEM2_BYTES;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return 0;
    int n = slots[dev].load();
    if (n == 0) {
        auto kern = k_gemm_tc2<kFP8, OutT, kAG>;
        n = -1;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             smem);
        if (e == cudaSuccess) {
            cudaLaunchConfig_t cfg = {};
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = 2;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.gridDim = dim3(2 * sm_count());
            cfg.blockDim = dim3(kThreads);
            cfg.dynamicSmemBytes = smem;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int c = 0;
            e = cudaOccupancyMaxActiveClusters(&c, kern, &cfg);
            if (e == cudaSuccess && c > 0) n = c;
        }
        // a refusal above only means: no pairs (clear that error, and no other)
        if (e != cudaSuccess) cudaGetLastError();
        slots[dev].store(n);
    }
    return n > 0 ? n : 0;
}

template <bool kFP8, typename OutT, bool kAG = false>
int launch_pair(const CUtensorMap& tmA, const CUtensorMap& tmB, const TcParams& p, int pairs,
                cudaStream_t st) {
    const int total = p.num_m * p.num_n;
    const int n_pairs = total < pairs ? total : pairs;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * n_pairs);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kAG ? SMEM2_BYTES_AG : SMEM2_BYTES;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    AMPB_CHECK_CUDA(cudaLaunchKernelEx(&cfg, k_gemm_tc2<kFP8, OutT, kAG>, tmA, tmB, p));
    AMPB_CHECK_LAUNCH("k_gemm_tc2");
    return AMP_OK;
}

template <bool kFP8, typename OutT>
int launch_tc(const void* A, const void* B, void* C, int M, int N, int K, const float* sa,
              const float* sb, int mode, cudaStream_t st, const float* sc = nullptr,
              float* amax = nullptr, const AllGather* ag = nullptr) {
    const int es = kFP8 ? 1 : 2;
    AMPB_REQUIRE(M > 0 && N > 0 && K > 0, AMP_ERR_INVALID, "GEMM sizes must be positive");
    AMPB_REQUIRE(A && B && (C || ag), AMP_ERR_INVALID, "NULL operand");
    AMPB_REQUIRE((int64_t)K * es % 16 == 0 && (int64_t)N * es % 16 == 0, AMP_ERR_UNSUPPORTED,
                 "tensor-core GEMM needs K and N to be multiples of %d (got K=%d N=%d)", 16 / es,
                 K, N);
    AMPB_REQUIRE(aligned16(A) && aligned16(B), AMP_ERR_INVALID,
                 "A and B must be 16-byte aligned");
    CUtensorMap tmA, tmB;
    int rc;
    if ((rc = make_tmap(&tmA, A, M, K, es, BM))) return rc;
    if ((rc = make_tmap(&tmB, B, K, N, es, SLAB / es))) return rc;
    int* status = nullptr;
    if ((rc = device_status(&status))) return rc;
    TcParams p;
    p.M = M;
    p.N = N;
    p.K = K;
    p.num_m = (M + BM - 1) / BM;
    p.num_n = (N + BN - 1) / BN;
    p.num_kb = (int)(((int64_t)K * es + SLAB - 1) / SLAB);
    p.C = C;
    p.scale_a = sa;
    p.scale_b = sb;
    p.scale_mode = mode;
    p.scale_c = sc;
    p.amax = amax;
    p.status = status;
    p.peers = nullptr;
    p.world = 1;
    p.rank = 0;
    p.ldc = N;
    p.col_base = 0;
    p.mbox = nullptr;
    p.seq = 0;
    p.done = nullptr;
    if (ag) {
        AMPB_REQUIRE(ag->peers && ag->mbox, AMP_ERR_INVALID, "all-gather needs C and mailbox tables");
        AMPB_REQUIRE(ag->world >= 1 && ag->world <= kMaxPeers && ag->rank >= 0 &&
                         ag->rank < ag->world, AMP_ERR_INVALID, "rank %d / world %d outside [0, %d)",
                     ag->rank, ag->world, kMaxPeers);
        AMPB_REQUIRE(ag->seq != 0, AMP_ERR_INVALID, "sequence numbers start at 1");
        AMPB_REQUIRE((int64_t)N * ag->world <= INT32_MAX, AMP_ERR_UNSUPPORTED, "C too wide");
        void* done = nullptr;
        AMPB_CHECK_CUDA(cudaGetSymbolAddress(&done, g_allgather_done));
        AMPB_CHECK_CUDA(cudaMemsetAsync(done, 0, sizeof(unsigned), st));
        p.peers = ag->peers;
        p.world = ag->world;
        p.rank = ag->rank;
        p.ldc = N * ag->world;
        p.col_base = N * ag->rank;
        p.mbox = ag->mbox;
        p.seq = ag->seq;
        p.done = static_cast<unsigned*>(done);
    }
    if (amax) AMPB_CHECK_CUDA(cudaMemsetAsync(amax, 0, sizeof(float), st));
    {
        // 256 x 256 tiles on SM pairs once there are enough of them to fill the pairs
        const int pm = (M + 2 * BM - 1) / (2 * BM), pn = p.num_n;
        const int pairs = ag ? pair_slots<kFP8, OutT, true>() : pair_slots<kFP8, OutT, false>();
        if (pairs > 0 && (int64_t)pm * pn >= pairs) {
            p.num_m = pm;
            return ag ? launch_pair<kFP8, OutT, true>(tmA, tmB, p, pairs, st)
                      : launch_pair<kFP8, OutT, false>(tmA, tmB, p, pairs, st);
        }
    }
    auto kern = ag ? k_gemm_tc<kFP8, OutT, true> : k_gemm_tc<kFP8, OutT, false>;
    static std::atomic<uint64_t> attr_done[2];  // one bit per device ordinal (< 64) and mode
    int dev = 0;
    AMPB_CHECK_CUDA(cudaGetDevice(&dev));
    std::atomic<uint64_t>& done_bits = attr_done[ag ? 1 : 0];
    if (dev >= 64 || !(done_bits.load() >> dev & 1)) {
        AMPB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             ag ? SMEM_BYTES_AG : SMEM_BYTES));
        if (dev < 64) done_bits.fetch_or(1ull << dev);
    }
    const int total = p.num_m * p.num_n;
    const int grid = total < sm_count() ? total : sm_count();
    kern<<<grid, kThreads, ag ? SMEM_BYTES_AG : SMEM_BYTES, st>>>(tmA, tmB, p);
    AMPB_CHECK_LAUNCH("k_gemm_tc");
    return AMP_OK;
}

}  // namespace

int gemm_bf16_dev(const void* A, const void* B, void* C, int c_is_bf16, int M, int N, int K,
                  cudaStream_t st) {
    if (c_is_bf16)
        return launch_tc<false, __nv_bfloat16>(A, B, C, M, N, K, nullptr, nullptr, kNoScale, st);
    return launch_tc<false, float>(A, B, C, M, N, K, nullptr, nullptr, kNoScale, st);
}

int gemm_fp8_dev(const void* A, const void* B, const float* sa, const float* sb, int mode,
                 void* C, int c_dtype, int M, int N, int K, cudaStream_t st,
                 const float* scale_c = nullptr, float* amax_c = nullptr,
                 const AllGather* ag = nullptr) {
    AMPB_REQUIRE(mode == kTensorScale || mode == kRowColScale, AMP_ERR_INVALID,
                 "FP8 scale mode must be 1 (per tensor) or 2 (per row of A / column of B)");
    AMPB_REQUIRE(sa && sb, AMP_ERR_INVALID, "FP8 GEMM needs both scale pointers");
    switch (c_dtype) {
        case AMP_DTYPE_F32:
            return launch_tc<true, float>(A, B, C, M, N, K, sa, sb, mode, st, nullptr, amax_c, ag);
        case AMP_DTYPE_BF16:
            return launch_tc<true, __nv_bfloat16>(A, B, C, M, N, K, sa, sb, mode, st, nullptr,
                                                  amax_c, ag);
        case AMP_DTYPE_E4M3:
            AMPB_REQUIRE(scale_c, AMP_ERR_INVALID, "E4M3 output needs scale_c");
            return launch_tc<true, uint8_t>(A, B, C, M, N, K, sa, sb, mode, st, scale_c, amax_c,
                                            ag);
        default:
            set_error(AMP_ERR_INVALID, "C dtype must be AMP_DTYPE_F32, _BF16 or _E4M3");
            return AMP_ERR_INVALID;
    }
}

// fp32 GEMM on the tensor cores (3 x TF32), opt-in.  Needs K and N multiples of 4 and
// 16-byte aligned operands (TMA: the row pitch of A and of B^T is K * 4 bytes,
// of C N * 4); the split operands live in library scratch
// (staging slots 8 and 9), so calls on one device must be ordered.
bool gemm_fp32_tc_eligible(const float* A, const float* B, const float* C, int M, int N, int K) {
    return M >= 1 && N >= 1 && K >= 1 && K % 4 == 0 && N % 4 == 0 && aligned16(A) &&
           aligned16(B) && aligned16(C);
}

int gemm_fp32_tc_dev(const float* A, const float* B, float* C, int M, int N, int K,
                     cudaStream_t st) {
    AMPB_REQUIRE(gemm_fp32_tc_eligible(A, B, C, M, N, K), AMP_ERR_UNSUPPORTED,
                 "3xTF32 GEMM needs K, N multiples of 4 and 16-byte aligned operands");
    const int64_t na = (int64_t)M * K, nb = (int64_t)K * N;
    void *sa = nullptr, *sb = nullptr;
    int rc;
    if ((rc = staging_get(8, (size_t)na * 8, &sa))) return rc;
    if ((rc = staging_get(9, (size_t)nb * 8, &sb))) return rc;
    float* ah = static_cast<float*>(sa);
    float* al = ah + na;
    float* bh = static_cast<float*>(sb);
    float* bl = bh + nb;
    const int sgrid_a = (int)std::min<int64_t>((na / 4 + 255) / 256 + 1, (int64_t)sm_count() * 16);
    k_tf32_split<<<sgrid_a, 256, 0, st>>>(A, na, ah, al);
    AMPB_CHECK_LAUNCH("k_tf32_split");
    k_tf32_split_t<<<dim3((N + 31) / 32, (K + 31) / 32), 256, 0, st>>>(B, K, N, bh, bl);
    AMPB_CHECK_LAUNCH("k_tf32_split_t");
    // 128-column tiles while they fill the machine, 64-column tiles otherwise
    const int tbn = (int64_t)((M + BM - 1) / BM) * ((N + 127) / 128) >= sm_count() ? 128 : 64;
    CUtensorMap tAh, tAl, tBh, tBl;
    if ((rc = make_tmap(&tAh, ah, M, K, 4, BM)) || (rc = make_tmap(&tAl, al, M, K, 4, BM)) ||
        (rc = make_tmap(&tBh, bh, N, K, 4, tbn)) || (rc = make_tmap(&tBl, bl, N, K, 4, tbn)))
        return rc;
    int* status = nullptr;
    if ((rc = device_status(&status))) return rc;
    auto go = [&](auto kern, int smem) {
        static std::atomic<uint64_t> attr_done[2];   // one bit per device ordinal and tile width
        int dev = 0;
        AMPB_CHECK_CUDA(cudaGetDevice(&dev));
        std::atomic<uint64_t>& bits = attr_done[tbn == 128 ? 1 : 0];
        if (dev >= 64 || !(bits.load() >> dev & 1)) {
            AMPB_CHECK_CUDA(
                cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
            if (dev < 64) bits.fetch_or(1ull << dev);
        }
        const int64_t total = (int64_t)((M + BM - 1) / BM) * ((N + tbn - 1) / tbn);
        const int grid = (int)std::min<int64_t>(total, sm_count());
        kern<<<grid, kThreads, smem, st>>>(tAh, tAl, tBh, tBl, C, M, N, K, status);
        AMPB_CHECK_LAUNCH("k_gemm_tf32x3");
        return AMP_OK;
    };
    if (tbn == 128) return go(k_gemm_tf32x3<128>, Tf32Cfg<128>::SMEM);
    return go(k_gemm_tf32x3<64>, Tf32Cfg<64>::SMEM);
}

}  // namespace ampb

using namespace ampb;

extern "C" {

// C = A B for fp32 row-major operands as three TF32 products on the tensor cores
// (see gemm_fp32_tc_dev).  Opt-in: the tensor core's fp32 accumulation makes the
// error grow with K (max_rel_err 1.9e-4 / 6e-4 / 1.5e-3 at 1024 / 2048 / 4096
// cubed for U[-1,1] inputs, against 3e-5 .. 1.7e-4 for amp_gemm_fp32_dev).
int amp_gemm_fp32_3xtf32_dev(const float* A, const float* B, float* C, int M, int N, int K,
                             void* stream) {
    AMPB_REQUIRE(M >= 1 && N >= 1 && K >= 1 && A && B && C, AMP_ERR_INVALID, "bad GEMM arguments");
    return gemm_fp32_tc_dev(A, B, C, M, N, K, as_stream(stream));
}

int amp_gemm_bf16_dev(const void* A, const void* B, void* C, int c_dtype, int M, int N, int K,
                      void* stream) {
    AMPB_REQUIRE(c_dtype == AMP_DTYPE_F32 || c_dtype == AMP_DTYPE_BF16, AMP_ERR_INVALID,
                 "C dtype must be AMP_DTYPE_F32 or AMP_DTYPE_BF16");
    return gemm_bf16_dev(A, B, C, c_dtype == AMP_DTYPE_BF16, M, N, K, as_stream(stream));
}

int amp_gemm_fp8e4m3_dev(const uint8_t* A, const uint8_t* B, const float* scale_a,
                         const float* scale_b, int scale_mode, void* C, int c_dtype, int M, int N,
                         int K, void* stream) {
    AMPB_REQUIRE(c_dtype == AMP_DTYPE_F32 || c_dtype == AMP_DTYPE_BF16, AMP_ERR_INVALID,
                 "C dtype must be AMP_DTYPE_F32 or AMP_DTYPE_BF16");
    return gemm_fp8_dev(A, B, scale_a, scale_b, scale_mode, C, c_dtype, M, N, K,
                        as_stream(stream));
}

// N-sharded GEMM with the all-gather of C fused into the epilogue (see the
// all-gather mode above).  B is this rank's [K, N] column block; C_peers and
// mailboxes are DEVICE arrays of `world` pointers (this rank's own at [rank]),
// every C being [M, N * world] row-major; seq is the mailbox sequence number of
// this exchange (the same on every rank, never 0, one more per exchange).
int amp_gemm_bf16_allgather_dev(const void* A, const void* B, void* const* C_peers, int c_dtype,
                                int rank, int world, void* const* mailboxes, unsigned seq, int M,
                                int N, int K, void* stream) {
    AMPB_REQUIRE(c_dtype == AMP_DTYPE_F32 || c_dtype == AMP_DTYPE_BF16, AMP_ERR_INVALID,
                 "C dtype must be AMP_DTYPE_F32 or AMP_DTYPE_BF16");
    AllGather ag;
    ag.peers = C_peers;
    ag.world = world;
    ag.rank = rank;
    ag.mbox = reinterpret_cast<unsigned long long* const*>(mailboxes);
    ag.seq = seq;
    if (c_dtype == AMP_DTYPE_BF16)
        return launch_tc<false, __nv_bfloat16>(A, B, nullptr, M, N, K, nullptr, nullptr, kNoScale,
                                               as_stream(stream), nullptr, nullptr, &ag);
    return launch_tc<false, float>(A, B, nullptr, M, N, K, nullptr, nullptr, kNoScale,
                                   as_stream(stream), nullptr, nullptr, &ag);
}

int amp_gemm_fp8e4m3_allgather_dev(const uint8_t* A, const uint8_t* B, const float* scale_a,
                                   const float* scale_b, int scale_mode, void* const* C_peers,
                                   int c_dtype, int rank, int world, void* const* mailboxes,
                                   unsigned seq, int M, int N, int K, void* stream) {
    AMPB_REQUIRE(c_dtype == AMP_DTYPE_F32 || c_dtype == AMP_DTYPE_BF16, AMP_ERR_INVALID,
                 "C dtype must be AMP_DTYPE_F32 or AMP_DTYPE_BF16");
    AllGather ag;
    ag.peers = C_peers;
    ag.world = world;
    ag.rank = rank;
    ag.mbox = reinterpret_cast<unsigned long long* const*>(mailboxes);
    ag.seq = seq;
    return gemm_fp8_dev(A, B, scale_a, scale_b, scale_mode, nullptr, c_dtype, M, N, K,
                        as_stream(stream), nullptr, nullptr, &ag);
}

int amp_gemm_fp8e4m3_ex_dev(const uint8_t* A, const uint8_t* B, const float* scale_a,
                            const float* scale_b, int scale_mode, void* C, int c_dtype,
                            const float* scale_c, float* amax_c, int M, int N, int K,
                            void* stream) {
    return gemm_fp8_dev(A, B, scale_a, scale_b, scale_mode, C, c_dtype, M, N, K,
                        as_stream(stream), scale_c, amax_c);
}

// Host-pointer forms (the plugin convention of amp_plugin.h): A, B, C in host
// memory, all device work done and synchronised before returning.
int amp_user_gemm_bf16(const uint16_t* A, const uint16_t* B, void* C, int c_dtype, int M, int N,
                       int K) {
    AMPB_REQUIRE(M > 0 && N > 0 && K > 0 && A && B && C, AMP_ERR_INVALID, "bad GEMM arguments");
    AMPB_REQUIRE(c_dtype == AMP_DTYPE_F32 || c_dtype == AMP_DTYPE_BF16, AMP_ERR_INVALID,
                 "C dtype must be AMP_DTYPE_F32 or AMP_DTYPE_BF16");
    const size_t a = (size_t)M * K * 2, b = (size_t)K * N * 2;
    const size_t c = (size_t)M * N * (c_dtype == AMP_DTYPE_F32 ? 4 : 2);
    void *dA, *dB, *dC;
    int rc;
    if ((rc = staging_get(0, a, &dA)) || (rc = staging_get(1, b, &dB)) ||
        (rc = staging_get(2, c, &dC)))
        return rc;
    cudaStream_t st = 0;
    AMPB_CHECK_CUDA(cudaMemcpyAsync(dA, A, a, cudaMemcpyHostToDevice, st));
    AMPB_CHECK_CUDA(cudaMemcpyAsync(dB, B, b, cudaMemcpyHostToDevice, st));
    if ((rc = gemm_bf16_dev(dA, dB, dC, c_dtype == AMP_DTYPE_BF16, M, N, K, st))) return rc;
    AMPB_CHECK_CUDA(cudaMemcpyAsync(C, dC, c, cudaMemcpyDeviceToHost, st));
    AMPB_CHECK_CUDA(cudaStreamSynchronize(st));
    const int status = amp_device_status(1);
    if (status) return status;
    return staging_end_of_call();
}

int amp_user_gemm_fp8e4m3(const uint8_t* A, const uint8_t* B, const float* scale_a,
                          const float* scale_b, int scale_mode, void* C, int c_dtype, int M,
                          int N, int K) {
    AMPB_REQUIRE(M > 0 && N > 0 && K > 0 && A && B && C && scale_a && scale_b, AMP_ERR_INVALID,
                 "bad GEMM arguments");
    AMPB_REQUIRE(c_dtype == AMP_DTYPE_F32 || c_dtype == AMP_DTYPE_BF16, AMP_ERR_INVALID,
                 "C dtype must be AMP_DTYPE_F32 or AMP_DTYPE_BF16");
    AMPB_REQUIRE(scale_mode == 1 || scale_mode == 2, AMP_ERR_INVALID, "scale_mode must be 1 or 2");
    const size_t a = (size_t)M * K, b = (size_t)K * N;
    const size_t c = (size_t)M * N * (c_dtype == AMP_DTYPE_F32 ? 4 : 2);
    const size_t ns_a = scale_mode == 2 ? (size_t)M : 1, ns_b = scale_mode == 2 ? (size_t)N : 1;
    void *dA, *dB, *dC, *dS;
    int rc;
    if ((rc = staging_get(0, a, &dA)) || (rc = staging_get(1, b, &dB)) ||
        (rc = staging_get(2, c, &dC)) || (rc = staging_get(3, (ns_a + ns_b) * 4, &dS)))
        return rc;
    float* dsa = static_cast<float*>(dS);
    float* dsb = dsa + ns_a;
    cudaStream_t st = 0;
    AMPB_CHECK_CUDA(cudaMemcpyAsync(dA, A, a, cudaMemcpyHostToDevice, st));
    AMPB_CHECK_CUDA(cudaMemcpyAsync(dB, B, b, cudaMemcpyHostToDevice, st));
    AMPB_CHECK_CUDA(cudaMemcpyAsync(dsa, scale_a, ns_a * 4, cudaMemcpyHostToDevice, st));
    AMPB_CHECK_CUDA(cudaMemcpyAsync(dsb, scale_b, ns_b * 4, cudaMemcpyHostToDevice, st));
    if ((rc = gemm_fp8_dev(dA, dB, dsa, dsb, scale_mode, dC, c_dtype, M, N, K, st)))
        return rc;
    AMPB_CHECK_CUDA(cudaMemcpyAsync(C, dC, c, cudaMemcpyDeviceToHost, st));
    AMPB_CHECK_CUDA(cudaStreamSynchronize(st));
    const int status = amp_device_status(1);
    if (status) return status;
    return staging_end_of_call();
}

}  // extern "C"
