/* amp_b200.h -- C ABI of the B200 (sm_100a) kernels.
 *
 * Conventions, shared with the plugin contract in amp_plugin.h:
 *   - every entry point returns an int status: 0 on success, nonzero on a
 *     hard failure (amp_plugin.h: "caller treats this as a hard error");
 *     negative values are argument/usage errors (AMP_ERR_*), positive values
 *     are CUDA runtime error codes; amp_last_error() returns the message;
 *   - `amp_user_*` functions take HOST pointers and own all device work
 *     (allocate, copy in, launch, copy out, synchronise) before returning,
 *     exactly like amp_user_gemm_fp32;
 *   - `*_dev` functions take DEVICE pointers and a stream (a cudaStream_t
 *     passed as void*, NULL = legacy default stream); they only enqueue work
 *     and do not synchronise;
 *   - bf16 data is passed as raw 16-bit patterns (uint16_t / void*), E4M3 as
 *     uint8_t codes; no CUDA or torch types appear in any signature.
 */
#ifndef AMP_B200_H
#define AMP_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define AMP_API __attribute__((visibility("default")))
#else
#define AMP_API
#endif

#define AMP_OK 0
#define AMP_ERR_INVALID (-1)     /* bad argument (size, pointer, alignment, config)  */
#define AMP_ERR_UNSUPPORTED (-2) /* valid request this build does not implement        */
#define AMP_ERR_TIMEOUT (-3)     /* a bounded device-side wait expired                 */
#define AMP_ERR_NO_DEVICE (-4)   /* no CUDA device visible                             */
#define AMP_ERR_COMM (-5)        /* a collective (NCCL) call failed                    */

/* Element types named in signatures that take a dtype selector. */
#define AMP_DTYPE_F32 0
#define AMP_DTYPE_BF16 1
#define AMP_DTYPE_E4M3 2   /* FP8 GEMM output; moved as bytes by the collectives */
#define AMP_DTYPE_I32 3    /* collectives only (block tables, context lengths) */

/* Reductions of amp_comm_allreduce, in the order of AMP::ReduceOp
 * (include/collective.hpp:49). */
#define AMP_REDUCE_SUM 0
#define AMP_REDUCE_MAX 1
#define AMP_REDUCE_MIN 2
#define AMP_REDUCE_PROD 3

/* Message for the last nonzero status returned on this thread. */
AMP_API const char* amp_last_error(void);
/* ABI version: major*10000 + minor*100 + patch. */
AMP_API int amp_abi_version(void);
/* Synchronises the current device and reports whether any kernel's bounded
 * wait expired since the last clear (AMP_ERR_TIMEOUT) -- the device-side
 * failure path of the pipelined tensor-core kernels, which end instead of
 * hanging.  clear != 0 resets the flag. */
AMP_API int amp_device_status(int clear);
/* The amp_user_* entry points stage their host data in per-device device
 * buffers that grow as needed and are kept across calls, so repeated calls do
 * not pay cudaMalloc / cudaFree.  AMP's plugin contract says a plugin frees its
 * device buffers before returning (include/amp_plugin.h:32-39): this call
 * frees them on the current device (after synchronising it), and with the
 * environment variable AMP_B200_RELEASE_STAGING=1 every amp_user_* call does so
 * itself before it returns. */
AMP_API int amp_release_staging(void);
/* Sets the current device's limit on every bounded device-side wait (mbarrier
 * waits of the pipelined kernels, peer-mailbox polls); 0 restores the default
 * of 2 s; limits below 1 ms act as 1 ms (kernels read the limit only after
 * a wait has lasted that long).  Takes effect for kernels launched after it
 * returns (it synchronises the device first).  The reference has no device-side waits; this is the
 * failure path's knob, e.g. a short limit in a test whose peer never posts. */
AMP_API int amp_set_wait_timeout_ns(uint64_t ns);

/* ------------------------------------------------------------------------
 * FP8 E4M3 per-tensor amax-scaled quantise / dequantise.
 * Replaces the host codec AMP::fp8::f32_to_e4m3 / e4m3_to_f32
 * (include/fp8.hpp:15-63), which has no amax and no device path; the amax
 * plumbing it would feed is GemmDesc::d_amax_c (include/gemm_vendor.hpp:55-56).
 * Semantics (bit-exact against the oracle):
 *   amax  = max |x| (NaN ignored);  scale = amax/448 (IEEE fp32), 1 if amax==0
 *   inv   = min(RN(1/scale), FLT_MAX)
 *   q[i]  = E4M3_RNE_satfinite(RN(x[i] * inv))
 *   y[i]  = bf16_RNE(e4m3_to_f32(q[i]) * scale)
 * ---------------------------------------------------------------------- */

/* Scratch bytes amp_fp8_quant_e4m3_dev / amp_fp8_amax_bf16_dev need (per-block
 * partial maxima; a small constant, independent of n). */
AMP_API size_t amp_fp8_quant_workspace_bytes(int64_t n);

/* Quantise n bf16 values; writes n codes, *scale_out and (if non-NULL) *amax_out. */
AMP_API int amp_fp8_quant_e4m3_dev(const void* x_bf16, int64_t n, uint8_t* q, float* scale_out,
                           float* amax_out, void* workspace, size_t workspace_bytes,
                           void* stream);

/* amax of n bf16 values into *amax_out (device float); the first half of the
 * quantiser, for sharded tensors whose global amax is an all-reduce(MAX) of
 * the per-rank values. */
AMP_API int amp_fp8_amax_bf16_dev(const void* x_bf16, int64_t n, float* amax_out, void* workspace,
                          size_t workspace_bytes, void* stream);

/* Sharded amax without NCCL: amax of this rank's n values, exchanged with every
 * rank of the node through the peer mailboxes below, max over ranks into
 * *amax_out (device float).  Replaces the all-reduce(MAX) of one float that
 * AMP's collective layer would do (include/collective.hpp:79-85, allreduce).
 * `mailboxes` is a DEVICE array of `world` mailbox pointers (own at [rank]);
 * every rank calls with the same seq, which starts at 1 and grows by one per
 * call, wrapping from 2^32 - 2 back to 1: consecutive calls on one set of
 * mailboxes use alternate rows (seq & 1), so seq never repeats its parity.
 * A peer that does not post within 2 s sets AMP_ERR_TIMEOUT in
 * amp_device_status(). */
AMP_API int amp_fp8_amax_allreduce_peer_dev(const void* x_bf16, int64_t n, float* amax_out,
                                            void* workspace, size_t workspace_bytes,
                                            void* const* mailboxes, int rank, int world,
                                            unsigned seq, void* stream);

/* Second half: quantise with a given device-resident amax. */
AMP_API int amp_fp8_quant_e4m3_from_amax_dev(const void* x_bf16, int64_t n, const float* amax_in,
                                     uint8_t* q, float* scale_out, void* stream);

/* Dequantise n codes with the device-resident scale into bf16. */
AMP_API int amp_fp8_dequant_e4m3_dev(const uint8_t* q, int64_t n, const float* scale, void* y_bf16,
                             void* stream);

/* Allocation-free form of amp_fp8_quant_e4m3_dev, for callers that cannot
 * call cudaMalloc when they quantise (an engine plugin limited to the memory
 * its engine hands it, a runtime that owns and budgets every device
 * allocation).  No counterpart in the reference.  The amax pass's partial
 * maxima live in a library-owned 8 KiB device array per GPU (held until
 * process exit), so only input and outputs are passed and nothing is
 * allocated; any n >= 0 is accepted (the pass grid-strides, its partial count
 * is capped at the array's size).  The first call on each device resolves the
 * array's address (cudaGetSymbolAddress) and caches it for the process: make
 * it before any stream capture, and not across a cudaDeviceReset.  Calls
 * share the array and it keeps the last call's partials: calls whose kernels
 * overlap on one GPU race. */
AMP_API int amp_fp8_quant_e4m3_noalloc_dev(const void* x_bf16, int64_t n, uint8_t* q,
                                           float* scale_out, float* amax_out, void* stream);

/* Host-pointer forms: quantise (and, if y_bf16 != NULL, dequantise back). */
AMP_API int amp_user_fp8_quant_e4m3(const uint16_t* x_bf16, int64_t n, uint8_t* q, float* scale_out,
                            uint16_t* y_bf16);
AMP_API int amp_user_fp8_dequant_e4m3(const uint8_t* q, int64_t n, float scale, uint16_t* y_bf16);

/* ------------------------------------------------------------------------
 * fp32 GEMM, row-major C[M,N] = A[M,K] * B[K,N].
 * Replaces AMP::launch_matmul(TileCfg, dA, dB, dC, M, N, K, stream)
 * (kernels/matmul.cuh:96-98, dispatcher kernels/matmul.cu:24-35).  The host
 * pointer form is amp_user_gemm_fp32 in amp_plugin.h.
 * amp_gemm_fp32_dev accumulates with FFMA (one rounding per multiply-add).
 * ---------------------------------------------------------------------- */
AMP_API int amp_gemm_fp32_dev(const float* A, const float* B, float* C, int M, int N, int K,
                              void* stream);
/* Exact form: each product rounded to fp32, then each sum, k ascending from
 * 0 -- the order and rounding of AMP's cpu_reference_gemm
 * (tests/amp_validate_kernel.cpp:20-28), so C is bit-identical to the CPU
 * reference AMP's validator and parity dump compare against.  The plugin
 * amp_user_gemm_fp32 and amp_gemm_fp32_tile_dev use this form. */
AMP_API int amp_gemm_fp32_exact_dev(const float* A, const float* B, float* C, int M, int N,
                                    int K, void* stream);
/* Exact form named by one of AMP's tile configs (bm,bn,bk) in {(16,16,16),
 * (32,16,16), (32,32,16), (32,32,32)} or (0,0,0); any other config is an
 * error, as in the reference dispatcher ("unknown FP32 tile cfg").  The tile
 * names the dump entry; the kernel's own blocking is chosen by size. */
AMP_API int amp_gemm_fp32_tile_dev(int bm, int bn, int bk, const float* A, const float* B,
                                   float* C, int M, int N, int K, void* stream);

/* fp32 C = A B (row-major) on the tensor cores as three TF32 products of a
 * hi/lo split of each operand, opt-in: ~5x the FFMA kernel's rate at 4096^3, but
 * the tensor core's fp32 accumulation makes the error grow with K (max_rel_err
 * 1.9e-4 at 1024^3 for U[-1,1] inputs; AMP's validator inputs in [-10, 10] fail
 * its 1e-3 bar), so the plugin stays on the exact CUDA-core form.  K and N must be
 * multiples of 4 and the operands 16-byte aligned; uses library scratch (calls on
 * one device must be ordered). */
AMP_API int amp_gemm_fp32_3xtf32_dev(const float* A, const float* B, float* C, int M, int N,
                                     int K, void* stream);
/* ------------------------------------------------------------------------
 * Tensor-core GEMM (tcgen05), row-major C[M,N] = A[M,K] * B[K,N].
 * bf16: replaces AMP::launch_matmul_bf16 (kernels/matmul.cuh:103-105,
 *       kernels/matmul.cu:47-110), fp32 accumulate, C in fp32 (AMP's choice)
 *       or bf16 (c_dtype).
 * FP8:  replaces AMP::launch_matmul_fp8e4m3 (kernels/matmul.cuh:120-123,
 *       kernels/matmul.cu:235-270 -> cuBLASLt).  scale_mode 1: per-tensor,
 *       scale_a/scale_b point to one device float each (as cuBLASLt's
 *       A/B_SCALE_POINTER); scale_mode 2: scale_a[M] per row of A and
 *       scale_b[N] per column of B.  C = (A8 * B8) * sa * sb.
 * Requirements: K and N multiples of 8 (bf16) / 16 (FP8), 16-byte aligned
 * A and B; any M.  Asynchronous on `stream`.
 * ---------------------------------------------------------------------- */
AMP_API int amp_gemm_bf16_dev(const void* A, const void* B, void* C, int c_dtype, int M, int N,
                              int K, void* stream);
AMP_API int amp_gemm_fp8e4m3_dev(const uint8_t* A, const uint8_t* B, const float* scale_a,
                                 const float* scale_b, int scale_mode, void* C, int c_dtype,
                                 int M, int N, int K, void* stream);

/* N-sharded GEMM with the all-gather of C fused into the epilogue; replaces
 * AMP's per-rank launch + ncclAllGather of C (include/collective.hpp:87-89,
 * src/collective.cpp:155-160).  B is this rank's [K, N] column block; every
 * rank holds C [M, N * world] row-major (amp_peer_buffer_create), and this
 * rank's epilogue stores its block C[:, rank*N : (rank+1)*N] into all of them
 * over NVLink.  C_peers / mailboxes: DEVICE arrays of `world` pointers (own at
 * [rank]); seq: the mailbox sequence number of this call (the same on every
 * rank, never 0, one more per exchange).  On return of the stream work every
 * rank's C is complete.  The next call into the same C may start only after
 * every rank has finished reading it.  One call in flight per device. */
AMP_API int amp_gemm_bf16_allgather_dev(const void* A, const void* B, void* const* C_peers,
                                        int c_dtype, int rank, int world, void* const* mailboxes,
                                        unsigned seq, int M, int N, int K, void* stream);
AMP_API int amp_gemm_fp8e4m3_allgather_dev(const uint8_t* A, const uint8_t* B,
                                           const float* scale_a, const float* scale_b,
                                           int scale_mode, void* const* C_peers, int c_dtype,
                                           int rank, int world, void* const* mailboxes,
                                           unsigned seq, int M, int N, int K, void* stream);
/* FP8 GEMM with output-side quantisation (AMP's GemmDesc d_scale_c / d_amax_c,
 * include/gemm_vendor.hpp:55-56, which it hands to cuBLASLt):
 *   v = scale_a * scale_b * (A8 . B8)  (fp32 accumulate)
 *   c_dtype F32 / BF16: C = v;  E4M3: C = E4M3_RNE_sat(RN(v * inv)), inv =
 *   min(RN(1/scale_c[0]), FLT_MAX) -- the quantiser's encode, so C dequantises
 *   as code * scale_c.  amax_c (optional, device float, overwritten) = max |v|
 *   over C, NaN ignored: the input to the next step's scale_c. */
AMP_API int amp_gemm_fp8e4m3_ex_dev(const uint8_t* A, const uint8_t* B, const float* scale_a,
                                    const float* scale_b, int scale_mode, void* C, int c_dtype,
                                    const float* scale_c, float* amax_c, int M, int N, int K,
                                    void* stream);

/* ------------------------------------------------------------------------
 * FlashAttention-2 forward, bf16 in/out, fp32 softmax and accumulation.
 * Replaces AMP::launch_flash_attn_bf16 (kernels/flash_attn.cuh:50-58,
 * kernels/flash_attn.cu:202-283): Q, O [B, Hq, S_q, head_dim]; K, V
 * [B, Hkv, S_kv, head_dim]; lse [B, Hq, S_q] = ln sum exp(scale * q.k) (may
 * be NULL).  GQA: kv head = q head / (Hq / Hkv).  causal != 0 masks key j >
 * query i (top-left aligned, as the reference).  scale <= 0 selects
 * 1/sqrt(head_dim) (AttnCfg::scale semantics).  head_dim 64 or 128.
 * ---------------------------------------------------------------------- */
AMP_API int amp_flash_attn_fwd_bf16_dev(const void* Q, const void* K, const void* V, void* O,
                                        float* lse, int B, int Hq, int Hkv, int S_q, int S_kv,
                                        int head_dim, int causal, float scale, void* stream);
/* (batch*head)-sharded attention with the all-gather of O and lse fused into
 * the epilogue; replaces the per-rank launch + ncclAllGather of O / lse
 * (include/collective.hpp:87-89).  Q, K, V hold this rank's slice (B*Hq and
 * B*Hkv heads); O_peers / lse_peers are DEVICE arrays of `world` pointers to
 * every rank's full O [bh_total][S_q][head_dim] bf16 and lse [bh_total][S_q]
 * fp32 (amp_peer_buffer_create; lse_peers may be NULL); this rank's
 * batch*head 0 is global index bh_base.  Mailboxes / seq / reuse rules as for
 * amp_gemm_bf16_allgather_dev. */
AMP_API int amp_flash_attn_fwd_allgather_dev(const void* Q, const void* K, const void* V,
                                             void* const* O_peers, float* const* lse_peers,
                                             int rank, int world, int bh_base,
                                             void* const* mailboxes, unsigned seq, int B, int Hq,
                                             int Hkv, int S_q, int S_kv, int head_dim, int causal,
                                             float scale, void* stream);

/* FlashAttention-2 backward (AMP has none; its forward's lse is "required for the
 * backward pass", kernels/flash_attn.cuh:48).  Inputs: the forward's Q, K, V, O
 * and lse (natural log) and dO; outputs dQ [B,Hq,S_q,D], dK and dV [B,Hkv,S_kv,D]
 * bf16 (a kv head's dK / dV sum over its query heads).  P is recomputed from
 * lse.  causal needs S_q == S_kv.  Workspace: amp_flash_attn_bwd_workspace_bytes
 * (the fp32 row sums of dO * O). */
AMP_API size_t amp_flash_attn_bwd_workspace_bytes(int B, int Hq, int S_q);
AMP_API int amp_flash_attn_bwd_bf16_dev(const void* Q, const void* K, const void* V,
                                        const void* O, const void* dO, const float* lse,
                                        void* dQ, void* dK, void* dV, int B, int Hq, int Hkv,
                                        int S_q, int S_kv, int head_dim, int causal, float scale,
                                        void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Attention over a paged KV cache (block tables of 16-token pages, the
 * format of Sequence::kv_page_ids / kv_page_size_tokens in the reference's
 * include/scheduler.hpp:61,88; the reference has no kernel that reads it).
 *   k_pool, v_pool  [num_pages][Hkv][16][head_dim] bf16
 *   block_table     int32 [B][max_pages_per_seq]: token t of sequence b is
 *                   slot t % 16 of page block_table[b][t / 16]
 *   ctx_lens        int32 [B], tokens in each sequence's cache (device)
 * Slots past a sequence's context in its last page may hold any finite
 * values.  Page ids outside [0, num_pages) are never dereferenced: they are
 * skipped and reported by amp_device_status (AMP_ERR_INVALID).
 * ---------------------------------------------------------------------- */
/* Decode: one query token per sequence, q/out [B][Hq][head_dim], lse [B][Hq]
 * (may be NULL); split-KV with a workspace of
 * amp_paged_decode_workspace_bytes(B, Hq, head_dim, max_context_len) bytes.
 * head_dim 128; Hq/Hkv in {1, 2, 4, 8}. */
AMP_API size_t amp_paged_decode_workspace_bytes(int B, int Hq, int head_dim, int max_context_len);
AMP_API int amp_paged_attn_decode_bf16_dev(const void* q, const void* k_pool, const void* v_pool,
                                           const int32_t* block_table, const int32_t* ctx_lens,
                                           void* out, float* lse, int B, int Hq, int Hkv,
                                           int head_dim, int num_pages, int max_pages_per_seq,
                                           int max_context_len, float scale, void* workspace,
                                           size_t workspace_bytes, void* stream);
/* Prefill: q/out [B][Hq][Lq][head_dim] are the LAST Lq tokens of each
 * sequence's context (ctx_lens[b] >= Lq), causal with bottom-right alignment
 * (query i sits at position ctx_lens[b] - Lq + i); lse [B][Hq][Lq].
 * head_dim 64 or 128. */
AMP_API int amp_paged_attn_prefill_bf16_dev(const void* q, const void* k_pool, const void* v_pool,
                                            const int32_t* block_table, const int32_t* ctx_lens,
                                            void* out, float* lse, int B, int Hq, int Hkv, int Lq,
                                            int head_dim, int num_pages, int max_pages_per_seq,
                                            float scale, void* stream);
/* Host-side check of a block table (host arrays) before upload: ids in range,
 * no page used twice, rows long enough for the contexts. */
AMP_API int amp_paged_validate_block_table(const int32_t* block_table, const int32_t* ctx_lens,
                                           int B, int max_pages_per_seq, int num_pages);

/* Padded block table from per-sequence page lists (AMP's Sequence::kv_page_ids,
 * include/scheduler.hpp:61, concatenated): sequence b's pages are
 * page_ids[seq_start[b] .. seq_start[b+1]) in token order (seq_start has B+1
 * entries).  Writes the HOST table block_table[B][max_pages_per_seq], -1 past
 * each list; AMP_ERR_INVALID if a list is longer than a row or shorter than
 * ceil(ctx_lens[b] / 16). */
AMP_API int amp_paged_pack_block_table(const int32_t* page_ids, const int32_t* seq_start,
                                       const int32_t* ctx_lens, int B, int max_pages_per_seq,
                                       int32_t* block_table);

/* Bytes of one contiguous K (or V) pool [num_pages][Hkv][16][head_dim] bf16; page id p
 * (e.g. from AMP's PagePoolFast, src/pool_fast.cpp:31-60) is row p, replacing the
 * pool's per-page cudaMalloc (src/pool_fast.cpp:11-13). */
AMP_API size_t amp_paged_pool_bytes(int num_pages, int Hkv, int head_dim);

/* Host-pointer form of the attention forward (plugin convention). */
AMP_API int amp_user_flash_attn_fwd_bf16(const uint16_t* Q, const uint16_t* K, const uint16_t* V,
                                         uint16_t* O, float* lse, int B, int Hq, int Hkv, int S_q,
                                         int S_kv, int head_dim, int causal, float scale);

/* Host-pointer forms of the two tensor-core GEMMs (plugin convention:
 * host buffers, all device work finished before returning).  Scales are
 * host arrays: 1 value each (scale_mode 1) or M and N values (scale_mode 2). */
AMP_API int amp_user_gemm_bf16(const uint16_t* A, const uint16_t* B, void* C, int c_dtype, int M,
                               int N, int K);
AMP_API int amp_user_gemm_fp8e4m3(const uint8_t* A, const uint8_t* B, const float* scale_a,
                                  const float* scale_b, int scale_mode, void* C, int c_dtype,
                                  int M, int N, int K);

/* ----------------------------------------------------------------------
 * Peer mailboxes: small device buffers that the other processes of the node
 * write into directly (CUDA IPC over NVLink), for one-word exchanges whose
 * NCCL launch cost would dominate (see amp_fp8_amax_allreduce_peer_dev).
 * A handle is amp_peer_handle_bytes() opaque bytes, shared by the caller
 * (e.g. an all-gather over the process group); peers open it with
 * amp_peer_mailbox_open.  Close peers' mailboxes before their owners free them.
 * ---------------------------------------------------------------------- */
AMP_API size_t amp_peer_mailbox_bytes(void);
AMP_API int amp_peer_handle_bytes(void);
AMP_API int amp_peer_mailbox_create(void** mailbox, void* handle_out);
AMP_API int amp_peer_mailbox_open(const void* handle, void** mailbox);
/* A zeroed device buffer of `bytes` that the other ranks open with
 * amp_peer_mailbox_open (close / free with the mailbox calls): the replicated
 * output C of the all-gather GEMMs below. */
AMP_API int amp_peer_buffer_create(size_t bytes, void** buffer, void* handle_out);
AMP_API int amp_peer_mailbox_close(void* mailbox);
AMP_API int amp_peer_mailbox_free(void* mailbox);
/* all-reduce(max) of one float per rank through the mailboxes (device in/out). */
AMP_API int amp_peer_allreduce_max_f32(const float* in, float* out, void* const* mailboxes,
                                       int rank, int world, unsigned seq, void* stream);

/* ----------------------------------------------------------------------
 * Collectives over NCCL for C and C++ hosts: one communicator per process
 * and GPU.  Replaces AMP's CommGroup / CommUniqueId and their operations
 * (include/collective.hpp:34-104, src/collective.cpp:101-203).  NCCL is
 * loaded at run time (libnccl.so.2, or the file named by AMP_B200_NCCL_LIB),
 * so the library itself does not depend on it.  Operations are asynchronous
 * on `stream`; every rank must issue the same operations in the same order.
 * ---------------------------------------------------------------------- */
#define AMP_COMM_UNIQUE_ID_BYTES 128 /* CommUniqueId::kBytes (collective.hpp:43-46) */
typedef struct amp_comm amp_comm;

/* 1 if NCCL could be loaded, else 0 (amp_last_error() says why). */
AMP_API int amp_comm_available(void);
AMP_API int amp_comm_nccl_version(int* version);
/* comm_get_unique_id (collective.hpp:60): on one rank, then shared out of band. */
AMP_API int amp_comm_unique_id(uint8_t* id /* AMP_COMM_UNIQUE_ID_BYTES */);
/* comm_init_rank (collective.hpp:64-65): makes device_id current, joins the group. */
AMP_API int amp_comm_init_rank(amp_comm** comm, int rank, int world, int device_id,
                               const uint8_t* id);
/* comm_destroy (collective.hpp:71); NULL is a no-op. */
AMP_API int amp_comm_destroy(amp_comm* comm);
AMP_API int amp_comm_rank(const amp_comm* comm, int* rank, int* world, int* device_id);
/* allreduce (collective.hpp:79-80), in place; dtype AMP_DTYPE_F32/BF16/I32,
 * op AMP_REDUCE_*. */
AMP_API int amp_comm_allreduce(amp_comm* comm, void* buf, size_t count, int dtype, int op,
                               void* stream);
/* The quantiser's exchange: all-reduce(MAX) of fp32 values (a sharded amax). */
AMP_API int amp_comm_allreduce_max_f32(amp_comm* comm, float* buf, size_t count, void* stream);
/* allgather (collective.hpp:87-89): recv[r * count ...] = send of rank r;
 * in place when send == recv + rank * count elements. */
AMP_API int amp_comm_allgather(amp_comm* comm, const void* send, void* recv, size_t count,
                               int dtype, void* stream);
/* broadcast (collective.hpp:83-84), in place. */
AMP_API int amp_comm_broadcast(amp_comm* comm, void* buf, size_t count, int dtype, int root,
                               void* stream);
/* barrier (collective.hpp:104): a 1-float all-reduce on library staging memory. */
AMP_API int amp_comm_barrier(amp_comm* comm, void* stream);

/* N-sharded GEMM, NCCL form (no reference counterpart; the reference's GEMM
 * is single-GPU): every rank holds all of A [M,K] and its column slab
 * B_slab [K,Np] of B (columns rank*Np .. rank*Np+Np-1), computes its block of
 * C in `workspace`, all-gathers the blocks in place and lays them out as the
 * full row-major C [M, world*Np] on every rank.  C fp32 or bf16.  The
 * workspace holds world*M*Np elements of C's type. */
AMP_API size_t amp_gemm_sharded_workspace_bytes(int M, int Np, int world, int c_dtype);
AMP_API int amp_gemm_bf16_sharded_dev(amp_comm* comm, const void* A, const void* B_slab, void* C,
                                      int c_dtype, int M, int Np, int K, void* workspace,
                                      size_t workspace_bytes, void* stream);
AMP_API int amp_gemm_fp8e4m3_sharded_dev(amp_comm* comm, const uint8_t* A, const uint8_t* B_slab,
                                         const float* scale_a, const float* scale_b,
                                         int scale_mode, void* C, int c_dtype, int M, int Np,
                                         int K, void* workspace, size_t workspace_bytes,
                                         void* stream);
/* Sharded FlashAttention-2 forward, NCCL form: q/k/v/o/lse as in
 * amp_flash_attn_fwd_bf16_dev on every rank; each rank computes a contiguous
 * slice -- of batch*heads when Hq == Hkv, of whole sequences (batch) under
 * GQA -- into its part of o / lse, then o and lse are all-gathered in place. */
AMP_API int amp_flash_attn_fwd_sharded_dev(amp_comm* comm, const void* q, const void* k,
                                           const void* v, void* o, float* lse, int B, int Hq,
                                           int Hkv, int S_q, int S_kv, int head_dim, int causal,
                                           float scale, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AMP_B200_H */
