// comm.cu -- the collective layer of the sharded hot path as a C ABI over NCCL,
// for C and C++ hosts (no torch, no Python).
//
// Replaces the reference's include/collective.hpp / src/collective.cpp, which
// wraps NCCL behind AMP::CommGroup and CommUniqueId:
//   comm_get_unique_id  (collective.hpp:60, collective.cpp:101-109) -> amp_comm_unique_id
//   comm_init_rank      (collective.hpp:64-65, collective.cpp:111-123) -> amp_comm_init_rank
//   comm_destroy        (collective.hpp:71) -> amp_comm_destroy
//   allreduce / allgather / broadcast / barrier (collective.hpp:79-104,
//   collective.cpp:143-160, 188-203) -> amp_comm_allreduce / _allgather /
//   _broadcast / _barrier
// and adds the two sharded operations of the hot path in their NCCL form:
//   amp_gemm_{bf16,fp8e4m3}_sharded_dev  N-split GEMM + all-gather of C
//   amp_flash_attn_fwd_sharded_dev       (batch*head)-split attention + all-gather
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, or AMP_B200_NCCL_LIB),
// so the library keeps needing only the driver: AMP's validator, which links
// no CUDA, still dlopens it without NCCL installed.  In a process that has
// NCCL loaded already (torch), the same soname resolves to that copy.
//
// Ops are asynchronous on the given stream, as in the reference; the caller
// synchronises.  Every rank must make the same calls in the same order.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "runtime.h"

struct amp_comm {
    ncclComm_t nccl;
    int rank, world, device;
};

namespace ampb {
namespace {

struct Nccl {
    ncclResult_t (*get_unique_id)(ncclUniqueId*);
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t,
                               ncclComm_t, cudaStream_t);
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                               cudaStream_t);
    ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t,
                              cudaStream_t);
    ncclResult_t (*group_start)();
    ncclResult_t (*group_end)();
    const char* (*error_string)(ncclResult_t);
    ncclResult_t (*get_version)(int*);
};

std::once_flag g_nccl_once;
Nccl g_nccl;
bool g_nccl_ok = false;
char g_nccl_why[256] = "";

void load_nccl() {
    const char* name = std::getenv("AMP_B200_NCCL_LIB");
    if (!name || !*name) name = "libnccl.so.2";
    void* h = dlopen(name, RTLD_NOW | RTLD_LOCAL);
    if (!h) {
        std::snprintf(g_nccl_why, sizeof g_nccl_why, "dlopen(%s): %s", name, dlerror());
        return;
    }
    auto sym = [&](const char* s, auto& fp) {
        void* p = dlsym(h, s);
        std::memcpy(&fp, &p, sizeof p);
        return p != nullptr;
    };
    const bool ok = sym("ncclGetUniqueId", g_nccl.get_unique_id) &&
                    sym("ncclCommInitRank", g_nccl.comm_init_rank) &&
                    sym("ncclCommDestroy", g_nccl.comm_destroy) &&
                    sym("ncclAllReduce", g_nccl.all_reduce) &&
                    sym("ncclAllGather", g_nccl.all_gather) &&
                    sym("ncclBroadcast", g_nccl.broadcast) &&
                    sym("ncclGroupStart", g_nccl.group_start) &&
                    sym("ncclGroupEnd", g_nccl.group_end) &&
                    sym("ncclGetErrorString", g_nccl.error_string) &&
                    sym("ncclGetVersion", g_nccl.get_version);
    if (!ok) {
        std::snprintf(g_nccl_why, sizeof g_nccl_why, "%s lacks an NCCL entry point", name);
        return;
    }
    g_nccl_ok = true;
}

int nccl(const Nccl** out) {
    std::call_once(g_nccl_once, load_nccl);
    AMPB_REQUIRE(g_nccl_ok, AMP_ERR_UNSUPPORTED, "NCCL is not available: %s", g_nccl_why);
    *out = &g_nccl;
    return AMP_OK;
}

int nccl_status(const Nccl* n, ncclResult_t r, const char* where) {
    if (r == ncclSuccess) return AMP_OK;
    set_error(AMP_ERR_COMM, "%s: NCCL error %d (%s)", where, (int)r, n->error_string(r));
    return AMP_ERR_COMM;
}

#define AMPB_NCCL(n, call)                                                 \
    do {                                                                   \
        int _rc = ::ampb::nccl_status((n), (n)->call, #call);              \
        if (_rc) return _rc;                                               \
    } while (0)

int dtype_of(int t, ncclDataType_t* nt, size_t* es) {
    switch (t) {
        case AMP_DTYPE_F32: *nt = ncclFloat32; *es = 4; return AMP_OK;
        case AMP_DTYPE_BF16: *nt = ncclBfloat16; *es = 2; return AMP_OK;
        case AMP_DTYPE_E4M3: *nt = ncclUint8; *es = 1; return AMP_OK;
        case AMP_DTYPE_I32: *nt = ncclInt32; *es = 4; return AMP_OK;
        default: break;
    }
    set_error(AMP_ERR_INVALID, "unknown element type %d", t);
    return AMP_ERR_INVALID;
}

int op_of(int op, ncclRedOp_t* no) {
    switch (op) {
        case AMP_REDUCE_SUM: *no = ncclSum; return AMP_OK;
        case AMP_REDUCE_MAX: *no = ncclMax; return AMP_OK;
        case AMP_REDUCE_MIN: *no = ncclMin; return AMP_OK;
        case AMP_REDUCE_PROD: *no = ncclProd; return AMP_OK;
        default: break;
    }
    set_error(AMP_ERR_INVALID, "unknown reduction %d", op);
    return AMP_ERR_INVALID;
}

int check_comm(const amp_comm* c) {
    AMPB_REQUIRE(c != nullptr && c->nccl != nullptr, AMP_ERR_INVALID, "NULL communicator");
    int dev = -1;
    AMPB_CHECK_CUDA(cudaGetDevice(&dev));
    AMPB_REQUIRE(dev == c->device, AMP_ERR_INVALID,
                 "current device %d is not the communicator's device %d", dev, c->device);
    return AMP_OK;
}

// [p][M][row_bytes] (rank-major blocks of the N-split C) -> [M][p * row_bytes]
__global__ void k_interleave_rows(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                  int p, int M, int64_t row_bytes, int vec16) {
    const int64_t rows = (int64_t)p * M;
    for (int64_t rr = blockIdx.x; rr < rows; rr += gridDim.x) {
        const int r = (int)(rr / M), m = (int)(rr % M);
        const uint8_t* s = src + rr * row_bytes;
        uint8_t* d = dst + ((int64_t)m * p + r) * row_bytes;
        if (vec16) {
            const int64_t n16 = row_bytes >> 4;
            for (int64_t i = threadIdx.x; i < n16; i += blockDim.x)
                reinterpret_cast<uint4*>(d)[i] = reinterpret_cast<const uint4*>(s)[i];
        } else {
            for (int64_t i = threadIdx.x; i < row_bytes; i += blockDim.x) d[i] = s[i];
        }
    }
}

int interleave_rows(const void* src, void* dst, int p, int M, int64_t row_bytes,
                    cudaStream_t st) {
    if ((int64_t)p * M == 0 || row_bytes == 0) return AMP_OK;
    const int vec16 = (row_bytes % 16 == 0) && aligned16(src) && aligned16(dst);
    const int64_t rows = (int64_t)p * M;
    const int grid = (int)(rows < (int64_t)sm_count() * 16 ? rows : (int64_t)sm_count() * 16);
    k_interleave_rows<<<grid, 256, 0, st>>>(static_cast<const uint8_t*>(src),
                                            static_cast<uint8_t*>(dst), p, M, row_bytes, vec16);
    AMPB_CHECK_LAUNCH("k_interleave_rows");
    return AMP_OK;
}

size_t gemm_ws_bytes(int M, int Np, int world, int c_dtype) {
    const size_t es = c_dtype == AMP_DTYPE_F32 ? 4 : c_dtype == AMP_DTYPE_E4M3 ? 1 : 2;
    return (size_t)M * Np * world * es;
}

// Common part of the two sharded GEMMs: this rank's block is already in
// ws[rank]; gather every rank's block in place, then lay C out row-major.
int gather_c(amp_comm* c, void* C, int c_dtype, int M, int Np, void* ws, cudaStream_t st) {
    const Nccl* n = nullptr;
    int rc = nccl(&n);
    if (rc) return rc;
    const size_t es = c_dtype == AMP_DTYPE_F32 ? 4 : c_dtype == AMP_DTYPE_E4M3 ? 1 : 2;
    const size_t block = (size_t)M * Np * es;
    uint8_t* w = static_cast<uint8_t*>(ws);
    if (c->world > 1)
        AMPB_NCCL(n, all_gather(w + (size_t)c->rank * block, w, block, ncclUint8, c->nccl, st));
    return interleave_rows(ws, C, c->world, M, (int64_t)Np * es, st);
}

int check_gemm_args(amp_comm* c, const void* A, const void* B, void* C, int c_dtype, int M,
                    int Np, int K, void* ws, size_t ws_bytes) {
    int rc = check_comm(c);
    if (rc) return rc;
    AMPB_REQUIRE(M > 0 && Np > 0 && K > 0, AMP_ERR_INVALID, "bad GEMM shape %d x %d x %d", M, Np,
                 K);
    AMPB_REQUIRE(A && B && C && ws, AMP_ERR_INVALID, "NULL operand or workspace");
    AMPB_REQUIRE(c_dtype == AMP_DTYPE_F32 || c_dtype == AMP_DTYPE_BF16, AMP_ERR_INVALID,
                 "C must be fp32 or bf16");
    const size_t need = gemm_ws_bytes(M, Np, c->world, c_dtype);
    AMPB_REQUIRE(ws_bytes >= need, AMP_ERR_INVALID, "workspace of %zu bytes, need %zu", ws_bytes,
                 need);
    return AMP_OK;
}

}  // namespace
}  // namespace ampb

using namespace ampb;

extern "C" {

int amp_comm_available(void) {
    const Nccl* n = nullptr;
    return nccl(&n) == AMP_OK ? 1 : 0;
}

int amp_comm_nccl_version(int* version) {
    AMPB_REQUIRE(version != nullptr, AMP_ERR_INVALID, "NULL version");
    const Nccl* n = nullptr;
    int rc = nccl(&n);
    if (rc) return rc;
    AMPB_NCCL(n, get_version(version));
    return AMP_OK;
}

int amp_comm_unique_id(uint8_t* id) {
    AMPB_REQUIRE(id != nullptr, AMP_ERR_INVALID, "NULL id buffer");
    static_assert(sizeof(ncclUniqueId) <= AMP_COMM_UNIQUE_ID_BYTES, "unique id size");
    const Nccl* n = nullptr;
    int rc = nccl(&n);
    if (rc) return rc;
    ncclUniqueId u;
    AMPB_NCCL(n, get_unique_id(&u));
    std::memset(id, 0, AMP_COMM_UNIQUE_ID_BYTES);
    std::memcpy(id, &u, sizeof u);
    return AMP_OK;
}

int amp_comm_init_rank(amp_comm** out, int rank, int world, int device_id, const uint8_t* id) {
    AMPB_REQUIRE(out != nullptr && id != nullptr, AMP_ERR_INVALID, "NULL argument");
    *out = nullptr;
    AMPB_REQUIRE(world >= 1 && rank >= 0 && rank < world, AMP_ERR_INVALID,
                 "rank %d outside a world of %d", rank, world);
    AMPB_REQUIRE(device_id >= 0, AMP_ERR_INVALID, "bad device id %d", device_id);
    const Nccl* n = nullptr;
    int rc = nccl(&n);
    if (rc) return rc;
    AMPB_CHECK_CUDA(cudaSetDevice(device_id));
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof u);
    ncclComm_t nc = nullptr;
    AMPB_NCCL(n, comm_init_rank(&nc, world, u, rank));
    amp_comm* c = new (std::nothrow) amp_comm{nc, rank, world, device_id};
    if (!c) {
        n->comm_destroy(nc);
        set_error(AMP_ERR_INVALID, "out of host memory");
        return AMP_ERR_INVALID;
    }
    *out = c;
    return AMP_OK;
}

int amp_comm_destroy(amp_comm* c) {
    if (c == nullptr) return AMP_OK;
    const Nccl* n = nullptr;
    int rc = nccl(&n);
    if (rc) return rc;
    rc = nccl_status(n, n->comm_destroy(c->nccl), "ncclCommDestroy");
    delete c;
    return rc;
}

int amp_comm_rank(const amp_comm* c, int* rank, int* world, int* device_id) {
    AMPB_REQUIRE(c != nullptr, AMP_ERR_INVALID, "NULL communicator");
    if (rank) *rank = c->rank;
    if (world) *world = c->world;
    if (device_id) *device_id = c->device;
    return AMP_OK;
}

int amp_comm_allreduce(amp_comm* c, void* buf, size_t count, int dtype, int op, void* stream) {
    ncclDataType_t nt;
    ncclRedOp_t no;
    size_t es;
    int rc;
    if ((rc = dtype_of(dtype, &nt, &es)) || (rc = op_of(op, &no))) return rc;
    AMPB_REQUIRE(dtype != AMP_DTYPE_E4M3, AMP_ERR_INVALID, "no arithmetic on E4M3 codes");
    if ((rc = check_comm(c))) return rc;
    if (count == 0) return AMP_OK;
    AMPB_REQUIRE(buf != nullptr, AMP_ERR_INVALID, "NULL buffer");
    const Nccl* n = nullptr;
    if ((rc = nccl(&n))) return rc;
    AMPB_NCCL(n, all_reduce(buf, buf, count, nt, no, c->nccl, as_stream(stream)));
    return AMP_OK;
}

int amp_comm_allreduce_max_f32(amp_comm* c, float* buf, size_t count, void* stream) {
    return amp_comm_allreduce(c, buf, count, AMP_DTYPE_F32, AMP_REDUCE_MAX, stream);
}

int amp_comm_allgather(amp_comm* c, const void* send, void* recv, size_t count, int dtype,
                       void* stream) {
    ncclDataType_t nt;
    size_t es;
    int rc;
    if ((rc = dtype_of(dtype, &nt, &es))) return rc;
    if ((rc = check_comm(c))) return rc;
    if (count == 0) return AMP_OK;
    AMPB_REQUIRE(send != nullptr && recv != nullptr, AMP_ERR_INVALID, "NULL buffer");
    const Nccl* n = nullptr;
    if ((rc = nccl(&n))) return rc;
    AMPB_NCCL(n, all_gather(send, recv, count, nt, c->nccl, as_stream(stream)));
    return AMP_OK;
}

int amp_comm_broadcast(amp_comm* c, void* buf, size_t count, int dtype, int root, void* stream) {
    ncclDataType_t nt;
    size_t es;
    int rc;
    if ((rc = dtype_of(dtype, &nt, &es))) return rc;
    if ((rc = check_comm(c))) return rc;
    AMPB_REQUIRE(root >= 0 && root < c->world, AMP_ERR_INVALID, "root %d outside a world of %d",
                 root, c->world);
    if (count == 0) return AMP_OK;
    AMPB_REQUIRE(buf != nullptr, AMP_ERR_INVALID, "NULL buffer");
    const Nccl* n = nullptr;
    if ((rc = nccl(&n))) return rc;
    AMPB_NCCL(n, broadcast(buf, buf, count, nt, root, c->nccl, as_stream(stream)));
    return AMP_OK;
}

// The reference's barrier is a 1-float all-reduce on a buffer it allocates
// and frees per call (collective.cpp:188-203); here the float lives in the
// per-device staging pool, so the barrier allocates nothing after its first use.
int amp_comm_barrier(amp_comm* c, void* stream) {
    int rc = check_comm(c);
    if (rc) return rc;
    void* one = nullptr;
    if ((rc = staging_get(7, sizeof(float), &one))) return rc;
    const Nccl* n = nullptr;
    if ((rc = nccl(&n))) return rc;
    AMPB_NCCL(n, all_reduce(one, one, 1, ncclFloat32, ncclSum, c->nccl, as_stream(stream)));
    return AMP_OK;
}

size_t amp_gemm_sharded_workspace_bytes(int M, int Np, int world, int c_dtype) {
    if (M <= 0 || Np <= 0 || world <= 0) return 0;
    return gemm_ws_bytes(M, Np, world, c_dtype);
}

int amp_gemm_bf16_sharded_dev(amp_comm* c, const void* A, const void* B_slab, void* C,
                              int c_dtype, int M, int Np, int K, void* workspace,
                              size_t workspace_bytes, void* stream) {
    int rc = check_gemm_args(c, A, B_slab, C, c_dtype, M, Np, K, workspace, workspace_bytes);
    if (rc) return rc;
    const size_t es = c_dtype == AMP_DTYPE_F32 ? 4 : 2;
    void* mine = static_cast<uint8_t*>(workspace) + (size_t)c->rank * M * Np * es;
    if ((rc = amp_gemm_bf16_dev(A, B_slab, mine, c_dtype, M, Np, K, stream))) return rc;
    return gather_c(c, C, c_dtype, M, Np, workspace, as_stream(stream));
}

int amp_gemm_fp8e4m3_sharded_dev(amp_comm* c, const uint8_t* A, const uint8_t* B_slab,
                                 const float* scale_a, const float* scale_b, int scale_mode,
                                 void* C, int c_dtype, int M, int Np, int K, void* workspace,
                                 size_t workspace_bytes, void* stream) {
    int rc = check_gemm_args(c, A, B_slab, C, c_dtype, M, Np, K, workspace, workspace_bytes);
    if (rc) return rc;
    const size_t es = c_dtype == AMP_DTYPE_F32 ? 4 : 2;
    void* mine = static_cast<uint8_t*>(workspace) + (size_t)c->rank * M * Np * es;
    if ((rc = amp_gemm_fp8e4m3_dev(A, B_slab, scale_a, scale_b, scale_mode, mine, c_dtype, M, Np,
                                   K, stream)))
        return rc;
    return gather_c(c, C, c_dtype, M, Np, workspace, as_stream(stream));
}

int amp_flash_attn_fwd_sharded_dev(amp_comm* c, const void* q, const void* k, const void* v,
                                   void* o, float* lse, int B, int Hq, int Hkv, int S_q,
                                   int S_kv, int D, int causal, float scale, void* stream) {
    int rc = check_comm(c);
    if (rc) return rc;
    AMPB_REQUIRE(q && k && v && o, AMP_ERR_INVALID, "NULL q, k, v or o");
    AMPB_REQUIRE(B > 0 && Hq > 0 && Hkv > 0 && S_q > 0 && S_kv > 0 && D > 0 && Hq % Hkv == 0,
                 AMP_ERR_INVALID, "bad attention shape B=%d Hq=%d Hkv=%d S_q=%d S_kv=%d D=%d", B,
                 Hq, Hkv, S_q, S_kv, D);
    // Shards are contiguous slices of the outer dims: batch*head when every
    // query head has its own kv head, whole sequences (batch) under GQA so
    // that a kv head stays with its query group.
    const int p = c->world;
    int b0, nb, hq, hkv;
    if (Hq == Hkv) {
        AMPB_REQUIRE((B * Hq) % p == 0, AMP_ERR_INVALID, "%d batch*heads do not split over %d",
                     B * Hq, p);
        nb = 1;
        hq = hkv = B * Hq / p;
        b0 = c->rank * hq;  // in units of (batch*head) rows of S x D
    } else {
        AMPB_REQUIRE(B % p == 0, AMP_ERR_INVALID,
                     "GQA attention splits over whole sequences: batch %d over %d ranks", B, p);
        nb = B / p;
        hq = Hq;
        hkv = Hkv;
        b0 = c->rank * nb;
    }
    const int64_t q_rows = (int64_t)(Hq == Hkv ? 1 : Hq), kv_rows = (int64_t)(Hq == Hkv ? 1 : Hkv);
    const int64_t q_off = (int64_t)b0 * q_rows * S_q * D, kv_off = (int64_t)b0 * kv_rows * S_kv * D;
    const int64_t lse_off = (int64_t)b0 * q_rows * S_q;
    const uint16_t* qs = static_cast<const uint16_t*>(q) + q_off;
    const uint16_t* ks = static_cast<const uint16_t*>(k) + kv_off;
    const uint16_t* vs = static_cast<const uint16_t*>(v) + kv_off;
    uint16_t* os = static_cast<uint16_t*>(o) + q_off;
    float* ls = lse ? lse + lse_off : nullptr;
    if ((rc = amp_flash_attn_fwd_bf16_dev(qs, ks, vs, os, ls, nb, hq, hkv, S_q, S_kv, D, causal,
                                          scale, stream)))
        return rc;
    if (p == 1) return AMP_OK;
    const Nccl* n = nullptr;
    if ((rc = nccl(&n))) return rc;
    const size_t o_count = (size_t)nb * hq * S_q * D, l_count = (size_t)nb * hq * S_q;
    cudaStream_t st = as_stream(stream);
    AMPB_NCCL(n, group_start());
    rc = nccl_status(n, n->all_gather(os, o, o_count, ncclBfloat16, c->nccl, st), "ncclAllGather(O)");
    if (!rc && ls)
        rc = nccl_status(n, n->all_gather(ls, lse, l_count, ncclFloat32, c->nccl, st),
                         "ncclAllGather(lse)");
    const int rc_end = nccl_status(n, n->group_end(), "ncclGroupEnd");
    return rc ? rc : rc_end;
}

}  // extern "C"
