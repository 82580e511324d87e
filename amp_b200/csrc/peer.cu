// peer.cu -- peer-memory mailboxes shared by the processes of one node.
//
// The reference's collective layer (include/collective.hpp:34-104) moves data
// with NCCL only.  For the one exchange on the quantiser's path -- the
// all-reduce(max) of one float per step -- NCCL's launch and protocol cost
// (tens of microseconds) is a large share of a ~100 us step, so this file
// gives each rank a small device mailbox that every other rank writes into
// directly over NVLink:
//
//   amp_peer_mailbox_create   cudaMalloc + zero + cudaIpcGetMemHandle
//   amp_peer_mailbox_open     cudaIpcOpenMemHandle of a peer's mailbox
//   amp_peer_mailbox_close / _free
//   amp_peer_buffer_create    the same for a buffer of any size (opened, closed
//                             and freed with the mailbox calls)
//
// A mailbox is [2][kMaxPeers] 64-bit words.  Rank r posts (seq << 32 | value)
// into slot [seq & 1][r] of every rank's mailbox with st.release.sys and
// polls its own [seq & 1][*] with ld.acquire.sys until every word carries the
// step's sequence number.  Alternating the two rows by parity means a fast
// rank can never overwrite a value a slow rank has not read yet: posting step
// s + 2 needs every rank's step s + 1 value, which each rank writes only after
// it has read all of step s.  Sequence numbers run 1 .. 2^32 - 2 and wrap to 1,
// so the parity alternates across the wrap too.  The poll is bounded (2 s) and
// reports through the device status word.
#include <cstring>

#include "peer.cuh"
#include "runtime.h"

namespace ampb {

namespace {

// all-reduce(max) of one non-negative float per rank
__global__ void __launch_bounds__(32) k_mailbox_max(const float* in, float* out,
                                                    unsigned long long* const* mbox, int rank,
                                                    int world, unsigned seq, int* status) {
    __shared__ unsigned got[kMaxPeers];
    const int lane = threadIdx.x;
    const float v = *in;
    mailbox_exchange(mbox, rank, world, seq, __float_as_uint(v), got, status);
    __syncwarp();
    float m = v;
    for (int p = lane; p < world; p += 32) m = fmaxf(m, __uint_as_float(got[p]));
    m = warp_max(m);
    if (lane == 0) *out = m;
}

}  // namespace

int mailbox_max_dev(const float* in, float* out, unsigned long long* const* mbox, int rank,
                    int world, unsigned seq, cudaStream_t st) {
    AMPB_REQUIRE(in && out && mbox, AMP_ERR_INVALID, "NULL argument");
    AMPB_REQUIRE(world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world, AMP_ERR_INVALID,
                 "rank %d / world %d outside [0, %d)", rank, world, kMaxPeers);
    AMPB_REQUIRE(seq != 0, AMP_ERR_INVALID, "sequence numbers start at 1");
    int* status = nullptr;
    int rc = device_status(&status);
    if (rc) return rc;
    k_mailbox_max<<<1, 32, 0, st>>>(in, out, mbox, rank, world, seq, status);
    AMPB_CHECK_LAUNCH("k_mailbox_max");
    return AMP_OK;
}

namespace {

// cudaMalloc + zero + IPC handle of `bytes`; on any failure nothing stays allocated.
int create_shared(size_t bytes, void** out, void* handle_out) {
    void* p = nullptr;
    AMPB_CHECK_CUDA(cudaMalloc(&p, bytes));
    const cudaError_t ez = cudaMemset(p, 0, bytes);
    if (ez != cudaSuccess) {
        cudaFree(p);
        return cuda_status(ez, "cudaMemset");
    }
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        set_error(AMP_ERR_UNSUPPORTED, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
        return AMP_ERR_UNSUPPORTED;
    }
    memcpy(handle_out, &h, sizeof(h));
    *out = p;
    return AMP_OK;
}

}  // namespace

}  // namespace ampb

using namespace ampb;

extern "C" {

size_t amp_peer_mailbox_bytes(void) { return kMailboxBytes; }

int amp_peer_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

int amp_peer_mailbox_create(void** mailbox, void* handle_out) {
    AMPB_REQUIRE(mailbox && handle_out, AMP_ERR_INVALID, "NULL argument");
    return create_shared(kMailboxBytes, mailbox, handle_out);
}

// A device buffer of `bytes` (zeroed) that the other processes of the node can
// map with amp_peer_mailbox_open and write into directly: the replicated output
// of the all-gather GEMM.  Freed with amp_peer_mailbox_free.
int amp_peer_buffer_create(size_t bytes, void** buffer, void* handle_out) {
    AMPB_REQUIRE(buffer && handle_out && bytes > 0, AMP_ERR_INVALID, "bad peer buffer arguments");
    return create_shared(bytes, buffer, handle_out);
}

int amp_peer_mailbox_open(const void* handle, void** mailbox) {
    AMPB_REQUIRE(handle && mailbox, AMP_ERR_INVALID, "NULL argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        set_error(AMP_ERR_UNSUPPORTED, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
        return AMP_ERR_UNSUPPORTED;
    }
    *mailbox = p;
    return AMP_OK;
}

int amp_peer_mailbox_close(void* mailbox) {
    AMPB_REQUIRE(mailbox, AMP_ERR_INVALID, "NULL mailbox");
    AMPB_CHECK_CUDA(cudaIpcCloseMemHandle(mailbox));
    return AMP_OK;
}

int amp_peer_mailbox_free(void* mailbox) {
    AMPB_REQUIRE(mailbox, AMP_ERR_INVALID, "NULL mailbox");
    AMPB_CHECK_CUDA(cudaFree(mailbox));
    return AMP_OK;
}

// mailboxes: DEVICE array of `world` mailbox pointers (this rank's own at [rank]).
int amp_peer_allreduce_max_f32(const float* in, float* out, void* const* mailboxes, int rank,
                               int world, unsigned seq, void* stream) {
    return mailbox_max_dev(in, out, reinterpret_cast<unsigned long long* const*>(mailboxes), rank,
                           world, seq, as_stream(stream));
}

}  // extern "C"
