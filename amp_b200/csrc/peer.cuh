// peer.cuh -- device side of the peer-memory mailboxes (see peer.cu).
#pragma once

#include "common.cuh"
#include "tc_common.cuh"

namespace ampb {

constexpr int kMaxPeers = 64;
constexpr size_t kMailboxBytes = 2 * kMaxPeers * sizeof(unsigned long long);

// Post this rank's word to every rank, then wait for all of them; returns the
// values through `got` (lane p holds rank p's value).  Called by one warp.
__device__ __forceinline__ bool mailbox_exchange(unsigned long long* const* mbox, int rank,
                                                 int world, unsigned seq, unsigned value,
                                                 unsigned* got, int* status) {
    const int lane = threadIdx.x & 31;
    const unsigned long long word = ((unsigned long long)seq << 32) | value;
    const int row = (seq & 1u) * kMaxPeers;
    for (int p = lane; p < world; p += 32) {
        unsigned long long* dst = mbox[p] + row + rank;
        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(dst), "l"(word) : "memory");
    }
    bool ok = true;
    for (int p = lane; p < world; p += 32) {
        const unsigned long long* src = mbox[rank] + row + p;
        const uint64_t t0 = globaltimer_ns();
        unsigned long long v = 0;
        while (true) {
            asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(src) : "memory");
            if ((unsigned)(v >> 32) == seq) break;
            if (wait_expired(globaltimer_ns() - t0, status)) {
                atomicExch(status, AMP_DEV_ERR_TIMEOUT);
                ok = false;
                break;
            }
        }
        got[p] = (unsigned)v;
    }
    return __all_sync(0xffffffffu, ok);
}

}  // namespace ampb
