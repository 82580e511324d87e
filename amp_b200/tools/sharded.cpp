// sharded.cpp -- a C++ host that runs the sharded hot path through the C ABI
// alone: one process per GPU, the NCCL communicator of amp_b200.h
// (amp_comm_*), and the NCCL forms of the N-split GEMM and the
// (batch*head)-split attention.  No Python and no torch are involved.
//
//   amp_b200_sharded <world> [M N K] [--op bf16|fp8|attn|attn_gqa]
//
// The parent forks `world` ranks before anything touches CUDA; rank 0 makes
// the communicator's unique id (AMP's comm_get_unique_id,
// include/collective.hpp:60) and hands it to the others through pipes, the
// out-of-band broadcast collective.hpp:59 asks for.  Rank r runs on device r.
// Every rank builds the same seeded inputs, runs the sharded operation and
// checks the gathered result bit for bit against the same operation run
// unsharded on its own GPU, then reports one line.  Exit status 0 when every
// rank matched.
#include <cuda_runtime.h>
#include <sys/wait.h>
#include <unistd.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "amp_b200.h"

namespace {

#define CK(x)                                                                              \
    do {                                                                                   \
        cudaError_t e_ = (x);                                                              \
        if (e_ != cudaSuccess) {                                                           \
            std::fprintf(stderr, "rank %d: %s: %s\n", rank, #x, cudaGetErrorString(e_));   \
            return 1;                                                                      \
        }                                                                                  \
    } while (0)
#define AK(x)                                                                              \
    do {                                                                                   \
        if ((x) != 0) {                                                                    \
            std::fprintf(stderr, "rank %d: %s: %s\n", rank, #x, amp_last_error());         \
            return 1;                                                                      \
        }                                                                                  \
    } while (0)

uint64_t g_state;
uint32_t next_u32() {  // splitmix64
    uint64_t z = (g_state += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return (uint32_t)((z ^ (z >> 31)) >> 32);
}
// bf16 bit pattern of a value in (-2, 2), and an E4M3 code that is not NaN
uint16_t rand_bf16() { return (uint16_t)((next_u32() & 0x80FF) | 0x3E00 | ((next_u32() & 1) << 8)); }
uint8_t rand_e4m3() {
    uint8_t c = (uint8_t)next_u32();
    return (c & 0x7F) == 0x7F ? (uint8_t)(c - 1) : c;
}

template <typename T>
int upload(const std::vector<T>& h, void** d, int rank) {
    CK(cudaMalloc(d, h.size() * sizeof(T)));
    CK(cudaMemcpy(*d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice));
    return 0;
}

int compare(const void* a, const void* b, size_t bytes, int rank, size_t* diff) {
    std::vector<uint8_t> ha(bytes), hb(bytes);
    CK(cudaMemcpy(ha.data(), a, bytes, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(hb.data(), b, bytes, cudaMemcpyDeviceToHost));
    *diff = 0;
    for (size_t i = 0; i < bytes; ++i) *diff += ha[i] != hb[i];
    return 0;
}

int run_rank(int rank, int world, int M, int N, int K, const std::string& op, int id_fd_in,
             const std::vector<int>& id_fds_out) {
    uint8_t id[AMP_COMM_UNIQUE_ID_BYTES];
    if (rank == 0) {
        AK(amp_comm_unique_id(id));
        for (int fd : id_fds_out)
            if (write(fd, id, sizeof id) != (ssize_t)sizeof id) return 1;
    } else if (read(id_fd_in, id, sizeof id) != (ssize_t)sizeof id) {
        return 1;
    }
    amp_comm* comm = nullptr;
    AK(amp_comm_init_rank(&comm, rank, world, rank, id));
    cudaStream_t st;
    CK(cudaStreamCreate(&st));
    size_t diff = 0, bytes = 0;
    g_state = 12345;  // the same inputs on every rank
    if (op == "attn" || op == "attn_gqa") {
        // q [B, H, S, D], k/v [B, Hkv, S, D]: B = 2 * world sequences, H = 8 heads (Hkv = 8,
        // split over batch*heads; or Hkv = 2 under GQA, split over whole sequences), S = M
        const int B = 2 * world, H = 8, Hkv = op == "attn" ? 8 : 2, S = M, D = 128;
        const size_t n = (size_t)B * H * S * D, nkv = (size_t)B * Hkv * S * D;
        std::vector<uint16_t> hq(n), hk(nkv), hv(nkv);
        for (auto* v : {&hq, &hk, &hv})
            for (auto& x : *v) x = rand_bf16();
        void *q, *k, *v, *o, *o_ref, *l, *l_ref;
        if (upload(hq, &q, rank) || upload(hk, &k, rank) || upload(hv, &v, rank)) return 1;
        CK(cudaMalloc(&o, n * 2));
        CK(cudaMalloc(&o_ref, n * 2));
        CK(cudaMalloc(&l, (size_t)B * H * S * 4));
        CK(cudaMalloc(&l_ref, (size_t)B * H * S * 4));
        AK(amp_flash_attn_fwd_sharded_dev(comm, q, k, v, o, (float*)l, B, H, Hkv, S, S, D, 1, 0.f,
                                          st));
        AK(amp_flash_attn_fwd_bf16_dev(q, k, v, o_ref, (float*)l_ref, B, H, Hkv, S, S, D, 1, 0.f,
                                       st));
        CK(cudaStreamSynchronize(st));
        size_t d2 = 0;
        if (compare(o, o_ref, n * 2, rank, &diff) ||
            compare(l, l_ref, (size_t)B * H * S * 4, rank, &d2))
            return 1;
        diff += d2;
        bytes = n * 2;
    } else {
        const int Np = N / world;
        const bool fp8 = op == "fp8";
        const size_t es = fp8 ? 1 : 2;
        std::vector<uint16_t> a16, b16;
        std::vector<uint8_t> a8, b8;
        if (fp8) {
            a8.resize((size_t)M * K);
            b8.resize((size_t)K * N);
            for (auto& x : a8) x = rand_e4m3();
            for (auto& x : b8) x = rand_e4m3();
        } else {
            a16.resize((size_t)M * K);
            b16.resize((size_t)K * N);
            for (auto& x : a16) x = rand_bf16();
            for (auto& x : b16) x = rand_bf16();
        }
        // this rank's column slab of B, row-major [K, Np]
        std::vector<uint8_t> slab((size_t)K * Np * es);
        const uint8_t* bsrc = fp8 ? b8.data() : reinterpret_cast<const uint8_t*>(b16.data());
        for (int kk = 0; kk < K; ++kk)
            std::memcpy(&slab[(size_t)kk * Np * es], bsrc + ((size_t)kk * N + (size_t)rank * Np) * es,
                        (size_t)Np * es);
        void *A, *Bfull, *Bslab, *C, *C_ref, *ws, *sa, *sb;
        if ((fp8 ? upload(a8, &A, rank) : upload(a16, &A, rank)) ||
            (fp8 ? upload(b8, &Bfull, rank) : upload(b16, &Bfull, rank)) ||
            upload(slab, &Bslab, rank))
            return 1;
        std::vector<float> hsa(M), hsb(N), hsb_slab(Np);
        for (auto& x : hsa) x = 0.5f + (next_u32() & 255) / 256.0f;
        for (auto& x : hsb) x = 0.5f + (next_u32() & 255) / 256.0f;
        std::memcpy(hsb_slab.data(), hsb.data() + (size_t)rank * Np, Np * sizeof(float));
        void* sb_full;
        if (upload(hsa, &sa, rank) || upload(hsb_slab, &sb, rank) || upload(hsb, &sb_full, rank))
            return 1;
        CK(cudaMalloc(&C, (size_t)M * N * 2));
        CK(cudaMalloc(&C_ref, (size_t)M * N * 2));
        const size_t wsb = amp_gemm_sharded_workspace_bytes(M, Np, world, AMP_DTYPE_BF16);
        CK(cudaMalloc(&ws, wsb));
        if (fp8) {
            AK(amp_gemm_fp8e4m3_sharded_dev(comm, (const uint8_t*)A, (const uint8_t*)Bslab,
                                            (const float*)sa, (const float*)sb, 2, C,
                                            AMP_DTYPE_BF16, M, Np, K, ws, wsb, st));
            AK(amp_gemm_fp8e4m3_dev((const uint8_t*)A, (const uint8_t*)Bfull, (const float*)sa,
                                    (const float*)sb_full, 2, C_ref, AMP_DTYPE_BF16, M, N, K, st));
        } else {
            AK(amp_gemm_bf16_sharded_dev(comm, A, Bslab, C, AMP_DTYPE_BF16, M, Np, K, ws, wsb, st));
            AK(amp_gemm_bf16_dev(A, Bfull, C_ref, AMP_DTYPE_BF16, M, N, K, st));
        }
        CK(cudaStreamSynchronize(st));
        bytes = (size_t)M * N * 2;
        if (compare(C, C_ref, bytes, rank, &diff)) return 1;
    }
    // one collective more: every rank's mismatch count, all-reduced (MAX) as fp32
    float* dflag;
    CK(cudaMalloc(&dflag, sizeof(float)));
    float h = (float)diff;
    CK(cudaMemcpy(dflag, &h, sizeof h, cudaMemcpyHostToDevice));
    AK(amp_comm_allreduce_max_f32(comm, dflag, 1, st));
    AK(amp_comm_barrier(comm, st));
    CK(cudaStreamSynchronize(st));
    CK(cudaMemcpy(&h, dflag, sizeof h, cudaMemcpyDeviceToHost));
    AK(amp_device_status(0));
    AK(amp_comm_destroy(comm));
    std::printf("{\"rank\": %d, \"world\": %d, \"op\": \"%s\", \"bytes\": %zu, "
                "\"mismatched_bytes\": %zu, \"max_over_ranks\": %.0f}\n",
                rank, world, op.c_str(), bytes, diff, h);
    std::fflush(stdout);
    return (diff == 0 && h == 0.f) ? 0 : 2;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) {
        std::fprintf(stderr, "usage: %s <world> [M N K] [--op bf16|fp8|attn|attn_gqa]\n", argv[0]);
        return 2;
    }
    const int world = std::atoi(argv[1]);
    int M = 1024, N = 2048, K = 512;
    std::string op = "bf16";
    std::vector<std::string> pos;
    for (int i = 2; i < argc; ++i) {
        if (std::string(argv[i]) == "--op" && i + 1 < argc)
            op = argv[++i];
        else
            pos.push_back(argv[i]);
    }
    if (pos.size() >= 3) {
        M = std::atoi(pos[0].c_str());
        N = std::atoi(pos[1].c_str());
        K = std::atoi(pos[2].c_str());
    }
    if (world < 1 || world > 64 || M <= 0 || N <= 0 || K <= 0 || N % world ||
        (op != "bf16" && op != "fp8" && op != "attn" && op != "attn_gqa")) {
        std::fprintf(stderr, "bad arguments\n");
        return 2;
    }
    std::vector<int> rd(world, -1), wr(world, -1);
    for (int r = 1; r < world; ++r) {
        int fds[2];
        if (pipe(fds) != 0) return 1;
        rd[r] = fds[0];
        wr[r] = fds[1];
    }
    std::vector<pid_t> kids;
    for (int r = 0; r < world; ++r) {
        pid_t pid = fork();
        if (pid < 0) return 1;
        if (pid == 0) {
            std::vector<int> outs;
            if (r == 0)
                for (int q = 1; q < world; ++q) outs.push_back(wr[q]);
            _exit(run_rank(r, world, M, N, K, op, rd[r], outs));
        }
        kids.push_back(pid);
    }
    int rc = 0;
    for (pid_t pid : kids) {
        int status = 0;
        waitpid(pid, &status, 0);
        if (!WIFEXITED(status) || WEXITSTATUS(status) != 0) rc = 1;
    }
    return rc;
}
