// parity_dump.cpp -- the "A side" dump of AMP's cross-vendor parity flow,
// produced by the B200 kernels.
//
// Mirrors AMP's amp_parity_dump (tests/parity_dump.cpp:109-140 of the
// reference): AMP's harness inputs (srand(seed); (rand()%2000-1000)/100,
// A then B), AMP's CPU reference GEMM for max_rel_err_vs_cpu, one entry per
// tile config with 3 warm-up + 20 timed launches, and the same JSON schema
// (tests/parity_dump.cpp:85-107), so scripts/parity_check.py diffs this dump
// against any other vendor's dump unchanged.
//
//   amp_b200_parity_dump [out.json] [M N K] [--seed S] [--vendor TAG]
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "amp_b200.h"

namespace {

void cpu_gemm_fp32(const std::vector<float>& A, const std::vector<float>& B, std::vector<float>& C,
                   int M, int N, int K) {
    // Same loop order and fp32 accumulator as the reference's CPU GEMM.
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) {
            float acc = 0.0f;
            for (int k = 0; k < K; ++k) acc += A[(size_t)i * K + k] * B[(size_t)k * N + j];
            C[(size_t)i * N + j] = acc;
        }
}

struct Entry {
    int bm, bn, bk;
    double gflops, latency_ms;
    float max_rel_err;
    std::vector<float> out;
};

#define CK(x)                                                                             \
    do {                                                                                  \
        cudaError_t e_ = (x);                                                             \
        if (e_ != cudaSuccess) {                                                          \
            std::fprintf(stderr, "%s: %s\n", #x, cudaGetErrorString(e_));                  \
            std::exit(1);                                                                 \
        }                                                                                 \
    } while (0)

Entry run(int bm, int bn, int bk, int M, int N, int K, const std::vector<float>& A,
          const std::vector<float>& B, const std::vector<float>& ref) {
    float *dA, *dB, *dC;
    CK(cudaMalloc(&dA, std::max<size_t>(4, (size_t)M * K * 4)));
    CK(cudaMalloc(&dB, std::max<size_t>(4, (size_t)K * N * 4)));
    CK(cudaMalloc(&dC, std::max<size_t>(4, (size_t)M * N * 4)));
    CK(cudaMemcpy(dA, A.data(), (size_t)M * K * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dB, B.data(), (size_t)K * N * 4, cudaMemcpyHostToDevice));
    auto launch = [&] {
        if (amp_gemm_fp32_tile_dev(bm, bn, bk, dA, dB, dC, M, N, K, nullptr) != 0) {
            std::fprintf(stderr, "amp_gemm_fp32_tile_dev: %s\n", amp_last_error());
            std::exit(1);
        }
    };
    for (int i = 0; i < 3; ++i) launch();
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    CK(cudaDeviceSynchronize());
    CK(cudaEventRecord(e0));
    for (int i = 0; i < 20; ++i) launch();
    CK(cudaEventRecord(e1));
    CK(cudaEventSynchronize(e1));
    float ms = 0;
    CK(cudaEventElapsedTime(&ms, e0, e1));
    Entry r{bm, bn, bk, 0, ms / 20.0, 0.0f, std::vector<float>((size_t)M * N)};
    r.gflops = 2.0 * M * N * K / (r.latency_ms * 1e6);
    CK(cudaMemcpy(r.out.data(), dC, (size_t)M * N * 4, cudaMemcpyDeviceToHost));
    for (size_t i = 0; i < ref.size(); ++i) {
        float abs_err = std::fabs(r.out[i] - ref[i]);
        r.max_rel_err = std::max(r.max_rel_err, abs_err / std::max(1.0f, std::fabs(ref[i])));
    }
    cudaFree(dA);
    cudaFree(dB);
    cudaFree(dC);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    return r;
}

void write_json(const std::string& path, const std::string& vendor, int M, int N, int K,
                unsigned seed, const std::vector<Entry>& es) {
    std::ofstream f(path);
    f << "{\n  \"vendor\": \"" << vendor << "\",\n";
    f << "  \"M\": " << M << ", \"N\": " << N << ", \"K\": " << K << ", \"seed\": " << seed
      << ",\n  \"tiles\": [\n";
    for (size_t t = 0; t < es.size(); ++t) {
        const Entry& e = es[t];
        f << "    {\"bm\": " << e.bm << ", \"bn\": " << e.bn << ", \"bk\": " << e.bk
          << ", \"gflops\": " << e.gflops << ", \"latency_ms\": " << e.latency_ms
          << ", \"max_rel_err_vs_cpu\": " << e.max_rel_err << ", \"output\": [";
        for (size_t i = 0; i < e.out.size(); ++i) f << (i ? "," : "") << e.out[i];
        f << "]}" << (t + 1 != es.size() ? "," : "") << "\n";
    }
    f << "  ]\n}\n";
}

}  // namespace

int main(int argc, char** argv) {
    std::vector<std::string> pos;
    unsigned seed = 42;
    std::string vendor = "nvidia";
    for (int i = 1; i < argc; ++i) {
        std::string a = argv[i];
        if (a == "--seed" && i + 1 < argc) seed = (unsigned)std::atoi(argv[++i]);
        else if (a == "--vendor" && i + 1 < argc) vendor = argv[++i];
        else pos.push_back(a);
    }
    const std::string out = pos.size() > 0 ? pos[0] : "parity_dump.json";
    const int M = pos.size() > 3 ? std::atoi(pos[1].c_str()) : 96;
    const int N = pos.size() > 3 ? std::atoi(pos[2].c_str()) : 96;
    const int K = pos.size() > 3 ? std::atoi(pos[3].c_str()) : 96;

    std::vector<float> A((size_t)M * K), B((size_t)K * N), ref((size_t)M * N);
    std::srand(seed);
    for (auto& v : A) v = (float)(std::rand() % 2000 - 1000) / 100.0f;
    for (auto& v : B) v = (float)(std::rand() % 2000 - 1000) / 100.0f;
    cpu_gemm_fp32(A, B, ref, M, N, K);

    std::printf("Parity dump (amp_b200, sm_100a) -- vendor=%s M=%d N=%d K=%d seed=%u\n",
                vendor.c_str(), M, N, K, seed);
    const int tiles[4][3] = {{16, 16, 16}, {32, 16, 16}, {32, 32, 16}, {32, 32, 32}};
    std::vector<Entry> es;
    for (auto& t : tiles) {
        es.push_back(run(t[0], t[1], t[2], M, N, K, A, B, ref));
        const Entry& e = es.back();
        std::printf("  tile (%2d,%2d,%2d): %9.1f GFLOPS  %7.4f ms  max_rel_err_vs_cpu=%.6f\n",
                    e.bm, e.bn, e.bk, e.gflops, e.latency_ms, e.max_rel_err);
    }
    write_json(out, vendor, M, N, K, seed, es);
    float worst = 0;
    for (auto& e : es) worst = std::max(worst, e.max_rel_err);
    std::printf("\nWrote %s\n", out.c_str());
    return worst < 1e-3f ? 0 : 1;
}
