// ref_amp_gemm_shim.cpp -- TEST INFRASTRUCTURE ONLY (the CPU baseline / checker).
//
// Compiles AMP's plugin validator source (tests/amp_validate_kernel.cpp of the
// reference tree, included in place, never copied) so that its CPU reference
// GEMM -- a file-local helper there -- can be called and timed directly.
// Every header that file uses is included first; `static` is then defined
// away for the included file only, and its main() is renamed.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <dlfcn.h>
#include <fstream>
#include <string>
#include <thread>
#include <vector>

#include "amp_plugin.h"

#define static
#define main amp_validate_kernel_main
#include "amp_validate_kernel.cpp"
#undef main
#undef static

extern "C" {

// AMP's cpu_reference_gemm on raw row-major buffers (A MxK, B KxN, C MxN).
__attribute__((visibility("default"))) void ref_cpu_reference_gemm(const float* A,
                                                                   const float* B, float* C,
                                                                   int M, int N, int K) {
    std::vector<float> a(A, A + (size_t)M * K), b(B, B + (size_t)K * N), c((size_t)M * N);
    cpu_reference_gemm(a, b, c, M, N, K);
    std::memcpy(C, c.data(), c.size() * sizeof(float));
}

// The same function run on `threads` host threads, each over a slice of A's rows.
__attribute__((visibility("default"))) void ref_cpu_reference_gemm_mt(const float* A,
                                                                      const float* B, float* C,
                                                                      int M, int N, int K,
                                                                      int threads) {
    if (threads < 1) threads = 1;
    const std::vector<float> b(B, B + (size_t)K * N);
    std::vector<std::thread> ts;
    const int chunk = (M + threads - 1) / threads;
    for (int t = 0; t < threads; ++t) {
        const int r0 = t * chunk, r1 = std::min(M, r0 + chunk);
        if (r0 >= r1) break;
        ts.emplace_back([&, r0, r1] {
            const int m = r1 - r0;
            std::vector<float> a(A + (size_t)r0 * K, A + (size_t)r1 * K), c((size_t)m * N);
            cpu_reference_gemm(a, b, c, m, N, K);
            std::memcpy(C + (size_t)r0 * N, c.data(), c.size() * sizeof(float));
        });
    }
    for (auto& t : ts) t.join();
}

}  // extern "C"
