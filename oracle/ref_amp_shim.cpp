// ref_amp_shim.cpp -- TEST INFRASTRUCTURE ONLY (the checker / CPU baseline).
//
// Exposes the reference's own FP8 codec (include/fp8.hpp:15-63 of the AMP
// source tree, included in place from the reference checkout, never copied)
// through a C ABI so that tests can pin the oracle against it and bench.py's
// reference arm can time AMP's CPU path on the host cores.
//
// The quantise pipeline around the codec (amax loop, scale = amax/448,
// x/scale, dequantise) is the build's definition of the operation; AMP has
// no amax/quantise routine of its own, only the scalar codec.
#include "fp8.hpp"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {
inline float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)(((u >> 16) & 0x8000u) | 0x7fc0u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

template <class F>
void parallel_for(int64_t n, int threads, F&& body) {
    if (threads <= 1 || n < (1 << 16)) { body(0, n, 0); return; }
    std::vector<std::thread> ts;
    int64_t chunk = (n + threads - 1) / threads;
    for (int t = 0; t < threads; ++t) {
        int64_t lo = t * chunk, hi = std::min<int64_t>(n, lo + chunk);
        if (lo >= hi) break;
        ts.emplace_back([&, lo, hi, t] { body(lo, hi, t); });
    }
    for (auto& t : ts) t.join();
}
}  // namespace

extern "C" {

__attribute__((visibility("default"))) uint8_t ref_f32_to_e4m3(float v) {
    return AMP::fp8::f32_to_e4m3(v);
}

__attribute__((visibility("default"))) float ref_e4m3_to_f32(uint8_t v) {
    return AMP::fp8::e4m3_to_f32(v);
}

__attribute__((visibility("default"))) void ref_f32_to_e4m3_n(const float* x, int64_t n,
                                                              uint8_t* q) {
    for (int64_t i = 0; i < n; ++i) q[i] = AMP::fp8::f32_to_e4m3(x[i]);
}

// Per-tensor amax quantise + dequantise of n bf16 values with AMP's codec,
// split over `threads` host threads.  Returns the scale.
__attribute__((visibility("default"))) float ref_quant_dequant_bf16(const uint16_t* x, int64_t n,
                                                                    uint8_t* q, uint16_t* y,
                                                                    int threads) {
    if (threads < 1) threads = 1;
    std::vector<float> part(threads, 0.0f);
    parallel_for(n, threads, [&](int64_t lo, int64_t hi, int t) {
        float m = 0.0f;
        for (int64_t i = lo; i < hi; ++i) m = std::max(m, std::fabs(bf16_to_f32(x[i])));
        part[t] = m;
    });
    float amax = 0.0f;
    for (float m : part) amax = std::max(amax, m);
    const float scale = amax == 0.0f ? 1.0f : amax / 448.0f;
    const float inv = std::min(1.0f / scale, 3.402823466e38f);
    parallel_for(n, threads, [&](int64_t lo, int64_t hi, int) {
        for (int64_t i = lo; i < hi; ++i) q[i] = AMP::fp8::f32_to_e4m3(bf16_to_f32(x[i]) * inv);
        if (y)
            for (int64_t i = lo; i < hi; ++i)
                y[i] = f32_to_bf16(AMP::fp8::e4m3_to_f32(q[i]) * scale);
    });
    return scale;
}

}  // extern "C"
