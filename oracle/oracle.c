/*
 * oracle.c -- CPU restatement of AMP's hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA kernels
 * in amp_b200/csrc are compared against.  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / reference leg may load liboracle.so; the
 * product path never calls into it and has no CPU fallback.
 *
 * Every function cites the reference file:line whose behaviour it restates
 * (paths relative to the AMP source tree).
 *
 * Pinned against: the reference's own FP8 codec (include/fp8.hpp) compiled
 * from its sources into oracle/_ref (amp-compat mode must agree on every
 * float32 bit pattern class probed), torch's float8_e4m3fn (RNE mode), and
 * the verify_fixes.cpp:29-46 probes; see tests/test_oracle_*.py.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stddef.h>

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------- */
/* bf16 <-> fp32                                                              */
/* ------------------------------------------------------------------------- */

static inline float u32_as_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f32_as_u32(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

ORC_API float orc_bf16_to_f32(uint16_t h) { return u32_as_f32((uint32_t)h << 16); }

/* Round-to-nearest-even fp32 -> bf16; NaN maps to the quiet NaN 0x7FC0 (sign kept). */
ORC_API uint16_t orc_f32_to_bf16(float f) {
    uint32_t u = f32_as_u32(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)(((u >> 16) & 0x8000u) | 0x7fc0u);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

/* ------------------------------------------------------------------------- */
/* FP8 E4M3 (OCP "fn" flavour: bias 7, no inf, S.1111.111 is NaN, max 448)    */
/* ------------------------------------------------------------------------- */

/* Decode one E4M3 code.  Follows the format definition used by
 * include/fp8.hpp:15-32 (e4m3_to_f32): E==0 subnormal m/8*2^-6, E==15&&M==7
 * NaN, otherwise (1+m/8)*2^(E-7).  Code 0x80 decodes to -0.0. */
ORC_API float orc_e4m3_to_f32(uint8_t v) {
    int s = v >> 7, e = (v >> 3) & 15, m = v & 7;
    float r;
    if (e == 15 && m == 7) r = NAN;
    else if (e == 0) r = ldexpf((float)m, -9);
    else r = ldexpf((float)(8 + m), e - 10);
    return s ? -r : r;
}

/* Encode fp32 -> E4M3 with round-to-nearest-even and saturation to +-448.
 * This is the semantics the quantiser is specified with (RNE, saturating).
 * The reference codec include/fp8.hpp:34-63 saturates the same way but
 * rounds ties away from zero and clamps the subnormal mantissa at 7; the
 * amp-compat encoder below restates that behaviour for comparison.
 *   NaN            -> 0x7F (sign dropped)
 *   |x| >= 448     -> S|0x7E  (inf included; 448 < |x| < 464 rounds to 448
 *                   under RNE, larger values saturate)
 *   otherwise      -> nearest representable, ties to even mantissa        */
ORC_API uint8_t orc_f32_to_e4m3_rne(float x) {
    uint32_t u = f32_as_u32(x);
    uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7F;
    float a = fabsf(x);
    if (a >= 448.0f) return sign | 0x7E;
    if (a == 0.0f) return sign;
    int e2;
    frexpf(a, &e2);            /* a = f * 2^e2, f in [0.5,1) -> a in [2^(e2-1), 2^e2) */
    int unb = e2 - 1;
    if (unb < -6) unb = -6;    /* below the min normal the spacing stays 2^-9 */
    float quantum = ldexpf(1.0f, unb - 3);
    float q = a / quantum;     /* exact: power-of-two scaling of a normal float */
    float r = rintf(q);        /* default rounding mode: nearest, ties to even */
    uint32_t val = (uint32_t)r;
    if (unb == -6 && val < 8) return sign | (uint8_t)val;   /* subnormal or zero */
    int E = unb + 7;
    if (val == 16) { val = 8; E += 1; }
    return sign | (uint8_t)(E << 3) | (uint8_t)(val - 8);
}

/* Restatement of the reference encoder include/fp8.hpp:34-63 (f32_to_e4m3):
 * clamp to 448, frexp, subnormal mantissa round-half-away then clamp to 7,
 * normal mantissa round-half-away with carry into the exponent, E=15,M=7
 * mapped to 0x7E.  Kept only to compare against the reference codec. */
ORC_API uint8_t orc_f32_to_e4m3_ampcompat(float v) {
    if (isnan(v)) return 0x7F;
    uint8_t sign = (v < 0.0f) ? 0x80 : 0;
    v = fabsf(v);
    if (v > 448.0f) v = 448.0f;
    if (v == 0.0f) return sign;
    int ex;
    float frac = frexpf(v, &ex);
    int biased = ex - 1 + 7;
    if (biased <= 0) {
        float mr = roundf(v * 512.0f);
        uint8_t mant = (uint8_t)mr;
        if (mant > 7) mant = 7;
        return sign | mant;
    }
    uint8_t e = (uint8_t)(biased > 15 ? 15 : biased);
    float nm = frac * 2.0f - 1.0f;
    uint8_t m = (uint8_t)roundf(nm * 8.0f);
    if (m >= 8) { m = 0; e++; }
    if (e > 15 || (e == 15 && m >= 7)) return sign | 0x7E;
    return sign | (uint8_t)(e << 3) | m;
}

ORC_API void orc_f32_to_e4m3_rne_n(const float* x, int64_t n, uint8_t* q) {
    for (int64_t i = 0; i < n; ++i) q[i] = orc_f32_to_e4m3_rne(x[i]);
}

ORC_API void orc_f32_to_e4m3_ampcompat_n(const float* x, int64_t n, uint8_t* q) {
    for (int64_t i = 0; i < n; ++i) q[i] = orc_f32_to_e4m3_ampcompat(x[i]);
}

/* ------------------------------------------------------------------------- */
/* amax-scaled quantise / dequantise                                          */
/* The reference has no amax or device quantiser (only the host codec in     */
/* include/fp8.hpp and cuBLASLt's AMAX_D_POINTER plumbing at                  */
/* src/gemm_vendor.cpp:186-187); the pipeline semantics are:                  */
/*   amax  = max |x| over the bf16 inputs widened to fp32 (NaN ignored)       */
/*   scale = amax / 448 (IEEE fp32 division); amax == 0 -> scale = 1          */
/*   inv   = min(1 / scale, FLT_MAX)  (IEEE fp32 division, clamped so that    */
/*           0 * inv stays 0 when scale is tiny)                              */
/*   q     = E4M3_RNE_sat(x * inv)    (IEEE fp32 multiply)                    */
/*   y     = bf16_RNE(e4m3_to_f32(q) * scale)                                 */
/* ------------------------------------------------------------------------- */

ORC_API float orc_amax_bf16(const uint16_t* x, int64_t n) {
    float m = 0.0f;
    for (int64_t i = 0; i < n; ++i) {
        float a = fabsf(orc_bf16_to_f32(x[i]));
        if (a > m) m = a;      /* NaN compares false: ignored */
    }
    return m;
}

ORC_API float orc_scale_from_amax(float amax) {
    return amax == 0.0f ? 1.0f : amax / 448.0f;
}

#include <float.h>
ORC_API float orc_inv_scale(float scale) {
    /* The reciprocal is taken of a volatile copy: inlined into a caller, GCC's
       value-range propagation would conclude from "1/scale is infinite" that
       scale == 0 and rewrite the caller's scale, which is wrong for a subnormal
       scale (a tiny amax), whose reciprocal overflows. */
    const volatile float s = scale;
    float inv = 1.0f / s;
    return inv > FLT_MAX ? FLT_MAX : inv;   /* NaN stays NaN */
}

static inline uint8_t quant1(uint16_t xb, float inv) {
    return orc_f32_to_e4m3_rne(orc_bf16_to_f32(xb) * inv);   /* one rounded multiply */
}

/* Per-tensor quantise; returns the scale through *scale_out. */
ORC_API void orc_quant_e4m3(const uint16_t* x, int64_t n, uint8_t* q, float* scale_out,
                            float* amax_out) {
    float amax = orc_amax_bf16(x, n);
    float s = orc_scale_from_amax(amax), inv = orc_inv_scale(s);
    for (int64_t i = 0; i < n; ++i) q[i] = quant1(x[i], inv);
    if (scale_out) *scale_out = s;
    if (amax_out) *amax_out = amax;
}

/* Quantise with a given amax (the sharded path: global amax comes from an all-reduce). */
ORC_API void orc_quant_e4m3_with_amax(const uint16_t* x, int64_t n, float amax, uint8_t* q) {
    float inv = orc_inv_scale(orc_scale_from_amax(amax));
    for (int64_t i = 0; i < n; ++i) q[i] = quant1(x[i], inv);
}

ORC_API void orc_dequant_e4m3(const uint8_t* q, int64_t n, float scale, uint16_t* y) {
    for (int64_t i = 0; i < n; ++i) y[i] = orc_f32_to_bf16(orc_e4m3_to_f32(q[i]) * scale);
}

/* Per-row quantise of a row-major rows x cols bf16 matrix: one scale per row. */
ORC_API void orc_quant_e4m3_rows(const uint16_t* x, int64_t rows, int64_t cols, uint8_t* q,
                                 float* scales) {
    for (int64_t r = 0; r < rows; ++r) {
        const uint16_t* xr = x + r * cols;
        float s = orc_scale_from_amax(orc_amax_bf16(xr, cols)), inv = orc_inv_scale(s);
        for (int64_t c = 0; c < cols; ++c) q[r * cols + c] = quant1(xr[c], inv);
        scales[r] = s;
    }
}

/* Per-column quantise of a row-major rows x cols bf16 matrix: one scale per column. */
ORC_API void orc_quant_e4m3_cols(const uint16_t* x, int64_t rows, int64_t cols, uint8_t* q,
                                 float* scales) {
    for (int64_t c = 0; c < cols; ++c) {
        float m = 0.0f;
        for (int64_t r = 0; r < rows; ++r) {
            float a = fabsf(orc_bf16_to_f32(x[r * cols + c]));
            if (a > m) m = a;
        }
        scales[c] = orc_scale_from_amax(m);
    }
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < cols; ++c)
            q[r * cols + c] = quant1(x[r * cols + c], orc_inv_scale(scales[c]));
}

/* ------------------------------------------------------------------------- */
/* GEMM                                                                       */
/* ------------------------------------------------------------------------- */

/* AMP's CPU reference, tests/amp_validate_kernel.cpp:20-28 (identical copies
 * in tests/parity_dump.cpp:26-34 and tests/verify_matmul_correctness.cpp:18-26):
 * row-major, i-j-k order, fp32 accumulator, single thread. */
ORC_API void orc_gemm_fp32_amp(const float* A, const float* B, float* C, int M, int N, int K) {
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) {
            float acc = 0.0f;
            for (int k = 0; k < K; ++k) acc += A[(int64_t)i * K + k] * B[(int64_t)k * N + j];
            C[(int64_t)i * N + j] = acc;
        }
}

/* Same contraction with an fp64 accumulator (i-k-j order for cache reuse);
 * the tolerance reference for every GEMM parity test. */
ORC_API void orc_gemm_f64(const float* A, const float* B, double* C, int M, int N, int K) {
    for (int i = 0; i < M; ++i) {
        double* c = C + (int64_t)i * N;
        for (int j = 0; j < N; ++j) c[j] = 0.0;
        for (int k = 0; k < K; ++k) {
            double a = A[(int64_t)i * K + k];
            const float* b = B + (int64_t)k * N;
            for (int j = 0; j < N; ++j) c[j] += a * (double)b[j];
        }
    }
}

/* glibc rand() sequence used by AMP's harness inputs:
 * srand(seed); v = (rand() % 2000 - 1000) / 100 (tests/amp_validate_kernel.cpp:84-86).
 * Filling A then B from one call reproduces the harness exactly. */
#include <stdlib.h>
ORC_API void orc_amp_harness_fill(unsigned seed, float* A, int64_t na, float* B, int64_t nb) {
    srand(seed);
    for (int64_t i = 0; i < na; ++i) A[i] = (float)(rand() % 2000 - 1000) / 100.0f;
    for (int64_t i = 0; i < nb; ++i) B[i] = (float)(rand() % 2000 - 1000) / 100.0f;
}
