/* amp_plugin.h -- AMP's user-kernel plugin contract, implemented by libamp_b200.so.
 *
 * This is the ABI AMP's validator binds (reference include/amp_plugin.h:44-49,
 * loaded by tests/amp_validate_kernel.cpp:67-81 via dlopen + dlsym).  The
 * name, signature and meaning are AMP's; the implementation behind it is the
 * sm_100a GEMM in amp_b200/csrc/gemm_fp32.cu.
 *
 *   A, B, C  HOST (CPU) buffers, row-major: A is M x K, B is K x N, C is M x N,
 *            C[i*N + j] = sum_k A[i*K + k] * B[k*N + j], fp32.
 *   The callee does all device work (staging, copies, launch, synchronise)
 *   before returning; the caller times wall clock around the call.
 *   Returns 0 on success; nonzero is a hard failure (the validator stops),
 *   numerical agreement is judged separately against a CPU reference.
 */
#ifndef AMP_PLUGIN_H
#define AMP_PLUGIN_H

#ifdef __cplusplus
extern "C" {
#endif

typedef int (*amp_user_gemm_fp32_fn)(const float* A, const float* B, float* C, int M, int N,
                                     int K);

/* The exact symbol name the validator resolves with dlsym(). */
#define AMP_PLUGIN_GEMM_FP32_SYMBOL "amp_user_gemm_fp32"

#if defined(__GNUC__)
__attribute__((visibility("default")))
#endif
int amp_user_gemm_fp32(const float* A, const float* B, float* C, int M, int N, int K);

#ifdef __cplusplus
}
#endif

#endif /* AMP_PLUGIN_H */
