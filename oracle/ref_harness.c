/*
 * ref_harness.c -- exposes the reference's own hot-path functions.
 *
 * TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together
 * with the reference's gemma.c, included from where it lies (path given as
 * GEMMA_REF_SOURCE), with the reference Makefile's flags
 * (-O3 -ffast-math -march=... -fopenmp, DTYPE unset = FP32).  The result,
 * oracle/_ref/libgemma_ref_*.so, is used to pin the C restatement in
 * gemma_oracle.c and as the timed CPU baseline ("kind": "reference").
 *
 * gemma.c's functions are `static`, so they are wrapped here in the same
 * translation unit.  `main` is renamed before the include, and the one-letter
 * macros that the embedded stb blob leaks (gemma.c:7494 onwards) are
 * #undef'd by the generated header undef_blob.h before any code of ours.
 */
#define main gemma_ref_main
#include GEMMA_REF_SOURCE
#undef main
#include "undef_blob.h"

/* gemma.c:2590 */
float ref_quantize_act(int8_t *dst, const float *vec, int dim) {
  return quantize_act(dst, vec, dim, NULL);
}

/* gemma.c:2656; threads > 1 takes the OpenMP branch like the call sites
 * (gemma.c:4497, 5034) do with omp = true. */
void ref_quantize_acts(int8_t *dst, float *dsc, const float *src, int sstr,
                       int m, int n, int threads) {
  quantize_acts(dst, dsc, src, sstr, m, n, threads > 1, threads, NULL);
}

/* gemma.c:2770 */
void ref_gemv_int8(float *dst, const int8_t *mat, const float *matsc,
                   const int8_t *vec, float vsc, int m, int n, int threads) {
  gemv_int8(dst, mat, matsc, vec, vsc, m, n, threads > 1, threads, NULL);
}

/* gemma.c:2818; `jobs` points at GemvJob records (gemma.c:2795). */
void ref_gemv_int8_multi(const void *jobs, int njobs, const int8_t *vec,
                         float vsc, int n, int threads) {
  gemv_int8_multi((const GemvJob *)jobs, njobs, vec, vsc, n, threads, NULL);
}

/* gemma.c:3943 */
int ref_gemm_int8(float *dst, int dstr, const int8_t *mat, int mstr,
                  const float *matsc, const int8_t *src, int sstr,
                  const float *ssc, int m, int n, int k, int threads) {
  return gemm_int8(dst, dstr, mat, mstr, matsc, src, sstr, ssc, m, n, k,
                   threads > 1, threads, NULL);
}

/* gemma.c:2509: gemma-style RMSNorm of one row (dst may equal src). */
void ref_rmsnorm(float *dst, const float *src, const float *weight, int dim, float eps) {
  rmsnorm(dst, src, weight, dim, eps, NULL);
}

/* gemma.c:4150: dst[i] = gelu_tanh(src[i] + bias) * mul[i] over rows x dim,
 * here without bias and with `mul` (the GeGLU gate * up of 4921, 5379). */
void ref_gelu_mul(float *dst, const float *src, const float *mul, int rows, int dim) {
  gelu(dst, src, rows, dim, NULL, mul, false, 1, NULL);
}

/* gemma.c:484: GEMM_MC / GEMM_NC / GEMM_KC tile sizes from the environment. */
void ref_setup(void) { setup_runtime_config(); }

/* gemma.c:4056: frees the calling thread's GEMM scratch. */
void ref_free_thread_scratch(void) { gemm_free_thread_scratch(); }

/* sizeof(GemvJob), so callers can check their record layout. */
int ref_gemv_job_size(void) { return (int)sizeof(GemvJob); }

/* which int8 micro-kernel this build selected (gemma.c:537-545). */
const char *ref_isa(void) {
#if defined(GEMMA_GEMM_VNNI8)
  return "avx-vnni-int8";
#elif defined(GEMMA_GEMM_AVX2)
  return "avx2";
#else
  return "portable";
#endif
}
