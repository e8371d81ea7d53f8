/*
 * gemma_gcu.h -- drop-in CUDA versions of gemma.c's W8A8 hot-path functions.
 *
 * Included by gemma.c in place of its own definitions (see the integration
 * notes): every function keeps the reference's exact static signature,
 * argument meaning, PerfBench accounting and error convention, and forwards
 * to libgcu.so's C ABI (include/gcu.h).  The including translation unit
 * provides what gemma.c provides there: floatx (FP32 only), PerfBench with
 * PERF_TIC / PERF_TOC and the PERF_OP_* ids (gemma.c:2402-2497), GemvJob
 * (gemma.c:2795) and log_error (gemma.c:579).
 *
 *   quantize_act     gemma.c:2590      -> gcu_quantize_act
 *   quantize_acts    gemma.c:2656      -> gcu_quantize_acts
 *   gemv_int8        gemma.c:2770      -> gcu_gemv_int8
 *   gemv_int8_multi  gemma.c:2818      -> gcu_gemv_int8_multi
 *   gemm_int8        gemma.c:3943      -> gcu_gemm_int8
 *
 * The `omp` / `threads` arguments select OpenMP teams in the reference; the
 * GPU needs neither, so they are accepted and ignored.  All five may be
 * called concurrently from OpenMP worker threads (gemma.c:5045-5091):
 * libgcu.so gives each host thread its own stream and staging buffers.
 *
 * Errors: gemm_int8 returns 1 and sets the thread's error text through
 * log_error, exactly as the reference does when its scratch allocation fails
 * (gemma.c:3977-3982).  The other four cannot report an error in the
 * reference's signatures; they log it, raise the thread-local flag read by
 * gcu_shim_failed(), and leave their outputs as the CUDA call left them.
 */
#ifndef GEMMA_GCU_H
#define GEMMA_GCU_H

#include "gcu.h"

#if defined(DTYPE) && defined(FP32) && DTYPE != FP32
#error "the CUDA hot path computes in fp32: build gemma.c with DTYPE=FP32"
#endif

static _Thread_local int g_gcu_failed = 0;

/* 1 if a void hot-path call of this thread failed since the last check. */
static int gcu_shim_failed(void) {
  int f = g_gcu_failed;
  g_gcu_failed = 0;
  return f;
}

static void gcu_shim_fail(void) {
  log_error("cuda: %s", gcu_last_error());
  g_gcu_failed = 1;
}

/* gemma.c:2590 */
static floatx quantize_act(int8_t *dst, const floatx *vec, int dim,
                           PerfBench *perf) {
  double t0 = PERF_TIC(perf);
  float sc = gcu_quantize_act(dst, (const float *)vec, dim);
  if (sc != sc) { /* NaN: the call failed */
    gcu_shim_fail();
    sc = 1.0f;
  }
  PERF_TOC(perf, PERF_OP_QUANTIZE_ACT, t0);
  return (floatx)sc;
}

/* gemma.c:2656 */
static void quantize_acts(int8_t *dst, floatx *dsc, const floatx *src,
                          int sstr, int m, int n, bool omp, int threads,
                          PerfBench *perf) {
  (void)omp;
  (void)threads;
  double t0 = PERF_TIC(perf);
  if (gcu_quantize_acts(dst, (float *)dsc, (const float *)src, sstr, m, n))
    gcu_shim_fail();
  PERF_TOC(perf, PERF_OP_QUANTIZE_ACT, t0);
}

/* gemma.c:2770 (m = rows, n = reduction length) */
static void gemv_int8(floatx *dst, const int8_t *mat, const floatx *matsc,
                      const int8_t *vec, floatx vsc, int m, int n, bool omp,
                      int threads, PerfBench *perf) {
  (void)omp;
  (void)threads;
  double t0 = PERF_TIC(perf);
  if (gcu_gemv_int8((float *)dst, mat, (const float *)matsc, vec, (float)vsc,
                    m, n))
    gcu_shim_fail();
  PERF_TOC(perf, PERF_OP_GEMV_INT8, t0);
}

/* gemma.c:2818; GemvJob (gemma.c:2795) has gcu_gemv_job's layout */
static void gemv_int8_multi(const GemvJob *jobs, int njobs, const int8_t *vec,
                            floatx vsc, int n, int threads, PerfBench *perf) {
  (void)threads;
  double t0 = PERF_TIC(perf);
  _Static_assert(sizeof(GemvJob) == sizeof(gcu_gemv_job),
                 "GemvJob layout differs from gcu_gemv_job");
  if (gcu_gemv_int8_multi((const gcu_gemv_job *)jobs, njobs, vec, (float)vsc,
                          n))
    gcu_shim_fail();
  PERF_TOC(perf, PERF_OP_GEMV_INT8, t0);
}

/* gemma.c:3943 */
static int gemm_int8(floatx *dst, int dstr, const int8_t *mat, int mstr,
                     const floatx *matsc, const int8_t *src, int sstr,
                     const floatx *ssc, int m, int n, int k, bool omp,
                     int threads, PerfBench *perf) {
  (void)omp;
  (void)threads;
  double t0 = PERF_TIC(perf);
  int ret = gcu_gemm_int8((float *)dst, dstr, mat, mstr, (const float *)matsc,
                          src, sstr, (const float *)ssc, m, n, k);
  if (ret) log_error("cuda gemm_int8: %s", gcu_last_error());
  PERF_TOC(perf, PERF_OP_GEMM_INT8, t0);
  return ret;
}

/* The registration hook for setup_gemma_model (gemma.c:6867): upload one
 * QTensor (gemma.c:1102) of `rows` x `k` once.  Returns 0 / 1. */
static int gcu_register_qtensor(const int8_t *q, const floatx *scales,
                                int rows, int k) {
  int rc = gcu_register_weight(q, (const float *)scales, rows, k);
  if (rc) log_error("cuda register: %s", gcu_last_error());
  return rc;
}

#endif /* GEMMA_GCU_H */
