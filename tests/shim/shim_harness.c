/*
 * shim_harness.c -- compiles gemma.c_b200/host/gemma_gcu.h the way gemma.c
 * would include it, against minimal stand-ins for the gemma.c context it
 * needs (floatx, PerfBench + PERF_TIC/PERF_TOC, GemvJob, log_error; see
 * gemma.c:497-535, 577-587, 2402-2497, 2795), and exports the five shim
 * functions so tests can call them.  Test infrastructure only.
 */
#include <stdarg.h>
#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#include <time.h>

#define FP32 3
#define DTYPE FP32
typedef float floatx;

typedef enum {
  PERF_OP_QUANTIZE_ACT,
  PERF_OP_GEMV_INT8,
  PERF_OP_GEMM_INT8,
  PERF_OP_COUNT
} PerfOp;
typedef struct {
  double sec[PERF_OP_COUNT];
  long cnt[PERF_OP_COUNT];
} PerfBench;

static double now_sec(void) {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}
#define PERF_TIC(perf) ((perf) != NULL ? now_sec() : 0.0)
#define PERF_TOC(perf, o, t0)                                                  \
  do {                                                                         \
    if ((perf) != NULL) {                                                      \
      (perf)->sec[o] += now_sec() - (t0);                                      \
      (perf)->cnt[o]++;                                                        \
    }                                                                          \
  } while (0)

static _Thread_local char g_err[128];
static int log_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  int r = vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return r;
}

typedef struct {
  const void *w;
  const floatx *sc;
  floatx *dst;
  int m;
} GemvJob;

#include "gemma_gcu.h"

static PerfBench g_perf;

float shim_quantize_act(int8_t *dst, const float *vec, int dim) {
  return quantize_act(dst, vec, dim, &g_perf);
}
void shim_quantize_acts(int8_t *dst, float *dsc, const float *src, int sstr,
                        int m, int n) {
  quantize_acts(dst, dsc, src, sstr, m, n, true, 8, &g_perf);
}
void shim_gemv_int8(float *dst, const int8_t *mat, const float *matsc,
                    const int8_t *vec, float vsc, int m, int n) {
  gemv_int8(dst, mat, matsc, vec, vsc, m, n, true, 8, &g_perf);
}
void shim_gemv_int8_multi(const GemvJob *jobs, int njobs, const int8_t *vec,
                          float vsc, int n) {
  gemv_int8_multi(jobs, njobs, vec, vsc, n, 8, &g_perf);
}
int shim_gemm_int8(float *dst, int dstr, const int8_t *mat, int mstr,
                   const float *matsc, const int8_t *src, int sstr,
                   const float *ssc, int m, int n, int k) {
  return gemm_int8(dst, dstr, mat, mstr, matsc, src, sstr, ssc, m, n, k, false,
                   1, &g_perf);
}
int shim_register(const int8_t *q, const float *s, int rows, int k) {
  return gcu_register_qtensor(q, s, rows, k);
}
int shim_failed(void) { return gcu_shim_failed(); }
const char *shim_error(void) { return g_err; }
long shim_perf_count(int op) { return g_perf.cnt[op]; }
