// k_producers.cu -- the producers of the matmul inputs, fused with K1.
//
// gemma.c quantizes two kinds of activation right after computing them:
//   - every block input right after its RMSNorm: rmsnorm (gemma.c:2509-2524)
//     at 4754 / 5026, then quantize_act / quantize_acts at 4768 / 5034;
//   - the down projection's input right after the GeGLU gate: gelu with
//     `mul` (gemma.c:4139-4170) at 4921 / 5379, then quantize at 4927 / 5389.
// Each kernel here computes the producer on a row held in registers and
// quantizes the result in the same pass, so the fp32 activation is read once
// and the int8 codes (plus, optionally, the fp32 values) written once.
//
//   rmsnorm:  sq = sum x^2, rms = 1 / sqrt(sq / n + eps), xn = (x*rms)*(w+1)
//   geglu:    h = (0.5*x) * (1 + tanh(c*(x + ((0.044715*x)*x)*x))) * up,
//             c = sqrt(2/pi), tanhf is CUDA's
// The quantize step is K1's exact arithmetic on those values.  The sum of
// squares is reduced in a different order than gemma.c's vectorized loop
// and tanhf is a different library's, so the fp32 values match the
// reference to within ~1e-6 relative, not bit for bit; a code can then
// differ by one where a value sits that close to a rounding boundary.
//
// HBM-bound: one read of the input row(s) (and the norm weight, from L2),
// one int8 write (plus the optional fp32 write).  Same work split as K1's
// warp path: WPR warps per row, 8/WPR rows per 256-thread CTA.
#include "gcu_internal.cuh"
#include "producers.cuh"

#include <algorithm>

#define GCU_EXPORT extern "C" __attribute__((visibility("default")))

namespace gcu {
namespace {

// GEGLU_AMAX and QUANT_GIVEN split GEGLU in two for a hidden dimension
// sharded over ranks: the first writes h and each row's local |max| (in place
// of the scale), the second quantizes h with the row maxima all ranks agreed
// on (b = amax per row), so every rank forms the codes of the unsharded row.
enum Producer { RMSNORM = 0, GEGLU = 1, GEGLU_AMAX = 2, QUANT_GIVEN = 3 };

using prod::row_reduce;

// a: the row source (x, or the gate), b: the norm weight [n] (RMSNORM) or the
// up rows (GEGLU, same stride as a); out: optional fp32 result rows [m][n].
template <int VPT, int WPR, Producer P>
__global__ void __launch_bounds__(256) k_producer_quant(int8_t *__restrict__ dst, float *__restrict__ dsc,
                                                        float *__restrict__ out, const float *__restrict__ a,
                                                        const float *__restrict__ b, float eps, long astr,
                                                        int m, int n) {
  constexpr int kRows = 8 / WPR;
  __shared__ float red[8];
  ptx::griddep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = warp / WPR, wi = warp - grp * WPR;
  const int row = blockIdx.x * kRows + grp;
  const bool live = row < m;  // uniform per warp
  const int n4 = n >> 2;
  ptx::griddep_wait();
  float4 v[VPT];
  if (live) {
    const float4 *ar = reinterpret_cast<const float4 *>(a + (size_t)row * astr);
    const float4 *br = reinterpret_cast<const float4 *>(P == GEGLU || P == GEGLU_AMAX ? b + (size_t)row * astr : b);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = (i * WPR + wi) * 32 + lane;
      if (idx < n4) {
        v[i] = __ldcs(ar + idx);
        if (P == GEGLU || P == GEGLU_AMAX) {
          const float4 u = __ldcs(br + idx);
          v[i] = prod::geglu4(v[i], u);
        }
      }
    }
  }
  if (P == RMSNORM) {
    float sq = 0.0f;
    if (live) {
#pragma unroll
      for (int i = 0; i < VPT; ++i)
        if ((i * WPR + wi) * 32 + lane < n4)
          sq += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
    sq = row_reduce<WPR, false>(sq, red, warp, grp, lane);
    const float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sq, (float)n), eps)));
    if (live) {
      const float4 *wr = reinterpret_cast<const float4 *>(b);
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int idx = (i * WPR + wi) * 32 + lane;
        if (idx < n4) {
          const float4 w = __ldg(wr + idx);
          v[i] = make_float4(__fmul_rn(__fmul_rn(v[i].x, rms), __fadd_rn(w.x, 1.0f)),
                             __fmul_rn(__fmul_rn(v[i].y, rms), __fadd_rn(w.y, 1.0f)),
                             __fmul_rn(__fmul_rn(v[i].z, rms), __fadd_rn(w.z, 1.0f)),
                             __fmul_rn(__fmul_rn(v[i].w, rms), __fadd_rn(w.w, 1.0f)));
        }
      }
    }
  }
  float amax = 0.0f;
  if (P == QUANT_GIVEN) {
    if (live) amax = __ldg(b + row);  // the row's max over every rank's slice
  } else {
    if (live) {
#pragma unroll
      for (int i = 0; i < VPT; ++i)
        if ((i * WPR + wi) * 32 + lane < n4) amax = ptx::absmax4(v[i], amax);
    }
    amax = row_reduce<WPR, true>(amax, red, warp, grp, lane);
  }
  if (!live) return;
  if (P == GEGLU_AMAX) {
    float4 *o = reinterpret_cast<float4 *>(out + (size_t)row * n);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = (i * WPR + wi) * 32 + lane;
      if (idx < n4) o[idx] = v[i];
    }
    if (wi == 0 && lane == 0) dsc[row] = amax;
    return;
  }
  float scale, inv;
  ptx::quant_scale(amax, scale, inv);
  int *q = reinterpret_cast<int *>(dst + (size_t)row * n);
  float4 *o = out ? reinterpret_cast<float4 *>(out + (size_t)row * n) : nullptr;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = (i * WPR + wi) * 32 + lane;
    if (idx < n4) {
      q[idx] = ptx::quant_pack4(v[i], inv);
      if (o) o[idx] = v[i];
    }
  }
  if (wi == 0 && lane == 0) dsc[row] = scale;
}

template <Producer P, int WPR>
cudaError_t launch_wpr(int vpt, int grid, int8_t *dst, float *dsc, float *out, const float *a,
                       const float *b, float eps, long astr, int m, int n, cudaStream_t st) {
  switch (vpt) {
    case 2: return launch_k(k_producer_quant<2, WPR, P>, grid, 256, 0, st, dst, dsc, out, a, b, eps, astr, m, n);
    case 4: return launch_k(k_producer_quant<4, WPR, P>, grid, 256, 0, st, dst, dsc, out, a, b, eps, astr, m, n);
    case 8: return launch_k(k_producer_quant<8, WPR, P>, grid, 256, 0, st, dst, dsc, out, a, b, eps, astr, m, n);
    default: return launch_k(k_producer_quant<16, WPR, P>, grid, 256, 0, st, dst, dsc, out, a, b, eps, astr, m, n);
  }
}

template <Producer P>
int launch_producer(int8_t *dst, float *dsc, float *out, const float *a, const float *b, float eps,
                    long astr, int m, int n, cudaStream_t st, const char *what) {
  if (m <= 0) return 0;
  if (n <= 0 || n % 4 || n > 16384)
    return set_error("%s: row length %d must be a positive multiple of 4 up to 16384", what, n);
  if (astr < n || astr % 4) return set_error("%s: row stride %ld must be >= %d and a multiple of 4", what, astr, n);
  if ((P != GEGLU_AMAX && !dst) || !dsc || !a || !b || (P == GEGLU_AMAX && !out))
    return set_error("%s: null pointer", what);
  if ((uintptr_t)a % 16 || (uintptr_t)b % 16 || (uintptr_t)dst % 4 || (out && (uintptr_t)out % 16))
    return set_error("%s: rows must be 16-byte aligned (codes 4-byte)", what);
  const int n4 = n / 4;
  // the quantize kernel's split: fewest warps per row holding 8 float4 per
  // lane (16 past 8192 elements), more while the grid is small
  int wpr = 1;
  while (wpr < 8 && n4 > 32 * 8 * wpr) wpr *= 2;
  const int sms = num_sms();
  while (wpr < 8 && (long)m * wpr < 16L * sms && n4 >= 32 * 2 * (2 * wpr)) wpr *= 2;
  const int need = (n4 + 32 * wpr - 1) / (32 * wpr);
  const int vpt = need <= 2 ? 2 : need <= 4 ? 4 : need <= 8 ? 8 : 16;
  const long rows_per_cta = 8 / wpr;
  const int grid = (int)((m + rows_per_cta - 1) / rows_per_cta);
  cudaError_t e;
  switch (wpr) {
    case 1: e = launch_wpr<P, 1>(vpt, grid, dst, dsc, out, a, b, eps, astr, m, n, st); break;
    case 2: e = launch_wpr<P, 2>(vpt, grid, dst, dsc, out, a, b, eps, astr, m, n, st); break;
    case 4: e = launch_wpr<P, 4>(vpt, grid, dst, dsc, out, a, b, eps, astr, m, n, st); break;
    default: e = launch_wpr<P, 8>(vpt, grid, dst, dsc, out, a, b, eps, astr, m, n, st); break;
  }
  GCU_CUDA(e);
  GCU_CUDA(cudaGetLastError());
  return 0;
}

}  // namespace
}  // namespace gcu

using namespace gcu;

GCU_EXPORT int gcu_dev_rmsnorm_quantize(int8_t *q, float *s, float *xn, const float *x, int xstr,
                                        const float *weight, float eps, int m, int dim, void *stream) {
  return launch_producer<RMSNORM>(q, s, xn, x, weight, eps, xstr == 0 ? dim : xstr, m, dim,
                                  static_cast<cudaStream_t>(stream), "rmsnorm_quantize");
}

GCU_EXPORT int gcu_dev_geglu_quantize(int8_t *q, float *s, float *h, const float *gate,
                                      const float *up, int m, int dim, void *stream) {
  return launch_producer<GEGLU>(q, s, h, gate, up, 0.0f, dim, m, dim, static_cast<cudaStream_t>(stream),
                                "geglu_quantize");
}

namespace gcu {
// The two halves of gcu_dev_geglu_quantize for a sharded hidden dimension
// (gcu_comm.cu): h = gelu(gate) * up and each row's |max| over this slice;
// then the codes of h given every row's max over all slices.
int launch_geglu_amax(float *h, float *amax, const float *gate, const float *up, int m, int n,
                      cudaStream_t st) {
  return launch_producer<GEGLU_AMAX>(nullptr, amax, h, gate, up, 0.0f, n, m, n, st, "geglu_amax");
}
int launch_quantize_given_amax(int8_t *q, float *s, const float *h, const float *amax, int m, int n,
                               cudaStream_t st) {
  return launch_producer<QUANT_GIVEN>(q, s, nullptr, h, amax, 0.0f, n, m, n, st, "quantize_given_amax");
}
}  // namespace gcu

// ---------------------------------------------------------------------------
// residual stream: x = clamp(resid + rmsnorm(y)), and the logit softcap
// ---------------------------------------------------------------------------
namespace gcu {
namespace {

// gemma.c:4862-4881 (attention) and 4950-4962 (feedforward): the block's
// output y, RMSNorm'd with w when the model has post-norms (NULL: as is),
// added to the residual and clamped to the floatx range.  x may alias resid.
// One CTA of 256 threads per row, float4 columns, NC per thread.
template <int NC>
__global__ void __launch_bounds__(256) k_rmsnorm_residual(float *x, const float *__restrict__ y, const float *resid,
                                                          const float *__restrict__ w, float eps, int dim) {
  __shared__ float red[8];
  ptx::griddep_launch();
  const size_t row = blockIdx.x;
  const int d4 = dim >> 2, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  ptx::griddep_wait();
  float4 v[NC];
  float sq = 0.0f;
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = threadIdx.x + i * 256;
    v[i] = c < d4 ? __ldg(reinterpret_cast<const float4 *>(y + row * dim) + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    sq += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
  }
  float rms = 1.0f;
  if (w) {  // gemma.c:2513-2521
    sq = row_reduce<8, false>(sq, red, warp, 0, lane);
    rms = 1.0f / sqrtf(sq / (float)dim + eps);
  }
  const float m = 3.402823466e38f;  // FLT_MAX: clamp_fpx, gemma.c:2504-2506
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = threadIdx.x + i * 256;
    if (c >= d4) continue;
    float4 a = v[i];
    if (w) {
      const float4 g = __ldg(reinterpret_cast<const float4 *>(w) + c);
      a = make_float4(a.x * rms * (g.x + 1.0f), a.y * rms * (g.y + 1.0f), a.z * rms * (g.z + 1.0f),
                      a.w * rms * (g.w + 1.0f));
    }
    const float4 r = reinterpret_cast<const float4 *>(resid + row * dim)[c];
    reinterpret_cast<float4 *>(x + row * dim)[c] =
        make_float4(fminf(m, fmaxf(-m, a.x + r.x)), fminf(m, fmaxf(-m, a.y + r.y)), fminf(m, fmaxf(-m, a.z + r.z)),
                    fminf(m, fmaxf(-m, a.w + r.w)));
  }
}

// gemma.c:4971-4976: logits = tanh(logits / cap) * cap
__global__ void k_softcap(float *x, long n, float cap) {
  ptx::griddep_launch();
  ptx::griddep_wait();
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    x[i] = tanhf(x[i] / cap) * cap;
}

}  // namespace
}  // namespace gcu

GCU_EXPORT int gcu_dev_rmsnorm_residual(float *x, const float *y, const float *resid, const float *weight, float eps,
                                        int m, int dim, void *stream) {
  if (m <= 0) return 0;
  if (!x || !y || !resid) return set_error("rmsnorm_residual: null pointer");
  if (dim <= 0 || dim % 4 || dim > 4 * 256 * 4)
    return set_error("rmsnorm_residual: row length %d must be a positive multiple of 4 up to 4096", dim);
  if ((uintptr_t)x % 16 || (uintptr_t)y % 16 || (uintptr_t)resid % 16 || (weight && (uintptr_t)weight % 16))
    return set_error("rmsnorm_residual: rows must be 16-byte aligned");
  const int nc = (dim / 4 + 255) / 256;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (nc) {
    case 1: e = launch_k(k_rmsnorm_residual<1>, m, 256, 0, st, x, y, resid, weight, eps, dim); break;
    case 2: e = launch_k(k_rmsnorm_residual<2>, m, 256, 0, st, x, y, resid, weight, eps, dim); break;
    case 3: e = launch_k(k_rmsnorm_residual<3>, m, 256, 0, st, x, y, resid, weight, eps, dim); break;
    default: e = launch_k(k_rmsnorm_residual<4>, m, 256, 0, st, x, y, resid, weight, eps, dim); break;
  }
  GCU_CUDA(e);
  return 0;
}

GCU_EXPORT int gcu_dev_softcap(float *x, long n, float cap, void *stream) {
  if (n <= 0) return 0;
  if (!x || cap == 0.0f) return set_error("softcap: null pointer or zero cap");
  const int grid = (int)std::min<long>((n + 255) / 256, 4L * num_sms());
  GCU_CUDA(launch_k(k_softcap, grid, 256, 0, static_cast<cudaStream_t>(stream), x, n, cap));
  return 0;
}

// ---------------------------------------------------------------------------
// the residual update fused with the next block's norm + quantize
// ---------------------------------------------------------------------------
namespace gcu {
namespace {

// x = clamp(resid + rmsnorm(y, w_post))            gemma.c:4862-4881 / 4950-4962
// q, s = quantize_act(rmsnorm(x, w_next))          gemma.c:4885-4910 / 4754-4768
// One CTA per row: the two RMSNorms and the quantize step are the same
// arithmetic as gcu_dev_rmsnorm_residual followed by gcu_dev_rmsnorm_quantize
// (one launch instead of two).  w_post NULL: no post-norm.
template <int NC>
__global__ void __launch_bounds__(256) k_residual_norm_quant(float *x, int8_t *__restrict__ q, float *__restrict__ s,
                                                             const float *__restrict__ y, const float *resid,
                                                             const float *__restrict__ w_post,
                                                             const float *__restrict__ w_next, float eps, int dim) {
  __shared__ float red[8];
  ptx::griddep_launch();
  const size_t row = blockIdx.x;
  const int d4 = dim >> 2;
  ptx::griddep_wait();
  float4 v[NC];
  const float amax = prod::residual_norm_row<NC>(v, y + row * dim, resid + row * dim, w_post, w_next, eps, dim, red,
                                                 x + row * dim);
  float scale, inv;
  ptx::quant_scale(amax, scale, inv);
  int *qr = reinterpret_cast<int *>(q + row * dim);
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = threadIdx.x + i * 256;
    if (c < d4) qr[c] = ptx::quant_pack4(v[i], inv);
  }
  if (threadIdx.x == 0) s[row] = scale;
}

}  // namespace
}  // namespace gcu

GCU_EXPORT int gcu_dev_residual_norm_quantize(float *x, int8_t *q, float *s, const float *y, const float *resid,
                                              const float *w_post, const float *w_next, float eps, int m, int dim,
                                              void *stream) {
  if (m <= 0) return 0;
  if (!x || !q || !s || !y || !resid || !w_next) return set_error("residual_norm_quantize: null pointer");
  if (dim <= 0 || dim % 4 || dim > 4 * 256 * 4)
    return set_error("residual_norm_quantize: row length %d must be a positive multiple of 4 up to 4096", dim);
  if ((uintptr_t)x % 16 || (uintptr_t)y % 16 || (uintptr_t)resid % 16 || (uintptr_t)w_next % 16 ||
      (w_post && (uintptr_t)w_post % 16) || (uintptr_t)q % 4)
    return set_error("residual_norm_quantize: rows must be 16-byte aligned (codes 4-byte)");
  const int nc = (dim / 4 + 255) / 256;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (nc) {
    case 1: e = launch_k(k_residual_norm_quant<1>, m, 256, 0, st, x, q, s, y, resid, w_post, w_next, eps, dim); break;
    case 2: e = launch_k(k_residual_norm_quant<2>, m, 256, 0, st, x, q, s, y, resid, w_post, w_next, eps, dim); break;
    case 3: e = launch_k(k_residual_norm_quant<3>, m, 256, 0, st, x, q, s, y, resid, w_post, w_next, eps, dim); break;
    default: e = launch_k(k_residual_norm_quant<4>, m, 256, 0, st, x, q, s, y, resid, w_post, w_next, eps, dim); break;
  }
  GCU_CUDA(e);
  return 0;
}
