// producers.cuh -- the producer arithmetic shared by the standalone producer
// kernels (k_producers.cu) and the GEMV staging that runs the same producer
// in front of a decode projection (k_gemv.cu).  One definition, so the two
// forms give the same bits.
//
//   geglu    (gemma.c:4139-4170):  h = gelu_tanh(gate) * up
//   residual (gemma.c:4862-4881 / 4950-4962):
//            x  = clamp(resid + rmsnorm(y, w_post))    (w_post NULL: y as is)
//   norm     (gemma.c:2509-2524):  xn = rmsnorm(x, w_next), rms = 1/sqrt(ss/n + eps)
//
// gelu uses CUDA's tanhf; rmsnorm sums the squares per thread and then over
// the block in a fixed order, so the values match the reference within
// ~1e-6 relative (not bit for bit), and the fused and standalone forms match
// each other exactly.
#pragma once

#include "gcu_internal.cuh"

namespace gcu {
namespace prod {

// Sum (MAX false) or max (MAX true) over WPR warps of a row group: warp
// shuffles, then the WPR partials in warp order.  `red` holds one slot per
// warp of the CTA; the trailing barrier lets the caller reuse it.
template <int WPR, bool MAX>
__device__ __forceinline__ float row_reduce(float v, float *red, int warp, int grp, int lane) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = MAX ? fmaxf(v, u) : v + u;
  }
  if (WPR == 1) return v;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[grp * WPR];
#pragma unroll
  for (int w = 1; w < WPR; ++w) r = MAX ? fmaxf(r, red[grp * WPR + w]) : r + red[grp * WPR + w];
  __syncthreads();
  return r;
}

__device__ __forceinline__ float gelu_tanh(float x) {
  const float c = 0.79788456080287f;  // sqrt(2 / pi)
  const float t = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(__fmul_rn(c, __fadd_rn(x, t)))));
}

__device__ __forceinline__ float4 geglu4(const float4 &g, const float4 &u) {
  return make_float4(__fmul_rn(gelu_tanh(g.x), u.x), __fmul_rn(gelu_tanh(g.y), u.y),
                     __fmul_rn(gelu_tanh(g.z), u.z), __fmul_rn(gelu_tanh(g.w), u.w));
}

// One row of the residual update and the next block's norm, held by a CTA of
// 256 threads: thread t owns float4 columns t, t + 256, ... (NC of them).
// Leaves rmsnorm(x, w_next) in v, writes x to x_out (when not null; x_out may
// alias resid only if this CTA is the row's only reader) and returns the
// row's |max|.  `red`: 8 floats of shared memory.
template <int NC>
__device__ __forceinline__ float residual_norm_row(float4 (&v)[NC], const float *y, const float *resid,
                                                   const float *w_post, const float *w_next, float eps, int dim,
                                                   float *red, float *x_out) {
  const int d4 = dim >> 2, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float big = 3.402823466e38f;  // FLT_MAX: clamp_fpx, gemma.c:2504-2506
  float sq = 0.0f;
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = threadIdx.x + i * 256;
    v[i] = c < d4 ? __ldg(reinterpret_cast<const float4 *>(y) + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    sq += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
  }
  float rms = 1.0f;
  if (w_post) {
    sq = row_reduce<8, false>(sq, red, warp, 0, lane);
    rms = 1.0f / sqrtf(sq / (float)dim + eps);
  }
  float sq2 = 0.0f;
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = threadIdx.x + i * 256;
    if (c >= d4) continue;
    float4 a = v[i];
    if (w_post) {
      const float4 g = __ldg(reinterpret_cast<const float4 *>(w_post) + c);
      a = make_float4(a.x * rms * (g.x + 1.0f), a.y * rms * (g.y + 1.0f), a.z * rms * (g.z + 1.0f),
                      a.w * rms * (g.w + 1.0f));
    }
    const float4 r = reinterpret_cast<const float4 *>(resid)[c];
    v[i] = make_float4(fminf(big, fmaxf(-big, a.x + r.x)), fminf(big, fmaxf(-big, a.y + r.y)),
                       fminf(big, fmaxf(-big, a.z + r.z)), fminf(big, fmaxf(-big, a.w + r.w)));
    if (x_out) reinterpret_cast<float4 *>(x_out)[c] = v[i];
    sq2 += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
  }
  sq2 = row_reduce<8, false>(sq2, red, warp, 0, lane);
  const float rms2 = 1.0f / sqrtf(sq2 / (float)dim + eps);
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = threadIdx.x + i * 256;
    if (c >= d4) continue;
    const float4 g = __ldg(reinterpret_cast<const float4 *>(w_next) + c);
    v[i] = make_float4(v[i].x * rms2 * (g.x + 1.0f), v[i].y * rms2 * (g.y + 1.0f), v[i].z * rms2 * (g.z + 1.0f),
                       v[i].w * rms2 * (g.w + 1.0f));
    amax = ptx::absmax4(v[i], amax);
  }
  return row_reduce<8, true>(amax, red, warp, 0, lane);
}

}  // namespace prod
}  // namespace gcu
