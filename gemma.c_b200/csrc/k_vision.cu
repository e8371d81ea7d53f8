// k_vision.cu -- the SigLIP head around the vision tower's int8 matmuls.
//
//   patch embedding (gemma.c:4411-4466): Conv2d(3, dim, kernel = stride =
//     psize, bias) over the (img_px, img_px, 3) image, then the dequantized
//     int8 position embedding, each step clamped to the floatx range.  As a
//     GEMM: M = patches, N = dim, K = 3*psize^2, the A operand gathered from
//     the image on the fly (one image row segment of 3*psize contiguous floats
//     per patch and kernel row py).  fp32 FMA-bound (5.5 GFLOP for SigLIP at
//     896 px); K is summed in gemma.c's order (py, px, c).
//   pooling (gemma.c:4660-4705, 4714): LayerNorm of each patch row, the
//     average of ksize x ksize patches, gemma-style RMSNorm, then the int8
//     quantization of the pooled rows for the projection GEMM (quantize_acts's
//     exact arithmetic).  One CTA per pooled token; HBM/latency-bound (one
//     read of the patch rows).
#include "gcu_internal.cuh"

#include <cfloat>

#define GCU_EXPORT extern "C" __attribute__((visibility("default")))

namespace gcu {
namespace {

__device__ __forceinline__ float clamp_fpx(float v) {  // gemma.c:2504-2506, floatx = float
  return fminf(FLT_MAX, fmaxf(-FLT_MAX, v));
}

// ---------------------------------------------------------------------------
// patch embedding
// ---------------------------------------------------------------------------
constexpr int kPeBM = 64, kPeBN = 64, kPeThreads = 256;
constexpr int kMaxPatch = 16;  // psize supported (SigLIP: 14)
constexpr int kMaxKC = 3 * kMaxPatch;

// thread (tx, ty) = (tid % 16, tid / 16) owns patches ty*4 .. +3 and output
// channels tx*4 .. +3 of the CTA's 64 x 64 tile
__global__ void __launch_bounds__(kPeThreads) k_patch_embed(float *__restrict__ x, const float *__restrict__ img,
                                                            const float *__restrict__ pe,
                                                            const float *__restrict__ pe_b,
                                                            const int8_t *__restrict__ pos_q,
                                                            const float *__restrict__ pos_s, int img_px, int P,
                                                            int dim) {
  __shared__ __align__(16) float As[kMaxKC][kPeBM];
  __shared__ __align__(16) float Bs[kMaxKC][kPeBN];
  ptx::griddep_launch();
  const int ppi = img_px / P, npatch = ppi * ppi, KC = 3 * P, K = KC * P;
  const int m0 = blockIdx.x * kPeBM, n0 = blockIdx.y * kPeBN;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  ptx::griddep_wait();
  for (int py = 0; py < P; ++py) {
    __syncthreads();  // the previous kernel row's tiles are consumed
    // A: image row oy*P + py, columns ox*P .. ox*P + P - 1, 3 channels: kk = px*3 + c
    for (int idx = threadIdx.x; idx < kPeBM * KC; idx += kPeThreads) {
      const int mm = idx / KC, kk = idx - mm * KC;
      const int p = m0 + mm;
      float v = 0.0f;
      if (p < npatch) {
        const int oy = p / ppi, ox = p - oy * ppi;
        v = __ldg(img + ((size_t)(oy * P + py) * img_px + (size_t)ox * P) * 3 + kk);
      }
      As[kk][mm] = v;
    }
    // B: pe[oc][c][py][px] in the same (px, c) order
    for (int idx = threadIdx.x; idx < kPeBN * KC; idx += kPeThreads) {
      const int nn = idx / KC, kk = idx - nn * KC;
      const int oc = n0 + nn, px = kk / 3, c = kk - px * 3;
      Bs[kk][nn] = oc < dim ? __ldg(pe + (size_t)oc * K + (size_t)c * P * P + py * P + px) : 0.0f;
    }
    __syncthreads();
    for (int kk = 0; kk < KC; ++kk) {
      const float4 a = *reinterpret_cast<const float4 *>(&As[kk][ty * 4]);
      const float4 b = *reinterpret_cast<const float4 *>(&Bs[kk][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += av[i] * bv[j];
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= npatch) continue;
    const float ps = __ldg(pos_s + m);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= dim) continue;
      float v = clamp_fpx(acc[i][j] + __ldg(pe_b + n));
      v = clamp_fpx(v + (float)pos_q[(size_t)m * dim + n] * ps);
      x[(size_t)m * dim + n] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// LayerNorm -> average pool -> RMSNorm -> quantize, one CTA per pooled token
// ---------------------------------------------------------------------------
constexpr int kPoolThreads = 256;

template <bool MAX>
__device__ __forceinline__ float block_reduce(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = MAX ? fmaxf(v, u) : v + u;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int w = 1; w < kPoolThreads / 32; ++w) r = MAX ? fmaxf(r, red[w]) : r + red[w];
  __syncthreads();  // red is written again by the next reduction
  return r;
}

// NC float4 columns per thread (dim <= NC * 4 * kPoolThreads)
template <int NC>
__global__ void __launch_bounds__(kPoolThreads) k_vision_pool(int8_t *__restrict__ q, float *__restrict__ s,
                                                              float *__restrict__ out, const float *__restrict__ x,
                                                              const float *__restrict__ post_n,
                                                              const float *__restrict__ post_nb,
                                                              const float *__restrict__ norm, float eps, int ppi,
                                                              int side, int dim) {
  __shared__ float red[kPoolThreads / 32];
  ptx::griddep_launch();
  const int o = blockIdx.x, oy = o / side, ox = o - oy * side, ks = ppi / side;
  const int d4 = dim >> 2;
  const float fdim = (float)dim;
  float4 acc[NC], w[NC], b[NC];
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    const int c = threadIdx.x + i * kPoolThreads;
    w[i] = c < d4 ? __ldg(reinterpret_cast<const float4 *>(post_n) + c) : acc[i];
    b[i] = c < d4 ? __ldg(reinterpret_cast<const float4 *>(post_nb) + c) : acc[i];
  }
  ptx::griddep_wait();
  for (int ky = 0; ky < ks; ++ky) {
    for (int kx = 0; kx < ks; ++kx) {
      const float4 *row = reinterpret_cast<const float4 *>(x + ((size_t)(oy * ks + ky) * ppi + (ox * ks + kx)) * dim);
      float4 v[NC];
      float sum = 0.0f;
#pragma unroll
      for (int i = 0; i < NC; ++i) {
        const int c = threadIdx.x + i * kPoolThreads;
        v[i] = c < d4 ? __ldg(row + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
      }
      const float mean = block_reduce<false>(sum, red) / fdim;  // gemma.c:2530-2534
      float var = 0.0f;
#pragma unroll
      for (int i = 0; i < NC; ++i) {
        if (threadIdx.x + i * kPoolThreads < d4) {
          const float a = v[i].x - mean, bb = v[i].y - mean, cc = v[i].z - mean, dd = v[i].w - mean;
          var += (a * a + bb * bb) + (cc * cc + dd * dd);
        }
      }
      const float inv_std = 1.0f / sqrtf(block_reduce<false>(var, red) / fdim + eps);  // 2536-2544
#pragma unroll
      for (int i = 0; i < NC; ++i) {  // (x - mean) * inv_std * weight + bias, summed over the window
        acc[i].x += (v[i].x - mean) * inv_std * w[i].x + b[i].x;
        acc[i].y += (v[i].y - mean) * inv_std * w[i].y + b[i].y;
        acc[i].z += (v[i].z - mean) * inv_std * w[i].z + b[i].z;
        acc[i].w += (v[i].w - mean) * inv_std * w[i].w + b[i].w;
      }
    }
  }
  // average (gemma.c:4693), RMSNorm (2513-2521)
  const float area = (float)(ks * ks);
  float sq = 0.0f;
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    acc[i] = make_float4(acc[i].x / area, acc[i].y / area, acc[i].z / area, acc[i].w / area);
    if (threadIdx.x + i * kPoolThreads < d4)
      sq += (acc[i].x * acc[i].x + acc[i].y * acc[i].y) + (acc[i].z * acc[i].z + acc[i].w * acc[i].w);
  }
  const float rms = 1.0f / sqrtf(block_reduce<false>(sq, red) / fdim + eps);
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = threadIdx.x + i * kPoolThreads;
    if (c < d4) {
      const float4 g = __ldg(reinterpret_cast<const float4 *>(norm) + c);
      acc[i] = make_float4(acc[i].x * rms * (g.x + 1.0f), acc[i].y * rms * (g.y + 1.0f),
                           acc[i].z * rms * (g.z + 1.0f), acc[i].w * rms * (g.w + 1.0f));
      amax = ptx::absmax4(acc[i], amax);
    }
  }
  amax = block_reduce<true>(amax, red);
  float scale, inv;
  ptx::quant_scale(amax, scale, inv);  // quantize_acts (gemma.c:4714) on the pooled row
  int *qr = reinterpret_cast<int *>(q + (size_t)o * dim);
  float4 *orow = out ? reinterpret_cast<float4 *>(out + (size_t)o * dim) : nullptr;
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = threadIdx.x + i * kPoolThreads;
    if (c < d4) {
      qr[c] = ptx::quant_pack4(acc[i], inv);
      if (orow) orow[c] = acc[i];
    }
  }
  if (threadIdx.x == 0) s[o] = scale;
}

bool aligned(const void *p, int a) { return ((uintptr_t)p & (a - 1)) == 0; }

}  // namespace
}  // namespace gcu

using namespace gcu;

GCU_EXPORT int gcu_dev_patch_embed(float *x, const float *img, const float *pe, const float *pe_b,
                                   const int8_t *pos_q, const float *pos_s, int img_px, int psize, int dim,
                                   void *stream) {
  if (!x || !img || !pe || !pe_b || !pos_q || !pos_s) return set_error("patch_embed: null pointer");
  if (psize < 1 || psize > kMaxPatch || img_px < psize || img_px % psize || dim < 1)
    return set_error("patch_embed: %d px image in %d px patches (psize <= %d, dividing the image), dim %d", img_px,
                     psize, kMaxPatch, dim);
  const int ppi = img_px / psize;
  const dim3 grid((ppi * ppi + kPeBM - 1) / kPeBM, (dim + kPeBN - 1) / kPeBN);
  GCU_CUDA(launch_k(k_patch_embed, grid, dim3(kPeThreads), 0, static_cast<cudaStream_t>(stream), x, img, pe, pe_b,
                    pos_q, pos_s, img_px, psize, dim));
  return 0;
}

GCU_EXPORT int gcu_dev_vision_pool_quantize(int8_t *q, float *s, float *out, const float *x, const float *post_n,
                                            const float *post_nb, const float *norm, float eps, int ppi, int side,
                                            int dim, void *stream) {
  if (!q || !s || !x || !post_n || !post_nb || !norm) return set_error("vision_pool_quantize: null pointer");
  if (side < 1 || ppi < side || ppi % side)
    return set_error("vision_pool_quantize: %d x %d patches do not pool to %d x %d", ppi, ppi, side, side);
  if (dim < 4 || dim % 4 || dim > 4 * 4 * kPoolThreads)
    return set_error("vision_pool_quantize: dim %d must be a multiple of 4 up to %d", dim, 4 * 4 * kPoolThreads);
  if (!aligned(x, 16) || !aligned(post_n, 16) || !aligned(post_nb, 16) || !aligned(norm, 16) || !aligned(q, 4) ||
      (out && !aligned(out, 16)))
    return set_error("vision_pool_quantize: rows must be 16-byte aligned (codes 4-byte)");
  const int nc = (dim / 4 + kPoolThreads - 1) / kPoolThreads;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(side * side);
  cudaError_t e;
  switch (nc) {
    case 1: e = launch_k(k_vision_pool<1>, grid, dim3(kPoolThreads), 0, st, q, s, out, x, post_n, post_nb, norm, eps, ppi, side, dim); break;
    case 2: e = launch_k(k_vision_pool<2>, grid, dim3(kPoolThreads), 0, st, q, s, out, x, post_n, post_nb, norm, eps, ppi, side, dim); break;
    case 3: e = launch_k(k_vision_pool<3>, grid, dim3(kPoolThreads), 0, st, q, s, out, x, post_n, post_nb, norm, eps, ppi, side, dim); break;
    default: e = launch_k(k_vision_pool<4>, grid, dim3(kPoolThreads), 0, st, q, s, out, x, post_n, post_nb, norm, eps, ppi, side, dim); break;
  }
  GCU_CUDA(e);
  return 0;
}
