// k_quant.cu -- K1: per-row symmetric int8 activation quantization.
//
// Device restatement of gemma.c:2586-2674 (quantize_act / quantize_acts) in
// the arithmetic the reference's -ffast-math build executes:
//   amax  = max |x|                    (exact, order independent)
//   scale = amax * (1/127), inv = 127 / amax      (amax > 0)
//   scale = 1,              inv = 1               (amax == 0, gemma.c:2615)
//   q     = trunc(x*inv + copysign(0.5, x*inv)), clamped to [-127, 127]
// Every product and sum is an explicit round-to-nearest intrinsic so nvcc
// cannot contract them into an FMA; the division is IEEE (no fast math).
//
// HBM-bound: 4 bytes read + 1 byte written per element, 4 bytes per row.
// One CTA per row keeps the row in registers between the max pass and the
// quantize pass, so each element is read from HBM once.
#include "gcu_internal.cuh"

namespace gcu {
namespace {

using ptx::quant_one;

__device__ __forceinline__ float block_max(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = (blockDim.x + 31) >> 5;
  if (nw == 1) return v;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = lane < nw ? red[lane] : 0.0f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) r = fmaxf(r, __shfl_xor_sync(0xffffffffu, r, o));
  __syncthreads();  // red[] is reused by the next row
  return r;
}

__device__ __forceinline__ void scale_of(float amax, float &scale, float &inv) {
  ptx::quant_scale(amax, scale, inv);
}

// Vector path: src rows 16-byte aligned, n % 4 == 0.  VPT float4 per thread.
template <int VPT>
__global__ void __launch_bounds__(1024) k_quant_rows_v4(int8_t *__restrict__ dst,
                                                        float *__restrict__ dsc,
                                                        const float *__restrict__ src,
                                                        long sstr, int m, int n) {
  __shared__ float red[32];
  const int n4 = n >> 2;
  ptx::griddep_wait();
  for (int row = blockIdx.x; row < m; row += gridDim.x) {
    const float4 *x = reinterpret_cast<const float4 *>(src + (size_t)row * sstr);
    float4 v[VPT];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = threadIdx.x + i * blockDim.x;
      if (idx < n4) {
        v[i] = __ldcs(x + idx);
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)),
                                 fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
      }
    }
    amax = block_max(amax, red);
    float scale, inv;
    scale_of(amax, scale, inv);
    char4 *q = reinterpret_cast<char4 *>(dst + (size_t)row * n);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = threadIdx.x + i * blockDim.x;
      if (idx < n4) {
        char4 c;
        c.x = (signed char)quant_one(v[i].x, inv);
        c.y = (signed char)quant_one(v[i].y, inv);
        c.z = (signed char)quant_one(v[i].z, inv);
        c.w = (signed char)quant_one(v[i].w, inv);
        q[idx] = c;
      }
    }
    if (threadIdx.x == 0) dsc[row] = scale;
  }
  ptx::griddep_launch();
}

// Any alignment and length: two passes over global memory.
__global__ void __launch_bounds__(256) k_quant_rows_any(int8_t *__restrict__ dst,
                                                        float *__restrict__ dsc,
                                                        const float *__restrict__ src,
                                                        long sstr, int m, int n) {
  __shared__ float red[32];
  ptx::griddep_wait();
  for (int row = blockIdx.x; row < m; row += gridDim.x) {
    const float *x = src + (size_t)row * sstr;
    float amax = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) amax = fmaxf(amax, fabsf(x[i]));
    amax = block_max(amax, red);
    float scale, inv;
    scale_of(amax, scale, inv);
    int8_t *q = dst + (size_t)row * n;
    for (int i = threadIdx.x; i < n; i += blockDim.x) q[i] = (int8_t)quant_one(x[i], inv);
    if (threadIdx.x == 0) dsc[row] = scale;
  }
  ptx::griddep_launch();
}

}  // namespace

int launch_quantize_rows(int8_t *dst, float *dsc, const float *src, long sstr,
                         int m, int n, cudaStream_t st) {
  if (m <= 0 || n <= 0) return 0;
  const int grid = m < 1048576 ? m : 1048576;
  const bool vec = ((uintptr_t)src % 16 == 0) && (sstr % 4 == 0) && (n % 4 == 0) &&
                   ((uintptr_t)dst % 4 == 0);
  const int n4 = n / 4;
  if (vec && n4 <= 8 * 1024) {
    int vpt = (n4 + 1023) / 1024;
    vpt = vpt <= 1 ? 1 : vpt <= 2 ? 2 : vpt <= 4 ? 4 : 8;
    int threads = (n4 + vpt - 1) / vpt;
    threads = ((threads + 31) / 32) * 32;
    if (threads < 32) threads = 32;
    switch (vpt) {
      case 1: GCU_CUDA(launch_k(k_quant_rows_v4<1>, grid, threads, 0, st, dst, dsc, src, sstr, m, n)); break;
      case 2: GCU_CUDA(launch_k(k_quant_rows_v4<2>, grid, threads, 0, st, dst, dsc, src, sstr, m, n)); break;
      case 4: GCU_CUDA(launch_k(k_quant_rows_v4<4>, grid, threads, 0, st, dst, dsc, src, sstr, m, n)); break;
      default: GCU_CUDA(launch_k(k_quant_rows_v4<8>, grid, threads, 0, st, dst, dsc, src, sstr, m, n)); break;
    }
  } else {
    GCU_CUDA(launch_k(k_quant_rows_any, grid, 256, 0, st, dst, dsc, src, sstr, m, n));
  }
  GCU_CUDA(cudaGetLastError());
  return 0;
}

}  // namespace gcu
