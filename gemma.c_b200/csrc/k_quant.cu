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
// Each row stays in registers between the max pass and the quantize pass, so
// every element is read from HBM once.  Rows up to 16384 elements: WPR warps
// per row, 8/WPR rows per 256-thread CTA, every load of a lane issued before
// the first use (one barrier when WPR > 1, none otherwise).  Longer rows: one
// CTA per row.
//
// Every kernel lets the next launch on the stream start (griddepcontrol
// launch_dependents) as soon as it begins: the dependent's own wait still
// orders it after this grid's completion, so only its prologue overlaps.
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

// Warp path: src rows 16-byte aligned, n % 4 == 0, n/4 <= 32*WPR*VPT.  Lane
// `lane` of warp `wi` in the row's group holds float4 (i*WPR + wi)*32 + lane,
// so each warp load instruction reads 512 contiguous bytes.
template <int VPT, int WPR>
__global__ void __launch_bounds__(256) k_quant_warps(int8_t *__restrict__ dst,
                                                     float *__restrict__ dsc,
                                                     const float *__restrict__ src,
                                                     long sstr, int m, int n) {
  constexpr int kRows = 8 / WPR;
  __shared__ float red[8];
  ptx::griddep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = warp / WPR, wi = warp - grp * WPR;
  const int row = blockIdx.x * kRows + grp;
  const bool live = row < m;  // uniform per warp
  const int n4 = n >> 2;
  // Start the row's trip from DRAM while the previous kernel finishes: a
  // prefetch only moves lines into L2, where that kernel's writes land too.
  if (live && wi == 0 && lane == 0) ptx::bulk_prefetch_l2(src + (size_t)row * sstr, (uint32_t)n * 4u);
  ptx::griddep_wait();
  float4 v[VPT];
  float amax = 0.0f;
  if (live) {
    const float4 *x = reinterpret_cast<const float4 *>(src + (size_t)row * sstr);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = (i * WPR + wi) * 32 + lane;
      if (idx < n4) {
        v[i] = __ldcs(x + idx);
        amax = ptx::absmax4(v[i], amax);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (WPR > 1) {
    if (lane == 0) red[warp] = amax;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < WPR; ++w) amax = fmaxf(amax, red[grp * WPR + w]);
  }
  if (!live) return;
  float scale, inv;
  scale_of(amax, scale, inv);
  int *q = reinterpret_cast<int *>(dst + (size_t)row * n);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = (i * WPR + wi) * 32 + lane;
    if (idx < n4) q[idx] = ptx::quant_pack4(v[i], inv);
  }
  if (wi == 0 && lane == 0) dsc[row] = scale;
}

// Vector path for long rows: src rows 16-byte aligned, n % 4 == 0.  VPT
// float4 per thread, one CTA per row.
template <int VPT>
__global__ void __launch_bounds__(1024) k_quant_rows_v4(int8_t *__restrict__ dst,
                                                        float *__restrict__ dsc,
                                                        const float *__restrict__ src,
                                                        long sstr, int m, int n) {
  __shared__ float red[32];
  const int n4 = n >> 2;
  ptx::griddep_launch();
  if (threadIdx.x == 0 && blockIdx.x < m) ptx::bulk_prefetch_l2(src + (size_t)blockIdx.x * sstr, (uint32_t)n * 4u);
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
}

// Any alignment and length: two passes over global memory.
__global__ void __launch_bounds__(256) k_quant_rows_any(int8_t *__restrict__ dst,
                                                        float *__restrict__ dsc,
                                                        const float *__restrict__ src,
                                                        long sstr, int m, int n) {
  __shared__ float red[32];
  ptx::griddep_launch();
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
}

template <int WPR>
cudaError_t launch_warps(int vpt, int grid, int8_t *dst, float *dsc, const float *src, long sstr, int m,
                 int n, cudaStream_t st) {
  switch (vpt) {
    case 2: return launch_k(k_quant_warps<2, WPR>, grid, 256, 0, st, dst, dsc, src, sstr, m, n);
    case 4: return launch_k(k_quant_warps<4, WPR>, grid, 256, 0, st, dst, dsc, src, sstr, m, n);
    case 8: return launch_k(k_quant_warps<8, WPR>, grid, 256, 0, st, dst, dsc, src, sstr, m, n);
    default: return launch_k(k_quant_warps<16, WPR>, grid, 256, 0, st, dst, dsc, src, sstr, m, n);
  }
}

}  // namespace

int launch_quantize_rows(int8_t *dst, float *dsc, const float *src, long sstr,
                         int m, int n, cudaStream_t st) {
  if (m <= 0 || n <= 0) return 0;
  const int grid = m < 1048576 ? m : 1048576;
  const bool vec = ((uintptr_t)src % 16 == 0) && (sstr % 4 == 0) && (n % 4 == 0) &&
                   ((uintptr_t)dst % 4 == 0);
  const int n4 = n / 4;
  if (vec && n4 <= 8 * 32 * 16) {
    // fewest warps per row that hold the row in 8 float4 per lane (16 past
    // 8192 elements; fewer registers keep more CTAs resident), then more
    // while the grid is under two CTAs per SM and each lane keeps >= 2 loads
    int wpr = 1;
    while (wpr < 8 && n4 > 32 * 8 * wpr) wpr *= 2;
    const int sms = num_sms();
    while (wpr < 8 && (long)m * wpr < 16L * sms && n4 >= 32 * 2 * (2 * wpr)) wpr *= 2;
    const int need = (n4 + 32 * wpr - 1) / (32 * wpr);
    const int vpt = need <= 2 ? 2 : need <= 4 ? 4 : need <= 8 ? 8 : 16;
    const long rows_per_cta = 8 / wpr;
    const int wgrid = (int)((m + rows_per_cta - 1) / rows_per_cta);
    cudaError_t e;
    switch (wpr) {
      case 1: e = launch_warps<1>(vpt, wgrid, dst, dsc, src, sstr, m, n, st); break;
      case 2: e = launch_warps<2>(vpt, wgrid, dst, dsc, src, sstr, m, n, st); break;
      case 4: e = launch_warps<4>(vpt, wgrid, dst, dsc, src, sstr, m, n, st); break;
      default: e = launch_warps<8>(vpt, wgrid, dst, dsc, src, sstr, m, n, st); break;
    }
    GCU_CUDA(e);
  } else if (vec && n4 <= 8 * 1024) {
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
