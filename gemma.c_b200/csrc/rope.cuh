// rope.cuh -- one head row's RMSNorm and RoPE, done by one warp; shared by the
// QK-norm / RoPE / cache kernel (k_rope.cu) and the decode attention kernel
// that applies them itself (k_attention.cu), so both give the same bits.
//
// gemma.c: RMSNorm of a query or key head row with weight w (qk_norm models;
// x * rms * (w + 1), gemma.c:2509-2523), then rope_apply (gemma.c:4223-4245):
// pairs (d, d + HD/2) rotated by the (cos, sin) table entry d of the
// position, times `scale` (1 at decode, the attention scale at prefill).
// Lane l holds elements [l*P, l*P + P) of the row (P = HD/32), so the partner
// of element d < HD/2 sits in lane l ^ 16.
#pragma once

#include "gcu_internal.cuh"

namespace gcu {
namespace rope {

// src, dst: the row (8-byte aligned); w: the norm weight [HD] or null (no
// norm); fr: the position's table, HD floats (cos, sin interleaved).
template <int HD>
__device__ __forceinline__ void norm_rope_row(const float *src, const float *w, float eps, const float *fr,
                                              float scale, float *dst, int lane) {
  constexpr int P = HD / 32;
  float v[P];
#pragma unroll
  for (int i = 0; i < P; i += 2) {
    const float2 u = *reinterpret_cast<const float2 *>(src + lane * P + i);
    v[i] = u.x;
    v[i + 1] = u.y;
  }
  if (w) {  // gemma.c:2513-2521
    float sq = 0.0f;
#pragma unroll
    for (int i = 0; i < P; ++i) sq += v[i] * v[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const float rms = 1.0f / sqrtf(sq / (float)HD + eps);
#pragma unroll
    for (int i = 0; i < P; ++i) v[i] = v[i] * rms * (__ldg(w + lane * P + i) + 1.0f);
  }
  // first-half lanes hold a (element d), second-half lanes b (element
  // d + HD/2); both use table entry d
  const float *f = fr + 2 * ((lane & 15) * P);
  const bool first = lane < 16;
#pragma unroll
  for (int i = 0; i < P; ++i) {
    const float other = __shfl_xor_sync(0xffffffffu, v[i], 16);
    const float c = __ldg(f + 2 * i), s = __ldg(f + 2 * i + 1);
    const float aa = first ? v[i] : other, bb = first ? other : v[i];
    v[i] = first ? (aa * c - bb * s) * scale : (aa * s + bb * c) * scale;
  }
#pragma unroll
  for (int i = 0; i < P; i += 2)
    *reinterpret_cast<float2 *>(dst + lane * P + i) = make_float2(v[i], v[i + 1]);
}

// a value row copied as it is (one warp)
template <int HD>
__device__ __forceinline__ void copy_row(const float *src, float *dst, int lane) {
  constexpr int P = HD / 32;
#pragma unroll
  for (int i = 0; i < P; i += 2)
    *reinterpret_cast<float2 *>(dst + lane * P + i) = __ldg(reinterpret_cast<const float2 *>(src + lane * P + i));
}

}  // namespace rope
}  // namespace gcu
