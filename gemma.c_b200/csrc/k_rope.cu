// k_rope.cu -- the steps between the Q/K/V matmuls and attention.
//
// gemma.c runs, per layer (decode gemma.c:4775-4818, prefill 5095-5145):
//   - RMSNorm of every query and key head row (qk_norm models), weight nq / nk
//     (x * rms * (w + 1), gemma.c:2509-2523);
//   - RoPE (rope_apply, gemma.c:4223-4245): pairs (d, d + hdim/2) rotated by
//     the position's (cos, sin) table entry d, the queries also scaled (1 at
//     decode, the attention scale at prefill);
//   - the chunk's rotated keys and its values copied into the KV cache.
// One warp per head row.  The frequency table is an input: gemma.c builds it
// on the host (rope_freqs, gemma.c:4178-4216, libm powf / cosf / sinf), and
// the same table is used here.  Lane l holds elements [l*P, l*P + P) of a
// row (P = hdim/32), so the partner of element d < hdim/2 sits in lane l ^ 16.
#include "gcu_internal.cuh"
#include "rope.cuh"

#define GCU_EXPORT extern "C" __attribute__((visibility("default")))

namespace gcu {
namespace {

constexpr int kRopeThreads = 256;

struct RopeArgs {
  float *xq;
  const float *xk, *xv;
  float *kc, *vc;
  long kv_stride;
  const float *nq, *nk;
  float eps;
  const float *freqs;
  float q_scale;
  int n_heads, nkv, spos, ntok;
  // token-major input (ld > 0): row t of the fused Q|K|V projection at
  // qkv + t*ld, q heads first, then k, then v; rotated queries go to xq
  // ([n_heads][ntok][hdim]).  ld == 0: head-major xq (in place), xk, xv.
  const float *qkv;
  long ld;
};

template <int HD>
__global__ void __launch_bounds__(kRopeThreads) k_qk_norm_rope_cache(RopeArgs a) {
  ptx::griddep_launch();
  const int lane = threadIdx.x & 31;
  const long row = (long)blockIdx.x * (kRopeThreads / 32) + (threadIdx.x >> 5);
  const long nq_rows = (long)a.n_heads * a.ntok, nk_rows = (long)a.nkv * a.ntok;
  if (row >= nq_rows + 2 * nk_rows) return;  // whole warp
  ptx::griddep_wait();
  if (row >= nq_rows + nk_rows) {  // a value row: straight into the cache
    const long r = row - nq_rows - nk_rows;
    const int h = (int)(r / a.ntok), t = (int)(r - (long)h * a.ntok);
    const float *src = a.ld ? a.qkv + t * a.ld + (long)(a.n_heads + a.nkv + h) * HD : a.xv + r * HD;
    rope::copy_row<HD>(src, a.vc + (size_t)h * a.kv_stride + (size_t)(a.spos + t) * HD, lane);
    return;
  }
  const bool isq = row < nq_rows;
  const long r = isq ? row : row - nq_rows;
  const int h = (int)(r / a.ntok), t = (int)(r - (long)h * a.ntok);
  const float *src = a.ld ? a.qkv + t * a.ld + (long)((isq ? 0 : a.n_heads) + h) * HD
                          : (isq ? a.xq : a.xk) + r * HD;
  float *dst = isq ? a.xq + r * HD : a.kc + (size_t)h * a.kv_stride + (size_t)(a.spos + t) * HD;
  rope::norm_rope_row<HD>(src, isq ? a.nq : a.nk, a.eps, a.freqs + (size_t)t * HD, isq ? a.q_scale : 1.0f, dst,
                          lane);
}

}  // namespace
}  // namespace gcu

using namespace gcu;

static int qk_norm_rope_cache(float *xq, const float *xk, const float *xv, const float *qkv, long ld, float *k_cache,
                              float *v_cache, long kv_stride, const float *nq, const float *nk, float eps,
                              const float *freqs, float q_scale, int n_heads, int nkv, int hdim, int spos, int ntok,
                              void *stream) {
  if (ntok == 0) return 0;
  if (!xq || (!ld && (!xk || !xv)) || (ld && !qkv) || !k_cache || !v_cache || !freqs)
    return set_error("qk_norm_rope_cache: null pointer");
  if (ld && (ld < (long)(n_heads + 2 * nkv) * hdim || ld % 2))
    return set_error("qk_norm_rope_cache: row stride %ld below the %d fused q/k/v columns", ld,
                     (n_heads + 2 * nkv) * hdim);
  if (hdim != 64 && hdim != 128 && hdim != 256)
    return set_error("qk_norm_rope_cache: head size %d (64, 128 or 256 supported)", hdim);
  if (n_heads < 1 || nkv < 1 || ntok < 0 || spos < 0 || kv_stride < (long)(spos + ntok) * hdim || kv_stride % 2)
    return set_error("qk_norm_rope_cache: chunk [%d, %d) outside a cache of %ld floats per head", spos, spos + ntok,
                     kv_stride);
  const void *ptrs[] = {xq, ld ? qkv : xk, ld ? qkv : xv, k_cache, v_cache};
  for (const void *p : ptrs)
    if ((uintptr_t)p % 8) return set_error("qk_norm_rope_cache: buffers must be 8-byte aligned");
  RopeArgs a{xq, xk, xv, k_cache, v_cache, kv_stride, nq, nk, eps, freqs, q_scale, n_heads, nkv, spos, ntok, qkv, ld};
  const long rows = (long)(n_heads + 2 * nkv) * ntok;
  const dim3 grid((unsigned)((rows + kRopeThreads / 32 - 1) / (kRopeThreads / 32)));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = hdim == 256 ? launch_k(k_qk_norm_rope_cache<256>, grid, dim3(kRopeThreads), 0, st, a)
                  : hdim == 128 ? launch_k(k_qk_norm_rope_cache<128>, grid, dim3(kRopeThreads), 0, st, a)
                                : launch_k(k_qk_norm_rope_cache<64>, grid, dim3(kRopeThreads), 0, st, a);
  GCU_CUDA(e);
  return 0;
}

GCU_EXPORT int gcu_dev_qk_norm_rope_cache(float *xq, const float *xk, const float *xv, float *k_cache,
                                          float *v_cache, long kv_stride, const float *nq, const float *nk,
                                          float eps, const float *freqs, float q_scale, int n_heads, int nkv,
                                          int hdim, int spos, int ntok, void *stream) {
  return qk_norm_rope_cache(xq, xk, xv, nullptr, 0, k_cache, v_cache, kv_stride, nq, nk, eps, freqs, q_scale,
                            n_heads, nkv, hdim, spos, ntok, stream);
}

GCU_EXPORT int gcu_dev_qkv_norm_rope_cache(float *xq, const float *qkv, long ld, float *k_cache, float *v_cache,
                                           long kv_stride, const float *nq, const float *nk, float eps,
                                           const float *freqs, float q_scale, int n_heads, int nkv, int hdim,
                                           int spos, int ntok, void *stream) {
  return qk_norm_rope_cache(xq, nullptr, nullptr, qkv, ld, k_cache, v_cache, kv_stride, nq, nk, eps, freqs, q_scale,
                            n_heads, nkv, hdim, spos, ntok, stream);
}
