// k_attention.cu -- the fp32 attention around the W8A8 matmuls.
//
// gemma.c keeps attention in fp32 (gemma.c:5221).  Two forms:
//   decode  (gemma.c:4836-4848): one query token; att_scores_gqa
//           (2868-2896), att_finalize = q_scale, tanh softcap, softmax
//           (4117-4133), att_values_gqa (2902-2985) over the cache window
//           [spos, spos+attlen), the query heads of one kv head together;
//   prefill (gemma.c:5160-5295): a chunk of ntok tokens, causal (with the
//           sliding window of local layers) or dense, the queries already
//           rotated and scaled.
// Both use gemma.c's own exp (fast_expf, gemma.c:4066-4089; a cephes-style
// polynomial restated in dev_fast_expf below) so the softmax weights follow
// its arithmetic; the dot products are summed in a different order than the
// reference's vectorized loops, so results agree to fp32 reassociation.
//
// Cache layout is gemma.c's (gemma.c:4806-4808, 5136-5137): kv head hk's
// position t at cache + hk*kv_stride + t*hdim, K and V in separate arrays.
//
// decode: HBM-bound on the K/V window (2 * nkv * attlen * hdim * 4 bytes).
//   Grid (splits, nkv): a CTA streams one kv head's slice of the window once,
//   scoring every query head of the group against each key row (the row is
//   loaded once per group, as att_scores_gqa keeps it in L1), then the
//   softmax weights and the weighted V rows of the same slice.  With one
//   split the CTA normalises and writes xo itself; otherwise it leaves an
//   unnormalised partial (sum, row max, weight sum) that k_attn_combine
//   merges in split order.
// prefill: fp32 FMA-bound.  CTA = (head, 64-query tile, chunk of the key
//   range); two passes over the chunk's 64-key tiles: the first finds each
//   row's maximum score, the second forms fast_expf(s - max) exactly as
//   softmax does and accumulates the weights and the weighted V rows in
//   registers.  Chunks of one query tile are merged in chunk order.
#include "gcu_internal.cuh"
#include "rope.cuh"

#include <algorithm>
#include <cmath>
#include <mutex>

#define GCU_EXPORT extern "C" __attribute__((visibility("default")))

namespace gcu {
namespace {

constexpr int kMaxGroup = 8;  // query heads per kv head

// gemma.c:4066-4089 (fast_expf): clamp, split x*log2(e) into an integer and
// a remainder (log 2 in two parts), a degree-6 polynomial for exp(r), scale
// by 2^n through the exponent bits; exactly 0 below -87.33654.
// The reference is built with -ffast-math on FMA hardware, where the
// multiply-adds contract; they are left to contract here too.
__device__ __forceinline__ float dev_fast_expf(float x) {
  float xl = x < -87.33654f ? -87.33654f : x;
  xl = xl > 88.0f ? 88.0f : xl;
  const float fx = floorf(xl * 1.44269504088896341f + 0.5f);
  float r = xl - fx * 0.693359375f;
  r -= fx * -2.12194440e-4f;
  const float z = r * r;
  float y = 1.9875691500e-4f;
  y = y * r + 1.3981999507e-3f;
  y = y * r + 8.3334519073e-3f;
  y = y * r + 4.1665795894e-2f;
  y = y * r + 1.6666665459e-1f;
  y = y * r + 5.0000001201e-1f;
  y = y * z + r + 1.0f;
  y *= __int_as_float(((int)fx + 127) << 23);
  return x < -87.33654f ? 0.0f : y;
}

// the optional tanh softcap (gemma.c:4124-4129, 5245-5250)
__device__ __forceinline__ float softcap(float s, float sc) {
  return sc != 0.0f ? tanhf(s / sc) * sc : s;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

struct DecodeArgs {
  float *xo;
  const float *xq, *kc, *vc;
  long kv_stride;
  int n_heads, nkv, spos, attlen, chunk, splits;
  float asc, sc_att;
  float *part;  // [splits][n_heads][HD] sums, then [splits][n_heads] max, then weight sums
  unsigned int *err;
  // ROPE form: xq, xk, xv are the Q/K/V projections as they come out of the
  // GEMV; every CTA normalises and rotates its group's query heads itself,
  // and the kv head's last split the new key (and the value) of position
  // spos + attlen - 1, which it writes into the cache before reading it back
  const float *xk, *xv, *nq, *nk, *freqs;
  float eps;
};

// query heads [h0, h1) of kv head hk (gqa_head_of, gemma.c:2861-2863)
__device__ __forceinline__ int gqa_head_of(int hk, int n_heads, int nkv) {
  return (hk * n_heads + nkv - 1) / nkv;
}

// ---------------------------------------------------------------------------
// decode
// ---------------------------------------------------------------------------
constexpr int kDecThreads = 256;
constexpr int kMaxChunk = 1024;  // window positions per CTA

// Cache tiles move by 1D bulk copies (positions of one kv head are
// contiguous in the cache) through a ring of NS shared-memory stages (kStages,
// or more when the launch has few CTAs per SM): the K tiles of the CTA's
// slice, then its V tiles.  Thread 0 keeps NS copies in flight; every thread
// waits on a tile's mbarrier, and one CTA barrier per tile both agrees on the
// outcome of the (bounded) wait and frees the previous tile's stage for the
// next copy.
constexpr int kTR = 16;     // cache rows per copy
constexpr int kStages = 4;  // copies in flight per CTA

template <int HD, int GM, int NS = kStages>
struct DecSmem {
  static constexpr int C4 = HD / 4;            // float4 columns of a row
  static constexpr int R = kDecThreads / C4;   // row groups of the value phase
  static constexpr size_t region = (size_t)NS * kTR * HD > (size_t)R * GM * HD
                                       ? (size_t)NS * kTR * HD
                                       : (size_t)R * GM * HD;
  static size_t bytes(int chunk) { return (region + (size_t)GM * chunk) * sizeof(float); }
};

// smem: the stage ring (reused at the end for the row groups' partial sums),
// then the scores / weights [GM][chunk]
template <int HD, int GM, bool ROPE = false, int NS = kStages>
__global__ void __launch_bounds__(kDecThreads, GM <= 2 ? 3 : GM <= 4 ? 2 : 1) k_attn_decode(DecodeArgs a) {
  extern __shared__ __align__(128) float sm[];
  __shared__ __align__(16) float qs[ROPE ? GM * HD : 4];  // the rotated query heads (ROPE form)
  __shared__ __align__(8) uint64_t full[NS];
  __shared__ float red[kDecThreads / 32][GM];
  __shared__ float stat[2][GM];  // row max, weight sum
  using S = DecSmem<HD, GM, NS>;
  float *stage = sm, *sc = sm + S::region;
  ptx::griddep_launch();
  const int split = blockIdx.x, hk = blockIdx.y;
  const int h0 = gqa_head_of(hk, a.n_heads, a.nkv);
  const int G = gqa_head_of(hk + 1, a.n_heads, a.nkv) - h0;
  const int c0 = split * a.chunk;
  const int n = min(a.attlen, c0 + a.chunk) - c0;
  const int nt = (n + kTR - 1) / kTR, nload = 2 * nt;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float *kh = a.kc + (size_t)hk * a.kv_stride + (size_t)(a.spos + c0) * HD;
  const float *vh = a.vc + (size_t)hk * a.kv_stride + (size_t)(a.spos + c0) * HD;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) ptx::mbar_init(&full[s], 1);
    ptx::fence_mbar_init();
  }
  __syncthreads();
  ptx::griddep_wait();
  const uint64_t pol = ptx::policy_evict_first();
  int issued = 0;  // thread 0 only
  auto issue = [&](int j) {
    const int tile = j < nt ? j : j - nt;
    const uint32_t bytes = (uint32_t)min(kTR, n - tile * kTR) * HD * sizeof(float);
    ptx::mbar_arrive_expect_tx(&full[j % NS], bytes);
    ptx::bulk_load(stage + (size_t)(j % NS) * kTR * HD, (j < nt ? kh : vh) + (size_t)tile * kTR * HD, bytes,
                   &full[j % NS], pol);
  };
  // The first copies go out before the ROPE form's rotation work, except in
  // the last split the tile that holds the new position (its last K tile),
  // which waits until that row is written.
  const int first = (ROPE && split == a.splits - 1) ? min(NS, nt - 1) : NS;
  if (threadIdx.x == 0)
    for (; issued < first && issued < nload; ++issued) issue(issued);
  if constexpr (ROPE) {
    // tasks of this CTA, one warp each: the G query heads, then (last split:
    // it holds the window's last position) the new key and value rows
    const bool last = split == a.splits - 1;
    const int pos = a.spos + a.attlen - 1;
    for (int t = warp; t < G + (last ? 2 : 0); t += kDecThreads / 32) {
      if (t < G) {
        rope::norm_rope_row<HD>(a.xq + (size_t)(h0 + t) * HD, a.nq, a.eps, a.freqs, 1.0f, qs + t * HD, lane);
      } else if (t == G) {
        rope::norm_rope_row<HD>(a.xk + (size_t)hk * HD, a.nk, a.eps, a.freqs, 1.0f,
                                const_cast<float *>(a.kc) + (size_t)hk * a.kv_stride + (size_t)pos * HD, lane);
      } else {
        rope::copy_row<HD>(a.xv + (size_t)hk * HD,
                           const_cast<float *>(a.vc) + (size_t)hk * a.kv_stride + (size_t)pos * HD, lane);
      }
    }
    // the cache rows just stored (generic proxy) are read back by this CTA's
    // bulk copies (async proxy)
    if (last) asm volatile("fence.proxy.async.global;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0)
      for (; issued < NS && issued < nload; ++issued) issue(issued);
  }

  // scores: each half warp takes one row of a tile (16 lanes x HD/64
  // interleaved float4, conflict-free), two rows per warp at a time; a K row
  // is read once for every query head of the group (att_scores_gqa's order
  // of work)
  constexpr int Q4 = HD / 64;  // float4 per lane of a row
  const int half = lane >> 4, l16 = lane & 15;
  float4 q[GM][Q4];
#pragma unroll
  for (int g = 0; g < GM; ++g)
#pragma unroll
    for (int i = 0; i < Q4; ++i)
      q[g][i] = g >= G ? make_float4(0.f, 0.f, 0.f, 0.f)
                : ROPE ? reinterpret_cast<const float4 *>(qs + g * HD)[i * 16 + l16]
                       : __ldg(reinterpret_cast<const float4 *>(a.xq + (size_t)(h0 + g) * HD) + i * 16 + l16);
  float wmax[GM];
#pragma unroll
  for (int g = 0; g < GM; ++g) wmax[g] = -INFINITY;
  const int c = threadIdx.x % S::C4, r = threadIdx.x / S::C4;  // value phase: float4 column, row group
  float4 acc[GM];
#pragma unroll
  for (int g = 0; g < GM; ++g) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);

  int j = 0;
  for (; j < nload; ++j) {
    const bool ok = ptx::mbar_wait(&full[j % NS], (j / NS) & 1, a.err, DEV_TIMEOUT_FULL);
    if (__syncthreads_or(!ok)) break;  // also: every thread is done with tile j - 1
    if (threadIdx.x == 0 && j >= 1 && issued < nload) {
      ptx::fence_proxy_async_smem();
      issue(issued++);
    }
    const float *tl = stage + (size_t)(j % NS) * kTR * HD;
    const int tile = j < nt ? j : j - nt;
    const int rows = min(kTR, n - tile * kTR);
    if (j < nt) {
#pragma unroll
      for (int rr = 0; rr < kTR / (kDecThreads / 16); ++rr) {
        const int row = warp * 2 + half + rr * (kDecThreads / 16);
        const bool live = row < rows;  // the shuffles below run on every lane
        float4 k[Q4];
#pragma unroll
        for (int i = 0; i < Q4; ++i)
          k[i] = live ? reinterpret_cast<const float4 *>(tl + row * HD)[i * 16 + l16]
                      : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int g = 0; g < GM; ++g) {
          float d = 0.0f;
#pragma unroll
          for (int i = 0; i < Q4; ++i) {
            d += q[g][i].x * k[i].x;
            d += q[g][i].y * k[i].y;
            d += q[g][i].z * k[i].z;
            d += q[g][i].w * k[i].w;
          }
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
          if (live && g < G) {
            const float s = softcap(d * a.asc, a.sc_att);  // att_finalize: *asc, then the cap
            wmax[g] = fmaxf(wmax[g], s);
            if (l16 == 0) sc[g * a.chunk + tile * kTR + row] = s;
          }
        }
      }
      if (j == nt - 1) {
        // softmax weights fast_expf(s - max) (gemma.c:4094-4105) and sums
#pragma unroll
        for (int g = 0; g < GM; ++g) wmax[g] = fmaxf(wmax[g], __shfl_xor_sync(0xffffffffu, wmax[g], 16));
        if (lane == 0)
#pragma unroll
          for (int g = 0; g < GM; ++g) red[warp][g] = wmax[g];
        __syncthreads();
        if (threadIdx.x < G) {
          float m = red[0][threadIdx.x];
          for (int w = 1; w < kDecThreads / 32; ++w) m = fmaxf(m, red[w][threadIdx.x]);
          stat[0][threadIdx.x] = m;
        }
        __syncthreads();
        for (int g = 0; g < G; ++g) {
          const float m = stat[0][g];
          float l = 0.0f;
          for (int t = threadIdx.x; t < n; t += kDecThreads) {
            const float p = dev_fast_expf(sc[g * a.chunk + t] - m);
            sc[g * a.chunk + t] = p;
            l += p;
          }
          l = warp_sum(l);
          if (lane == 0) red[warp][g] = l;
        }
        __syncthreads();
        if (threadIdx.x < G) {
          float l = 0.0f;
          for (int w = 0; w < kDecThreads / 32; ++w) l += red[w][threadIdx.x];
          stat[1][threadIdx.x] = l;
        }
      }
    } else {
      // weighted V rows: thread (r, c) takes rows r, r + R, ... of the tile
      for (int row = r; row < rows; row += S::R) {
        const float4 v = *reinterpret_cast<const float4 *>(tl + row * HD + c * 4);
        const int t = tile * kTR + row;
#pragma unroll
        for (int g = 0; g < GM; ++g) {
          if (g < G) {
            const float p = sc[g * a.chunk + t];
            acc[g].x += p * v.x;
            acc[g].y += p * v.y;
            acc[g].z += p * v.z;
            acc[g].w += p * v.w;
          }
        }
      }
    }
  }
  if (j < nload) {
    // a copy never completed: the error word says so; wait (bounded) for the
    // copies still in flight into this CTA's shared memory, then leave
    if (threadIdx.x == 0)
      for (int jj = j; jj < issued; ++jj)
        ptx::mbar_wait(&full[jj % NS], (jj / NS) & 1, a.err, DEV_TIMEOUT_DRAIN);
    return;
  }
  // merge the row groups' sums in row-group order (the ring is free now)
  __syncthreads();
  float *rs = sm;  // [R][GM][HD]
#pragma unroll
  for (int g = 0; g < GM; ++g)
    if (g < G) *reinterpret_cast<float4 *>(rs + ((size_t)r * GM + g) * HD + c * 4) = acc[g];
  __syncthreads();
  if (r != 0) return;
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    if (g < G) {
      float4 s = *reinterpret_cast<const float4 *>(rs + (size_t)g * HD + c * 4);
      for (int rr = 1; rr < S::R; ++rr) {
        const float4 u = *reinterpret_cast<const float4 *>(rs + ((size_t)rr * GM + g) * HD + c * 4);
        s.x += u.x;
        s.y += u.y;
        s.z += u.z;
        s.w += u.w;
      }
      acc[g] = s;
    }
  }
  if (a.splits == 1) {
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      if (g < G) {
        const float l = stat[1][g];
        *reinterpret_cast<float4 *>(a.xo + (size_t)(h0 + g) * HD + c * 4) =
            make_float4(acc[g].x / l, acc[g].y / l, acc[g].z / l, acc[g].w / l);
      }
    }
    return;
  }
  float *po = a.part + (size_t)split * a.n_heads * HD;
  float *pm = a.part + (size_t)a.splits * a.n_heads * HD + (size_t)split * a.n_heads;
  float *pl = pm + (size_t)a.splits * a.n_heads;
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    if (g < G) {
      *reinterpret_cast<float4 *>(po + (size_t)(h0 + g) * HD + c * 4) = acc[g];
      if (c == 0) {
        pm[h0 + g] = stat[0][g];
        pl[h0 + g] = stat[1][g];
      }
    }
  }
}

// merge the splits of one head in split order: m = max over splits,
// xo = sum_s e_s * O_s / sum_s e_s * l_s with e_s = fast_expf(m_s - m).
// The split maxima and weight sums are read by all threads at once and the
// e_s staged in shared memory, and each thread keeps eight splits' partial
// loads in flight, so the merge costs a few L2 round trips rather than one
// per split; the sums still run in split order.
template <int HD>
__global__ void __launch_bounds__(HD) k_attn_combine(float *xo, const float *part, int n_heads, int splits) {
  __shared__ float s_e[HD], s_l[HD], s_red[HD / 32];
  ptx::griddep_launch();
  const int h = blockIdx.x, d = threadIdx.x;
  const float *pm = part + (size_t)splits * n_heads * HD;
  const float *pl = pm + (size_t)splits * n_heads;
  ptx::griddep_wait();
  float m = -INFINITY;
  for (int s = d; s < splits; s += HD) m = fmaxf(m, pm[(size_t)s * n_heads + h]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((d & 31) == 0) s_red[d >> 5] = m;
  __syncthreads();
  m = s_red[0];
#pragma unroll
  for (int w = 1; w < HD / 32; ++w) m = fmaxf(m, s_red[w]);
  float o = 0.0f, l = 0.0f;
  for (int s0 = 0; s0 < splits; s0 += HD) {
    const int ns = min(HD, splits - s0);
    __syncthreads();  // the previous group's weights are consumed
    if (d < ns) {
      s_e[d] = dev_fast_expf(pm[(size_t)(s0 + d) * n_heads + h] - m);
      s_l[d] = pl[(size_t)(s0 + d) * n_heads + h];
    }
    __syncthreads();
    const float *ps = part + ((size_t)s0 * n_heads + h) * HD + d;
    int s = 0;
    for (; s + 8 <= ns; s += 8) {
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = ps[(size_t)(s + i) * n_heads * HD];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float e = s_e[s + i];
        l += e * s_l[s + i];
        o += e * v[i];
      }
    }
    for (; s < ns; ++s) {
      const float e = s_e[s];
      l += e * s_l[s];
      o += e * ps[(size_t)s * n_heads * HD];
    }
  }
  xo[(size_t)h * HD + d] = o / l;
}

// ---------------------------------------------------------------------------
// prefill
// ---------------------------------------------------------------------------
constexpr int kPreThreads = 256;
constexpr int kBQ = 64;  // queries per CTA
constexpr int kBK = 64;  // keys per tile

struct PrefillArgs {
  float *xo;
  int xostr;
  const float *xq, *kc, *vc;
  long kv_stride;
  int n_heads, nkv, spos, ntok, slide, mask;
  float sc_att;
  int kpc, maxch;  // key tiles per chunk, chunks per query tile (grid z)
  float *part;     // maxch > 1: [n_heads][ntok][maxch][HD] sums, then maxima, then weight sums
  unsigned int *err;
};

// Q, K and V tiles move by 1D bulk copies, one per row (rows of one head
// are contiguous in xq and in the cache), issued by warp 0 and completing on
// one mbarrier per buffer.  Each buffer has at most one copy in flight, so a
// buffer's completed-copy count gives the parity of its next wait.
template <int HD>
struct PreSmem {
  static constexpr int KS = HD + 4;   // padded Q / K / V rows: conflict-free 16-byte reads
  static constexpr int PS = kBK + 4;  // padded weight rows
  static constexpr size_t q = 0;                      // [kBQ][KS]
  static constexpr size_t k = q + (size_t)kBQ * KS;   // [kBK][KS]
  static constexpr size_t v = k + (size_t)kBK * KS;   // [kBK][KS]
  static constexpr size_t p = v + (size_t)kBK * KS;   // [kBQ][PS]
  static constexpr size_t floats = p + (size_t)kBQ * PS;
  static constexpr size_t bytes = floats * sizeof(float);
};

struct TileRing {
  uint64_t *bar;  // [3]: Q, K, V
  int issued[3], done[3];
};

// the window of token i (gemma.c:5187-5199 / 5232-5236): [t0, t1]
__device__ __forceinline__ void row_window(const PrefillArgs &a, int i, int &t0, int &t1) {
  const int pos = a.spos + i;
  if (a.mask) {
    t0 = (a.slide > 0 && pos >= a.slide) ? pos + 1 - a.slide : 0;
    t1 = pos;
  } else {
    t0 = 0;
    t1 = a.spos + a.ntok - 1;
  }
}

// n rows of HD floats at src (contiguous) into smem rows of stride KS; every
// thread of the CTA calls it (the issue counts stay uniform), warp 0 issues.
// The issuing lanes order their earlier shared-memory reads of the buffer
// (made before the caller's CTA barrier) before the async writes.
template <int HD>
__device__ __forceinline__ void ring_copy(TileRing &r, int b, float *dst, const float *src, int n, uint64_t pol) {
  ++r.issued[b];
  if (threadIdx.x >= 32) return;
  ptx::fence_proxy_async_smem();
  if (threadIdx.x == 0) ptx::mbar_arrive_expect_tx(&r.bar[b], (uint32_t)n * HD * sizeof(float));
  __syncwarp();
  for (int row = threadIdx.x; row < n; row += 32)
    ptx::bulk_load(dst + (size_t)row * PreSmem<HD>::KS, src + (size_t)row * HD, HD * sizeof(float), &r.bar[b], pol);
}

// every thread waits (bounded) for buffer b's copy in flight; the CTA barrier
// both agrees on the outcome and orders the threads' earlier work before
// what follows.  false: a copy never completed (the error word says which).
__device__ __forceinline__ bool ring_wait(TileRing &r, int b, unsigned int *err) {
  const bool ok = ptx::mbar_wait(&r.bar[b], r.done[b] & 1, err, DEV_TIMEOUT_FULL);
  if (__syncthreads_or(!ok)) return false;
  ++r.done[b];
  return true;
}

// s[i][c] = q(row ty*4 + i) . k(row tx + 16c), i, c < 4, from smem: per
// 16-byte step 4 query and 4 key loads feed 64 multiply-adds.  The loads of
// step d + 4 are issued before the multiply-adds of step d, and the 16
// accumulators advance one component at a time (16 independent chains).
template <int HD>
__device__ __forceinline__ void tile_scores(const float *qs, const float *ks, int ty, int tx, float (&s)[4][4]) {
  constexpr int KS = PreSmem<HD>::KS;
  const float *qb = qs + ty * 4 * KS, *kb = ks + tx * KS;
  auto load = [&](float4 (&q)[4], float4 (&k)[4], int d) {
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = *reinterpret_cast<const float4 *>(qb + i * KS + d);
#pragma unroll
    for (int c = 0; c < 4; ++c) k[c] = *reinterpret_cast<const float4 *>(kb + 16 * c * KS + d);
  };
  // packed fp32 multiply-adds (two per instruction): each score keeps the
  // partial sums over even and odd dimensions, added at the end
  float2 s2[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < 4; ++c) s2[i][c] = make_float2(0.0f, 0.0f);
  float4 q[4], k[4];
  load(q, k, 0);
#pragma unroll 4
  for (int d = 0; d < HD; d += 4) {
    float4 qn[4], kn[4];
    load(qn, kn, d + 4 < HD ? d + 4 : d);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c)
        s2[i][c] = __ffma2_rn(make_float2(q[i].x, q[i].y), make_float2(k[c].x, k[c].y), s2[i][c]);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c)
        s2[i][c] = __ffma2_rn(make_float2(q[i].z, q[i].w), make_float2(k[c].z, k[c].w), s2[i][c]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      q[i] = qn[i];
      k[i] = kn[i];
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < 4; ++c) s[i][c] = s2[i][c].x + s2[i][c].y;
}

// CTA (64-query tile, head, chunk of the tile's key range).  Thread (ty, tx)
// = (tid / 16, tid % 16) scores query rows ty*4 .. +3 against keys tx + 16c
// of each 64-key tile (c < 4) and, in the weight pass, owns value columns
// tx*4 + 64c of the same rows.  The first V tile loads while the first pass
// runs; each later K or V tile is issued as soon as its buffer is free.
template <int HD>
__global__ void __launch_bounds__(kPreThreads, 1) k_attn_prefill(PrefillArgs a) {
  extern __shared__ __align__(128) float smem[];
  __shared__ __align__(8) uint64_t bars[3];
  using S = PreSmem<HD>;
  float *qs = smem + S::q, *ks = smem + S::k, *vs = smem + S::v, *ps = smem + S::p;
  ptx::griddep_launch();
  const int h = blockIdx.y, i0 = blockIdx.x * kBQ;
  const int nrows = min(kBQ, a.ntok - i0);
  const int hk = h * a.nkv / a.n_heads;  // gemma.c:5172
  const float *kh = a.kc + (size_t)hk * a.kv_stride, *vh = a.vc + (size_t)hk * a.kv_stride;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  int lo, hi, unused;
  row_window(a, i0, lo, unused);  // windows only move right with i
  row_window(a, i0 + nrows - 1, unused, hi);
  // this CTA's chunk of the tile's key range: kpc key tiles
  const int ntiles = (hi + 1 - lo + kBK - 1) / kBK, nch = (ntiles + a.kpc - 1) / a.kpc;
  const int chunk = blockIdx.z;
  if (chunk >= nch) return;
  const int kbeg = lo + chunk * a.kpc * kBK;
  const int kend = min(hi + 1, kbeg + a.kpc * kBK);
  const int ntl = (kend - kbeg + kBK - 1) / kBK;  // key tiles of this chunk
  const bool one = ntl == 1;  // a one-tile chunk keeps its scores for pass 2
  int t0[4], t1[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) row_window(a, i0 + min(ty * 4 + i, nrows - 1), t0[i], t1[i]);
  TileRing ring{bars, {0, 0, 0}, {0, 0, 0}};
  if (threadIdx.x == 0) {
    for (int b = 0; b < 3; ++b) ptx::mbar_init(&bars[b], 1);
    ptx::fence_mbar_init();
  }
  __syncthreads();
  ptx::griddep_wait();
  const uint64_t pol = ptx::policy_evict_last();  // K/V tiles are read by every query tile of the head
  auto krows = [&](int k0) { return min(kBK, kend - k0); };
  ring_copy<HD>(ring, 0, qs, a.xq + ((size_t)h * a.ntok + i0) * HD, nrows, pol);
  ring_copy<HD>(ring, 1, ks, kh + (size_t)kbeg * HD, krows(kbeg), pol);
  ring_copy<HD>(ring, 2, vs, vh + (size_t)kbeg * HD, krows(kbeg), pol);

  // Rows of a buffer past its copy hold stale values: a key past kend is
  // masked by a select (never multiplied), a V row past it is never read,
  // and a query row past nrows is never written out.
  float m[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY}, s[4][4], l[4] = {0.f, 0.f, 0.f, 0.f};
  float4 acc[4][HD / 64];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < HD / 64; ++c) acc[i][c] = make_float4(0.f, 0.f, 0.f, 0.f);
  auto scores = [&](int k0) {
    tile_scores<HD>(qs, ks, ty, tx, s);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[i][c] = softcap(s[i][c], a.sc_att);
  };
  auto valid = [&](int i, int t) { return t >= t0[i] && t <= t1[i] && t < kend; };

  auto body = [&]() -> bool {
    if (!ring_wait(ring, 0, a.err)) return false;
    // pass 1: the maximum capped score of each row over its window
    for (int k0 = kbeg; k0 < kend; k0 += kBK) {
      if (!ring_wait(ring, 1, a.err)) return false;
      scores(k0);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (valid(i, k0 + tx + 16 * c)) m[i] = fmaxf(m[i], s[i][c]);
      if (!one) {  // the next pass-1 tile, or pass 2's first
        __syncthreads();
        const int kn = k0 + kBK < kend ? k0 + kBK : kbeg;
        ring_copy<HD>(ring, 1, ks, kh + (size_t)kn * HD, krows(kn), pol);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) m[i] = fmaxf(m[i], __shfl_xor_sync(0xffffffffu, m[i], o));

    // pass 2: weights fast_expf(s - max) (gemma.c:4094-4105), their sums,
    // and the weighted V rows
    for (int k0 = kbeg; k0 < kend; k0 += kBK) {
      if (!one) {
        if (!ring_wait(ring, 1, a.err)) return false;
        scores(k0);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float p = valid(i, k0 + tx + 16 * c) ? dev_fast_expf(s[i][c] - m[i]) : 0.0f;
          ps[(ty * 4 + i) * S::PS + tx + 16 * c] = p;
          l[i] += p;
        }
      // V tile: its barrier also publishes the weights and frees the K buffer
      if (!ring_wait(ring, 2, a.err)) return false;
      const bool last = k0 + kBK >= kend;
      if (!one && !last) ring_copy<HD>(ring, 1, ks, kh + (size_t)(k0 + kBK) * HD, krows(k0 + kBK), pol);
      // weighted V rows, row j + 1's weights and values loaded ahead of row j's multiply-adds
      const int jn = krows(k0);
      auto pv_load = [&](float (&p)[4], float4 (&v)[HD / 64], int j) {
#pragma unroll
        for (int i = 0; i < 4; ++i) p[i] = ps[(ty * 4 + i) * S::PS + j];
#pragma unroll
        for (int c = 0; c < HD / 64; ++c) v[c] = *reinterpret_cast<const float4 *>(vs + j * S::KS + tx * 4 + 64 * c);
      };
      float p[4];
      float4 v[HD / 64];
      pv_load(p, v, 0);
#pragma unroll 2
      for (int j = 0; j < jn; ++j) {
        float pn[4];
        float4 vn[HD / 64];
        pv_load(pn, vn, j + 1 < jn ? j + 1 : j);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 pp = make_float2(p[i], p[i]);
#pragma unroll
          for (int c = 0; c < HD / 64; ++c) {  // packed fp32 multiply-adds, two columns each
            const float2 lo = __ffma2_rn(pp, make_float2(v[c].x, v[c].y), make_float2(acc[i][c].x, acc[i][c].y));
            const float2 hi = __ffma2_rn(pp, make_float2(v[c].z, v[c].w), make_float2(acc[i][c].z, acc[i][c].w));
            acc[i][c] = make_float4(lo.x, lo.y, hi.x, hi.y);
          }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) p[i] = pn[i];
#pragma unroll
        for (int c = 0; c < HD / 64; ++c) v[c] = vn[c];
      }
      if (!last) {
        __syncthreads();  // every thread is done with this V tile and its weights
        ring_copy<HD>(ring, 2, vs, vh + (size_t)(k0 + kBK) * HD, krows(k0 + kBK), pol);
      }
    }
    return true;
  };
  if (!body()) {
    // a copy never completed: wait (bounded) for the copies still in flight
    // into this CTA's shared memory, then leave
    if (threadIdx.x == 0)
      for (int b = 0; b < 3; ++b)
        if (ring.issued[b] > ring.done[b])
          ptx::mbar_wait(&bars[b], ring.done[b] & 1, a.err, DEV_TIMEOUT_DRAIN);
    return;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) l[i] += __shfl_xor_sync(0xffffffffu, l[i], o);
  const size_t nrec = (size_t)a.n_heads * a.ntok * a.maxch;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = ty * 4 + i;
    if (row >= nrows) continue;
    if (nch == 1) {
      float *out = a.xo + (size_t)(i0 + row) * a.xostr + (size_t)h * HD + tx * 4;
#pragma unroll
      for (int c = 0; c < HD / 64; ++c)
        *reinterpret_cast<float4 *>(out + 64 * c) =
            make_float4(acc[i][c].x / l[i], acc[i][c].y / l[i], acc[i][c].z / l[i], acc[i][c].w / l[i]);
    } else {
      // a chunk of several: the unnormalised sums, the maximum and the weight
      // sum (a row with no key in this chunk leaves -inf, 0, zeros)
      const size_t r = ((size_t)h * a.ntok + i0 + row) * a.maxch + chunk;
      float *po = a.part + r * HD + tx * 4;
#pragma unroll
      for (int c = 0; c < HD / 64; ++c) *reinterpret_cast<float4 *>(po + 64 * c) = acc[i][c];
      if (tx == 0) {
        a.part[nrec * HD + r] = m[i];
        a.part[nrec * (HD + 1) + r] = l[i];
      }
    }
  }
}

// merges the chunks of token i, head h in chunk order:
// m = max m_c, xo = sum e_c O_c / sum e_c l_c, e_c = fast_expf(m_c - m)
template <int HD>
__global__ void __launch_bounds__(HD / 4) k_attn_prefill_merge(PrefillArgs a) {
  ptx::griddep_launch();
  const int i = blockIdx.x, h = blockIdx.y, c = threadIdx.x;
  const int i0 = (i / kBQ) * kBQ, nrows = min(kBQ, a.ntok - i0);
  int lo, hi, unused;
  row_window(a, i0, lo, unused);
  row_window(a, i0 + nrows - 1, unused, hi);
  const int nch = ((hi + 1 - lo + kBK - 1) / kBK + a.kpc - 1) / a.kpc;
  if (nch == 1) return;  // the chunk kernel wrote this row
  const size_t r0 = ((size_t)h * a.ntok + i) * a.maxch;
  const size_t nrec = (size_t)a.n_heads * a.ntok * a.maxch;
  const float *pm = a.part + nrec * HD, *pl = a.part + nrec * (HD + 1);
  ptx::griddep_wait();
  // eight chunks' records are requested at a time (every CTA of the launch
  // is resident at once, so each one's chain of L2 round trips is the
  // launch's time); the sums still run in chunk order
  float m = -INFINITY;
  for (int ch0 = 0; ch0 < nch; ch0 += 8) {
    float mv[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) mv[t] = ch0 + t < nch ? pm[r0 + ch0 + t] : -INFINITY;
#pragma unroll
    for (int t = 0; t < 8; ++t) m = fmaxf(m, mv[t]);
  }
  float l = 0.0f;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int ch0 = 0; ch0 < nch; ch0 += 8) {
    float ev[8], lv[8];
    float4 uv[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      if (ch0 + t < nch) {
        ev[t] = pm[r0 + ch0 + t];
        lv[t] = pl[r0 + ch0 + t];
        uv[t] = *reinterpret_cast<const float4 *>(a.part + (r0 + ch0 + t) * HD + c * 4);
      }
    }
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      if (ch0 + t < nch) {
        const float e = dev_fast_expf(ev[t] - m);
        l += e * lv[t];
        o.x += e * uv[t].x;
        o.y += e * uv[t].y;
        o.z += e * uv[t].z;
        o.w += e * uv[t].w;
      }
    }
  }
  *reinterpret_cast<float4 *>(a.xo + (size_t)i * a.xostr + (size_t)h * HD + c * 4) =
      make_float4(o.x / l, o.y / l, o.z / l, o.w / l);
}

template <int HD, int GM, bool ROPE, int NS>
cudaError_t launch_decode_ns(const DecodeArgs &a, cudaStream_t st) {
  const size_t smem = DecSmem<HD, GM, NS>::bytes(a.chunk);
  static std::mutex mu;
  static unsigned long long done_mask = 0;
  {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    if (!(done_mask & (1ull << (dev & 63)))) {
      e = cudaFuncSetAttribute(k_attn_decode<HD, GM, ROPE, NS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)DecSmem<HD, GM, NS>::bytes(kMaxChunk));
      if (e != cudaSuccess) return e;
      done_mask |= 1ull << (dev & 63);
    }
  }
  cudaError_t e = launch_k(k_attn_decode<HD, GM, ROPE, NS>, dim3(a.splits, a.nkv), dim3(kDecThreads), smem, st, a);
  if (e != cudaSuccess || a.splits == 1) return e;
  return launch_k(k_attn_combine<HD>, dim3(a.n_heads), dim3(HD), 0, st, a.xo, (const float *)a.part, a.n_heads,
                  a.splits);
}

// A launch of at most one CTA per SM (short windows over few kv heads, as in
// a small model's decode step) takes a ring of eight stages, so all the K and
// V copies of a 64-position split are in flight at once instead of the V
// tiles waiting for a second round trip; one of up to two CTAs per SM takes
// six when two such CTAs still fit on an SM.
template <int HD, int GM, bool ROPE>
cudaError_t launch_decode(const DecodeArgs &a, cudaStream_t st) {
  if (a.splits * a.nkv <= num_sms()) return launch_decode_ns<HD, GM, ROPE, 8>(a, st);
  if (a.splits * a.nkv <= 2 * num_sms() && 2 * (DecSmem<HD, GM, 6>::bytes(a.chunk) + 1024) <= 228 * 1024)
    return launch_decode_ns<HD, GM, ROPE, 6>(a, st);
  return launch_decode_ns<HD, GM, ROPE, kStages>(a, st);
}

template <int HD>
cudaError_t launch_prefill(const PrefillArgs &a, cudaStream_t st) {
  // the shared-memory opt-in is per device: once for each device this runs on
  static std::mutex mu;
  static unsigned long long done_mask = 0;
  {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    if (!(done_mask & (1ull << (dev & 63)))) {
      e = cudaFuncSetAttribute(k_attn_prefill<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)PreSmem<HD>::bytes);
      if (e != cudaSuccess) return e;
      done_mask |= 1ull << (dev & 63);
    }
  }
  const dim3 grid((a.ntok + kBQ - 1) / kBQ, a.n_heads, a.maxch);
  cudaError_t e = launch_k(k_attn_prefill<HD>, grid, dim3(kPreThreads), PreSmem<HD>::bytes, st, a);
  if (e != cudaSuccess || a.maxch == 1) return e;
  return launch_k(k_attn_prefill_merge<HD>, dim3(a.ntok, a.n_heads), dim3(HD / 4), 0, st, a);
}

bool aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }

int check_heads(const char *what, int n_heads, int nkv, int hdim) {
  if (hdim != 64 && hdim != 128 && hdim != 256)
    return set_error("%s: head size %d (64, 128 or 256 supported)", what, hdim);
  if (n_heads < 1 || nkv < 1 || nkv > n_heads)
    return set_error("%s: %d query heads over %d kv heads", what, n_heads, nkv);
  if ((n_heads + nkv - 1) / nkv > kMaxGroup)
    return set_error("%s: more than %d query heads per kv head", what, kMaxGroup);
  return 0;
}

}  // namespace
}  // namespace gcu

using namespace gcu;

namespace {

template <bool ROPE>
cudaError_t launch_decode_hd(const DecodeArgs &a, int hdim, int gmax, cudaStream_t st) {
  // the group size as a compile-time bound: registers and score storage
  if (gmax <= 1)
    return hdim == 256 ? launch_decode<256, 1, ROPE>(a, st) : hdim == 128 ? launch_decode<128, 1, ROPE>(a, st)
                                                            : launch_decode<64, 1, ROPE>(a, st);
  if (gmax <= 2)
    return hdim == 256 ? launch_decode<256, 2, ROPE>(a, st) : hdim == 128 ? launch_decode<128, 2, ROPE>(a, st)
                                                            : launch_decode<64, 2, ROPE>(a, st);
  if (gmax <= 4)
    return hdim == 256 ? launch_decode<256, 4, ROPE>(a, st) : hdim == 128 ? launch_decode<128, 4, ROPE>(a, st)
                                                            : launch_decode<64, 4, ROPE>(a, st);
  return hdim == 256 ? launch_decode<256, 8, ROPE>(a, st) : hdim == 128 ? launch_decode<128, 8, ROPE>(a, st)
                                                          : launch_decode<64, 8, ROPE>(a, st);
}

int attention_decode(DecodeArgs a, int hdim, cudaStream_t st) {
  const int n_heads = a.n_heads, nkv = a.nkv, attlen = a.attlen;
  // splits of the window: enough CTAs to stream it at full bandwidth, at
  // least 64 positions each, at most kMaxChunk
  const int target = 2 * num_sms();
  int splits = attlen <= 64 ? 1 : std::min((attlen + 63) / 64, std::max(1, (target + nkv - 1) / nkv));
  // A launch that would have at most one CTA per SM (a small model's windows
  // over few kv heads, the 12B sliding layers) takes 32-position splits:
  // twice the CTAs, each with four copies in flight (1B decode step 0.922 ->
  // 0.868 ms, 4B 1.769 -> 1.742 ms, 12B attention 1.139 -> 1.130 ms).
  if (attlen > 64 && splits * nkv <= num_sms())
    splits = std::min((attlen + 31) / 32, std::max(1, (target + nkv - 1) / nkv));
  splits = std::max(splits, (attlen + kMaxChunk - 1) / kMaxChunk);
  a.chunk = (attlen + splits - 1) / splits;
  a.splits = (attlen + a.chunk - 1) / a.chunk;
  if (a.splits > 1) {
    void *ws;
    int *cnt;
    if (gemm_workspace((size_t)a.splits * n_heads * (hdim + 2) * sizeof(float), &ws, &cnt, 0, st)) return 1;
    a.part = static_cast<float *>(ws);
  }
  const int gmax = (n_heads + nkv - 1) / nkv;
  GCU_CUDA(a.xk ? launch_decode_hd<true>(a, hdim, gmax, st) : launch_decode_hd<false>(a, hdim, gmax, st));
  return 0;
}

}  // namespace

GCU_EXPORT int gcu_dev_attention_decode(float *xo, const float *xq, const float *k_cache, const float *v_cache,
                                        long kv_stride, int n_heads, int nkv, int hdim, int spos, int attlen,
                                        float asc, float sc_att, void *stream) {
  if (check_heads("attention_decode", n_heads, nkv, hdim)) return 1;
  if (!xo || !xq || !k_cache || !v_cache) return set_error("attention_decode: null pointer");
  if (!aligned16(xo) || !aligned16(xq) || !aligned16(k_cache) || !aligned16(v_cache) || kv_stride % 4)
    return set_error("attention_decode: buffers must be 16-byte aligned, kv_stride a multiple of 4");
  if (spos < 0 || attlen < 1 || kv_stride < (long)(spos + attlen) * hdim)
    return set_error("attention_decode: window [%d, %d) outside a cache of %ld floats per head", spos,
                     spos + attlen, kv_stride);
  DecodeArgs a{xo, xq, k_cache, v_cache, kv_stride, n_heads, nkv, spos, attlen, 0, 1, asc, sc_att, nullptr,
               dev_error_word()};
  return attention_decode(a, hdim, static_cast<cudaStream_t>(stream));
}

GCU_EXPORT int gcu_dev_attention_decode_rope(float *xo, const float *xq, const float *xk, const float *xv,
                                             float *k_cache, float *v_cache, long kv_stride, const float *nq,
                                             const float *nk, float eps, const float *freqs, int n_heads, int nkv,
                                             int hdim, int spos, int attlen, float asc, float sc_att,
                                             void *stream) {
  if (check_heads("attention_decode_rope", n_heads, nkv, hdim)) return 1;
  if (!xo || !xq || !xk || !xv || !k_cache || !v_cache || !freqs)
    return set_error("attention_decode_rope: null pointer");
  if (!aligned16(xo) || !aligned16(xq) || !aligned16(xk) || !aligned16(xv) || !aligned16(k_cache) ||
      !aligned16(v_cache) || kv_stride % 4 || (uintptr_t)freqs % 8)
    return set_error("attention_decode_rope: buffers must be 16-byte aligned, kv_stride a multiple of 4");
  if (spos < 0 || attlen < 1 || kv_stride < (long)(spos + attlen) * hdim)
    return set_error("attention_decode_rope: window [%d, %d) outside a cache of %ld floats per head", spos,
                     spos + attlen, kv_stride);
  DecodeArgs a{xo, xq, k_cache, v_cache, kv_stride, n_heads, nkv, spos, attlen, 0, 1, asc, sc_att, nullptr,
               dev_error_word(), xk, xv, nq, nk, freqs, eps};
  return attention_decode(a, hdim, static_cast<cudaStream_t>(stream));
}

GCU_EXPORT int gcu_dev_attention_prefill(float *xo, int xostr, const float *xq, const float *k_cache,
                                         const float *v_cache, long kv_stride, int n_heads, int nkv, int hdim,
                                         int spos, int ntok, int slide, float sc_att, int mask, void *stream) {
  if (ntok == 0) return 0;
  if (check_heads("attention_prefill", n_heads, nkv, hdim)) return 1;
  if (!xo || !xq || !k_cache || !v_cache) return set_error("attention_prefill: null pointer");
  if (xostr == 0) xostr = n_heads * hdim;
  if (!aligned16(xo) || !aligned16(xq) || !aligned16(k_cache) || !aligned16(v_cache) || kv_stride % 4 ||
      xostr % 4 || xostr < n_heads * hdim)
    return set_error("attention_prefill: buffers must be 16-byte aligned, strides multiples of 4 floats "
                     "(xostr >= n_heads*hdim)");
  if (spos < 0 || ntok < 0 || slide < 0 || kv_stride < (long)(spos + ntok) * hdim)
    return set_error("attention_prefill: chunk [%d, %d) outside a cache of %ld floats per head", spos, spos + ntok,
                     kv_stride);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  PrefillArgs a{xo, xostr, xq, k_cache, v_cache, kv_stride, n_heads, nkv, spos, ntok, slide, mask ? 1 : 0, sc_att,
                1, 1, nullptr, dev_error_word()};
  // the causal triangle gives late query tiles many key tiles and early ones
  // few: split every tile's key range into chunks of kpc key tiles (one tile
  // per chunk up to 8 tiles, at most 8 chunks beyond), so the longest CTA
  // does kpc tiles, not the whole range
  int max_tiles = 1;
  for (int i0 = 0; i0 < ntok; i0 += kBQ) {
    const int i1 = std::min(ntok, i0 + kBQ) - 1;
    int lo = 0, hi = spos + ntok - 1;
    if (a.mask) {
      lo = (slide > 0 && spos + i0 >= slide) ? spos + i0 + 1 - slide : 0;
      hi = spos + i1;
    }
    max_tiles = std::max(max_tiles, (hi + 1 - lo + kBK - 1) / kBK);
  }
  a.kpc = std::max(1, (max_tiles + 7) / 8);
  a.maxch = (max_tiles + a.kpc - 1) / a.kpc;
  if (a.maxch > 1) {
    void *ws;
    int *cnt;
    if (gemm_workspace((size_t)n_heads * ntok * a.maxch * (hdim + 2) * sizeof(float), &ws, &cnt, 0, st)) return 1;
    a.part = static_cast<float *>(ws);
  }
  cudaError_t e = hdim == 256 ? launch_prefill<256>(a, st) : hdim == 128 ? launch_prefill<128>(a, st)
                                                                         : launch_prefill<64>(a, st);
  GCU_CUDA(e);
  return 0;
}
