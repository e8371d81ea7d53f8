// k_gemv.cu -- K2: HBM-streaming int8 GEMV (decode) and small-batch GEMV.
//
// Device restatement of gemv_int8_row / gemv_int8 / gemv_int8_multi
// (gemma.c:2754-2837), extended to mb <= 8 activation rows so that the same
// kernel serves gemm_int8 calls with few tokens (batch-8 decode):
//   y[b][i] = (float)(sum_k W[i,k] * x[b,k]) * (xs[b] * ws[i])
// The int32 sum is exact (|sum| <= 15360*127^2 < 2^31) so any order gives
// the reference's bits; the epilogue is the -ffast-math build's
// (float)acc * (xs*ws) with explicit round-to-nearest multiplies.
//
// Roofline: HBM.  Each weight byte is read once (rows*k bytes + 4 per row
// of scales); x (mb*k bytes) is staged once per CTA in shared memory.
//
// Layout of the work: a weight row is split over LPR lanes, each lane
// streaming 16-byte chunks (ld.global.nc, no L1 allocation) of R rows at a
// time with U chunks per row in flight, accumulating with dp4a; LPR-lane
// shuffles reduce.  CTAs are persistent-ish (grid = SMs x occupancy) and
// stride over row groups.
#include "gcu_internal.cuh"
#include "producers.cuh"

#include <mutex>

namespace gcu {
namespace {

constexpr int kThreads = 256;
// weight sets up to this size are prefetched into L2 before the dependency wait
constexpr long kPrefetchMaxBytes = 32L << 20;

__device__ __forceinline__ int dot16(const int4 &w, const int4 &x, int acc) {
  acc = __dp4a(w.x, x.x, acc);
  acc = __dp4a(w.y, x.y, acc);
  acc = __dp4a(w.z, x.z, acc);
  acc = __dp4a(w.w, x.w, acc);
  return acc;
}

__device__ __forceinline__ float dequant(int acc, float xs, float ws) {
  return __fmul_rn(__int2float_rn(acc), __fmul_rn(xs, ws));
}

// Butterfly reduce-scatter of V per-lane partial sums over the LPR lanes of a
// row group (lane bit o of `sub`): each step the upper lane keeps the upper
// half of the values and the lower lane the lower half, each adding the half
// its partner sends -- V/2 shuffles per step instead of V.  On return v[0..]
// holds max(V/LPR, 1) complete sums with original indices idx, idx+1, ...;
// when V < LPR the remaining steps are plain xor-adds (lanes then share sums).
template <int V, int O>
struct ReduceScatter {
  static __device__ __forceinline__ void run(int *v, int sub, int &idx) {
    constexpr int H = V / 2;
    const bool up = (sub & O) != 0;
#pragma unroll
    for (int i = 0; i < H; ++i) {
      const int send = up ? v[i] : v[i + H];
      const int keep = up ? v[i + H] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, O);
    }
    if (up) idx += H;
    ReduceScatter<H, O / 2>::run(v, sub, idx);
  }
};
template <int O>
struct ReduceScatter<1, O> {
  static __device__ __forceinline__ void run(int *v, int sub, int &idx) {
    v[0] += __shfl_xor_sync(0xffffffffu, v[0], O);
    ReduceScatter<1, O / 2>::run(v, sub, idx);
  }
};
template <int V>
struct ReduceScatter<V, 0> {
  static __device__ __forceinline__ void run(int *, int, int &) {}
};
template <>
struct ReduceScatter<1, 0> {
  static __device__ __forceinline__ void run(int *, int, int &) {}
};

__device__ __forceinline__ void job_of(const GemvJobs &jobs, int row, int &j, int &local) {
  j = 0;
#pragma unroll
  for (int t = 0; t < GCU_MAX_JOBS - 1; ++t)
    if (t < jobs.njobs - 1 && row >= jobs.row_end[t]) j = t + 1;
  local = row - (j > 0 ? jobs.row_end[j - 1] : 0);
}

// One lane's share of a row group: the R weight rows from `row0`, their
// scales, and the first U chunks of each row (lane `sub` of LPR takes chunks
// sub, sub + LPR, ...).  Rows past the end read the last row and are not
// written.
template <int R, int U, int LPR>
__device__ __forceinline__ void load_chunks(const int8_t *const (&wp)[R], const bool (&valid)[R], int c0,
                                            int C, int4 (&wv)[U][R]) {
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int c = c0 + u * LPR;
#pragma unroll
    for (int r = 0; r < R; ++r)
      wv[u][r] = (c < C && valid[r]) ? ptx::ld_stream_v4(wp[r] + (size_t)c * 16) : make_int4(0, 0, 0, 0);
  }
}

template <int R, int U, int LPR>
__device__ __forceinline__ void load_rows(const GemvJobs &jobs, int row0, int sub, int k, int C,
                                          int total_rows, const int8_t *(&wp)[R], bool (&valid)[R],
                                          float (&wsc)[R], int4 (&wv)[U][R]) {
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int row = row0 + r;
    valid[r] = row < total_rows;
    int j, local;
    job_of(jobs, valid[r] ? row : total_rows - 1, j, local);
    wp[r] = jobs.w[j] + (size_t)local * k;
    wsc[r] = __ldg(jobs.ws[j] + local);
  }
  load_chunks<R, U, LPR>(wp, valid, sub, C, wv);
}

// Activation source of the GEMV (the kernel's SRC):
//   SRC_I8      already-quantized int8 rows with their scales;
//   SRC_QUANT   fp32 rows that every CTA quantizes itself while staging them
//               -- gemma.c's quantize_act + gemv_int8 pair in one launch;
//   SRC_GEGLU   one row h = gelu(gate) * up, quantized (the down projection's
//               input, gemma.c:4921-4927);
//   SRC_RESNORM one row: x = clamp(resid + rmsnorm(y, w_post)), then
//               rmsnorm(x, w_next), quantized (gemma.c:4862-4910 and
//               4950-4962 + 4754-4768); CTA 0 writes x to xout, which must
//               not alias resid (every CTA reads resid).
// The producer arithmetic is producers.cuh's, shared with the standalone
// producer kernels, so the codes are those of the two-launch sequence.  CTA 0
// also writes the codes and scales out, as quantize_act would.
enum { SRC_I8 = 0, SRC_QUANT = 1, SRC_GEGLU = 2, SRC_RESNORM = 3 };
struct GemvX {
  const int8_t *x;   // int8 rows (SRC_I8)
  long xstride;      // elements between rows (int8 or fp32)
  const float *xs;   // their scales (SRC_I8)
  const float *xf;   // fp32 rows (SRC_QUANT), the gate (SRC_GEGLU), y (SRC_RESNORM)
  int8_t *qout;      // codes out [mb][k] dense (may be null)
  float *sout;       // scales out [mb] (may be null)
  const float *xb;   // up (SRC_GEGLU), resid (SRC_RESNORM)
  const float *w_post, *w_next;  // SRC_RESNORM norm weights (w_post may be null)
  float *xout;       // SRC_RESNORM: the updated residual row
  float eps;
};

// Block-wide max; `red` (one slot per warp) is not reused by the caller.
__device__ __forceinline__ float block_max256(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int w = 1; w < kThreads / 32; ++w) r = fmaxf(r, red[w]);
  return r;
}

// Vector kernel: k % 16 == 0, every weight row and x row 16-byte aligned.
// VPT: float4 per thread of the producer row (SRC_GEGLU, SRC_RESNORM).
// Register bounds, as measured on the decode steps: the producer-staging
// variants compile with a minimum of one CTA per SM (more registers, faster
// staging: 1B step 1023 -> 986 us), the one-row int8 variants with four
// (64 registers, no spills); the quantize-staging variants keep the
// compiler's default (one CTA per SM doubled their registers and cost 14 %).
template <int MB, int LPR, int R, int U, int SRC, bool P2P, int VPT>
__global__ void __launch_bounds__(kThreads, (MB == 1 && U == 4 && SRC == SRC_I8) ? 4 : SRC >= SRC_GEGLU ? 1 : 0) k_gemv_v16(const GemvJobs jobs, const GemvX X, int mb,
                                                       long ystride, int k, int total_rows,
                                                       const PeerOut po) {
  constexpr bool FQ = SRC == SRC_QUANT;
  static_assert(SRC < SRC_GEGLU || (MB == 1 && VPT > 0 && !P2P), "producer staging: one row");
  extern __shared__ int4 xsm[];  // [MB][C] 16-byte chunks of x
  __shared__ float red[MB][kThreads / 32];  // per activation row: no reuse, no second barrier
  __shared__ float s_xsc[MB];  // activation scales, indexed by reduced-sum slot
  __shared__ int s_peers_ok;
  const int C = k >> 4;
  constexpr int kRowsPerWarp = (32 / LPR) * R;
  const int lane = threadIdx.x & 31;
  // The next launch on the stream may start its prologue now; its own wait
  // still orders it after this grid completes.
  ptx::griddep_launch();
  // Small weight sets: warm L2 with this warp's first rows while the previous
  // kernel finishes (an L2 prefetch cannot expose a stale value).  Warming
  // every row of a warp that reads two row groups measured slower (1B decode
  // step 0.943 -> 0.951 ms).
  if ((long)total_rows * k <= kPrefetchMaxBytes) {
    const int row = (blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5)) * kRowsPerWarp + lane;
    if (lane < kRowsPerWarp && row < total_rows) {
      int j, local;
      job_of(jobs, row, j, local);
      ptx::bulk_prefetch_l2(jobs.w[j] + (size_t)local * k, (uint32_t)k);
    }
  }
  // and the fp32 activation rows (the previous kernel may still be writing
  // them; a prefetch only moves lines into L2, where those writes land)
  if (FQ && blockIdx.x == 0 && threadIdx.x < mb)
    ptx::bulk_prefetch_l2(X.xf + (size_t)threadIdx.x * X.xstride, (uint32_t)k * 4u);
  if (SRC >= SRC_GEGLU && blockIdx.x == 0 && threadIdx.x < 4) {
    const float *row = threadIdx.x == 0 ? X.xf : threadIdx.x == 1 ? X.xb : threadIdx.x == 2 ? X.w_post : X.w_next;
    if (row && (SRC == SRC_RESNORM || threadIdx.x < 2)) ptx::bulk_prefetch_l2(row, (uint32_t)k * 4u);
  }
  ptx::griddep_wait();
  // fused all-gather: this launch's epoch picks the symmetric buffer half
  int epoch0 = 0;
  long half_off = 0;
  if (P2P) {
    epoch0 = *reinterpret_cast<volatile int *>(po.flag_local + 1);
    half_off = (epoch0 & 1) ? po.half_elems : 0;
  }
  // The first row group's weight chunks and scales do not depend on the
  // activation: they are requested before it is staged or quantized, so
  // their latency overlaps that work.
  const int slot = lane / LPR, sub = lane % LPR;
  const int nwarps = gridDim.x * (kThreads / 32);
  const int base0 = (blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5)) * kRowsPerWarp;
  const int8_t *wp[R];
  bool valid[R];
  float wsc[R];
  int4 wv[U][R];
  if (base0 < total_rows) load_rows<R, U, LPR>(jobs, base0 + slot * R, sub, k, C, total_rows, wp, valid, wsc, wv);
  // One barrier publishes the staged codes and the scales (every thread
  // derives the scale from the same block max).
  if (FQ) {
    for (int b = 0; b < MB; ++b) {
      if (b >= mb) {  // uniform: padding rows are zero
        for (int i = threadIdx.x; i < C; i += kThreads) xsm[b * C + i] = make_int4(0, 0, 0, 0);
        if (threadIdx.x == 0) s_xsc[b] = 0.0f;
        continue;
      }
      const float4 *xr = reinterpret_cast<const float4 *>(X.xf + (size_t)b * X.xstride);
      float amax = 0.0f;
      float scale, inv;
      if (4 * C <= 4 * kThreads) {
        // k <= 4096: each thread keeps its (at most four) float4 of the row
        // in registers across the max, one read of x
        float4 xv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int idx = threadIdx.x + i * kThreads;
          if (idx < 4 * C) {
            xv[i] = __ldg(xr + idx);
            amax = ptx::absmax4(xv[i], amax);
          }
        }
        amax = block_max256(amax, red[b]);
        ptx::quant_scale(amax, scale, inv);
        // float4 idx -> 32-bit word idx of the row's codes (word 4c + j of
        // 16-byte chunk c holds elements 16c + 4j .. 16c + 4j + 3)
        int *xw = reinterpret_cast<int *>(xsm + b * C);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int idx = threadIdx.x + i * kThreads;
          if (idx < 4 * C) {
            const int w = ptx::quant_pack4(xv[i], inv);
            xw[idx] = w;
            if (blockIdx.x == 0 && X.qout)
              reinterpret_cast<int *>(X.qout + (size_t)b * k)[idx] = w;
          }
        }
      } else {
        for (int i = threadIdx.x; i < 4 * C; i += kThreads) amax = ptx::absmax4(__ldg(xr + i), amax);
        amax = block_max256(amax, red[b]);
        ptx::quant_scale(amax, scale, inv);
        for (int i = threadIdx.x; i < C; i += kThreads) {
          int4 v;
          v.x = ptx::quant_pack4(__ldg(xr + 4 * i), inv);
          v.y = ptx::quant_pack4(__ldg(xr + 4 * i + 1), inv);
          v.z = ptx::quant_pack4(__ldg(xr + 4 * i + 2), inv);
          v.w = ptx::quant_pack4(__ldg(xr + 4 * i + 3), inv);
          xsm[b * C + i] = v;
          if (blockIdx.x == 0 && X.qout)
            *reinterpret_cast<int4 *>(X.qout + (size_t)b * k + (size_t)i * 16) = v;
        }
      }
      if (threadIdx.x == 0) {
        s_xsc[b] = scale;
        if (blockIdx.x == 0 && X.sout) X.sout[b] = scale;
      }
    }
  } else if constexpr (SRC >= SRC_GEGLU) {
    // the producer row (thread t holds float4 columns t, t + 256, ...), then
    // its codes in the same layout as above
    float4 v[VPT];
    float amax = 0.0f;
    if constexpr (SRC == SRC_GEGLU) {
      const float4 *g4 = reinterpret_cast<const float4 *>(X.xf);
      const float4 *u4 = reinterpret_cast<const float4 *>(X.xb);
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int idx = threadIdx.x + i * kThreads;
        if (idx < 4 * C) {
          v[i] = prod::geglu4(__ldg(g4 + idx), __ldg(u4 + idx));
          amax = ptx::absmax4(v[i], amax);
        }
      }
      amax = block_max256(amax, red[0]);
    } else {
      amax = prod::residual_norm_row<VPT>(v, X.xf, X.xb, X.w_post, X.w_next, X.eps, k, red[0],
                                          blockIdx.x == 0 ? X.xout : nullptr);
    }
    float scale, inv;
    ptx::quant_scale(amax, scale, inv);
    int *xw = reinterpret_cast<int *>(xsm);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = threadIdx.x + i * kThreads;
      if (idx < 4 * C) {
        const int w = ptx::quant_pack4(v[i], inv);
        xw[idx] = w;
        if (blockIdx.x == 0 && X.qout) reinterpret_cast<int *>(X.qout)[idx] = w;
      }
    }
    if (threadIdx.x == 0) {
      s_xsc[0] = scale;
      if (blockIdx.x == 0 && X.sout) X.sout[0] = scale;
    }
  } else {
    for (int i = threadIdx.x; i < MB * C; i += kThreads) {
      const int b = i / C, c = i - b * C;
      int4 v = make_int4(0, 0, 0, 0);
      if (b < mb) v = *reinterpret_cast<const int4 *>(X.x + (size_t)b * X.xstride + (size_t)c * 16);
      xsm[i] = v;
    }
    if (threadIdx.x < MB) s_xsc[threadIdx.x] = threadIdx.x < mb ? X.xs[threadIdx.x] : 0.0f;
  }
  __syncthreads();

  for (int base = base0; base < total_rows; base += nwarps * kRowsPerWarp) {
    if (base != base0) load_rows<R, U, LPR>(jobs, base + slot * R, sub, k, C, total_rows, wp, valid, wsc, wv);
    int acc[R][MB];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int b = 0; b < MB; ++b) acc[r][b] = 0;

    for (int c0 = sub; c0 < C; c0 += LPR * U) {
      if (c0 != sub) load_chunks<R, U, LPR>(wp, valid, c0, C, wv);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + u * LPR;
        if (c < C) {
#pragma unroll
          for (int b = 0; b < MB; ++b) {
            const int4 xv = xsm[b * C + c];
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r][b] = dot16(wv[u][r], xv, acc[r][b]);
          }
        }
      }
    }
    // reduce the R*MB sums over the LPR lanes; slot index vi = r*MB + b
    constexpr int V = R * MB;
    constexpr int KEEP = V >= LPR ? V / LPR : 1;
    int *v = &acc[0][0];
    int idx = 0;
    ReduceScatter<V, LPR / 2>::run(v, sub, idx);
    // when V < LPR several lanes hold the same sum: the lowest one writes
    const bool writer = V >= LPR || (sub & (LPR / V - 1)) == 0;
    if (writer) {
#pragma unroll
      for (int t = 0; t < KEEP; ++t) {
        const int vi = idx + t;
        const int r = vi / MB, b = vi - r * MB;
        const int row = base + slot * R + r;
        if (row < total_rows && b < mb) {
          int j, local;
          job_of(jobs, row, j, local);
          float ws = wsc[0];
#pragma unroll
          for (int rr = 1; rr < R; ++rr)
            if (r == rr) ws = wsc[rr];
          const float val = dequant(v[t], s_xsc[b], ws);
          if (P2P) {
            // this rank's slice of job j in the current half
            po.sym[half_off + po.off[j] + (size_t)b * po.n[j] + (size_t)po.rank * po.n_local[j] + local] = val;
          } else {
            jobs.y[j][(size_t)b * ystride + local] = val;
          }
        }
      }
    }
  }
  if (P2P) {
    // This CTA's slice stores reach this GPU's L2 (gpu scope) before it
    // counts itself; the CTA that counts last then releases everything it
    // observed at system scope (fences are cumulative), so one system-scope
    // fence per launch covers every CTA's stores.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const uint64_t t0 = ptx::globaltimer();
      if (atomicAdd(po.flag_local + 2, 1) == (int)gridDim.x - 1) {
        // last CTA of this rank: every CTA of the launch has read the epoch
        // and pushed its rows; arrive at every rank
        po.flag_local[2] = 0;
        po.flag_local[1] = epoch0 + 1;  // the next launch uses the other half
        __threadfence_system();
        for (int pr = 0; pr < po.world; ++pr) atomicAdd_system(po.flag_peer[pr], 1);
      }
      s_peers_ok = ptx::flag_wait_geq<true>(po.flag_local, (epoch0 + 1) * po.world, t0, po.err,
                                            DEV_TIMEOUT_PEER);
    }
    __syncthreads();
    // a peer that never arrived: its half may be unwritten, pull nothing (the
    // host reports code 6 and refuses further row-sharded calls)
    if (!s_peers_ok) return;
    // every rank's slices are ready in its own half: pull them into dst, 16
    // bytes at a time (a 4-float group never straddles two ranks' slices)
    for (int j = 0; j < po.njobs; ++j) {
      const long groups = ((long)po.mb * po.n[j]) >> 2;
      const float *reg = po.sym + half_off + po.off[j];
      float4 *d = reinterpret_cast<float4 *>(po.dst[j]);
      for (long g = (long)blockIdx.x * kThreads + threadIdx.x; g < groups; g += (long)gridDim.x * kThreads) {
        const long i = g << 2;
        const int owner = (int)((i % po.n[j]) / po.n_local[j]);
        d[g] = __ldcg(reinterpret_cast<const float4 *>(reinterpret_cast<const char *>(reg + i) + po.delta[owner]));
      }
    }
  }
}

// Generic kernel: any k, any alignment.  One warp per weight row, byte loads.
__global__ void __launch_bounds__(kThreads) k_gemv_any(const GemvJobs jobs,
                                                       const int8_t *__restrict__ x,
                                                       long xstride,
                                                       const float *__restrict__ xs,
                                                       int mb, long ystride, int k,
                                                       int total_rows) {
  const int lane = threadIdx.x & 31;
  const int nwarps = gridDim.x * (kThreads / 32);
  ptx::griddep_launch();
  ptx::griddep_wait();
  for (int row = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); row < total_rows;
       row += nwarps) {
    int j, local;
    job_of(jobs, row, j, local);
    const int8_t *w = jobs.w[j] + (size_t)local * k;
    int acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int l = lane; l < k; l += 32) {
      const int wv = w[l];
#pragma unroll
      for (int b = 0; b < 8; ++b)
        if (b < mb) acc[b] += wv * (int)x[(size_t)b * xstride + l];
    }
#pragma unroll
    for (int b = 0; b < 8; ++b)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[b] += __shfl_xor_sync(0xffffffffu, acc[b], o);
    if (lane == 0) {
      const float ws = jobs.ws[j][local];
      for (int b = 0; b < mb; ++b)
        jobs.y[j][(size_t)b * ystride + local] = dequant(acc[b], xs[b], ws);
    }
  }
}

template <int MB, int LPR, int SRC, bool P2P = false, int U = (MB >= 4) ? 2 : 4, int VPT = 0, int R = 2>
int launch_v16(const GemvJobs &jobs, const GemvX &X, int mb, long ystride, int k, int total_rows,
               cudaStream_t st, const PeerOut *po = nullptr) {
  auto kern = k_gemv_v16<MB, LPR, R, U, SRC, P2P, VPT>;
  PeerOut pz{};
  const PeerOut &pout = po ? *po : pz;
  const size_t smem = (size_t)MB * k;
  static std::once_flag once;
  static int regs = 0;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    cudaFuncAttributes fa;
    attr_err = cudaFuncGetAttributes(&fa, kern);
    regs = fa.numRegs;
  });
  GCU_CUDA(attr_err);
  if (smem > 48 * 1024)
    GCU_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  // resident CTAs per SM from registers (64K per SM) and shared memory
  // (228 KB per SM, 1 KB reserved per CTA), at most 2048 threads per SM
  int by_regs = 65536 / ((regs > 0 ? regs : 64) * kThreads);
  int by_smem = (int)((228 * 1024) / (smem + 1024));
  int blocks_per_sm = by_regs < by_smem ? by_regs : by_smem;
  if (blocks_per_sm > 2048 / kThreads) blocks_per_sm = 2048 / kThreads;
  if (blocks_per_sm < 1) blocks_per_sm = 1;
  constexpr int rows_per_block = (32 / LPR) * R * (kThreads / 32);
  long need = ((long)total_rows + rows_per_block - 1) / rows_per_block;
  long cap = (long)num_sms() * blocks_per_sm;
  const int grid = (int)(need < cap ? need : cap);
  GCU_CUDA(launch_k(kern, grid, kThreads, smem, st, jobs, X, mb, ystride, k, total_rows, pout));
  GCU_CUDA(cudaGetLastError());
  return 0;
}

// An L2-resident weight set at one activation row: one weight row per lane
// group instead of two when two would leave half the SMs idle and give each
// CTA 64 KB or more of weights -- twice the CTAs, each staging the same
// activation and loading half the weight bytes (1B GeGLU + down, k = 6912:
// decode step 0.957 -> 0.940 ms).  CTAs with less to load gain nothing from
// the split (one round of loads either way) and pay for the extra staging
// (270m decode, 20-32 KB per CTA: 0.2046 -> 0.2080 ms).  Integer sums are
// exact, so the split does not change the bits.
template <int MB, int LPR, int SRC, bool P2P, int U = (MB >= 4) ? 2 : 4, int VPT = 0>
int launch_fill(const GemvJobs &jobs, const GemvX &X, int mb, long ystride, int k, int total_rows,
                cudaStream_t st, const PeerOut *po = nullptr) {
  if constexpr (MB == 1 && !P2P) {
    constexpr long kRowsR1 = (32 / LPR) * (kThreads / 32);
    if (total_rows <= kRowsR1 * num_sms() && 2 * kRowsR1 * k >= (64L << 10))
      return launch_v16<MB, LPR, SRC, P2P, U, VPT, 1>(jobs, X, mb, ystride, k, total_rows, st, po);
  }
  return launch_v16<MB, LPR, SRC, P2P, U, VPT>(jobs, X, mb, ystride, k, total_rows, st, po);
}

template <int MB, int SRC, bool P2P = false>
int launch_mb(const GemvJobs &jobs, const GemvX &X, int mb, long ystride, int k, int total_rows,
              cudaStream_t st, const PeerOut *po = nullptr) {
  const int C = k / 16;
  // A set streamed from DRAM at several activation rows: four chunks per
  // lane in flight instead of two (the register budget of two was set by
  // L2-resident sets, where a round trip is short).
  const bool streamed = (long)total_rows * k > kPrefetchMaxBytes;
  if constexpr (MB >= 4 && !P2P) {
    if (streamed) {
      if (MB >= 8 || C < 64) return launch_v16<MB, 8, SRC, P2P, 4>(jobs, X, mb, ystride, k, total_rows, st, po);
      return launch_v16<MB, 16, SRC, P2P, 4>(jobs, X, mb, ystride, k, total_rows, st, po);
    }
  }
  // many activation rows: narrower lane groups keep the reduction short
  if (MB >= 8) return launch_v16<MB, 8, SRC, P2P>(jobs, X, mb, ystride, k, total_rows, st, po);
  if (MB <= 2 && (long)total_rows * k <= kPrefetchMaxBytes) {
    // One or two rows (decode) and a weight set that fits the L2 prefetch:
    // the rows are read from L2 after the dependency wait, where each round
    // of loads a lane waits for costs a round trip.  As many lanes per row as
    // make one round of U chunks cover the row (the first round is requested
    // before the activation is quantized), and rounds of 8 chunks past 128
    // chunks.  (A set streamed from DRAM keeps the split below: fewer lanes
    // per row keep more bytes in flight per warp.)
    if (C > 128) return launch_fill<MB, 32, SRC, P2P, 8>(jobs, X, mb, ystride, k, total_rows, st, po);
    if (C > 64) return launch_v16<MB, 32, SRC, P2P>(jobs, X, mb, ystride, k, total_rows, st, po);
    if (C > 32) return launch_v16<MB, 16, SRC, P2P>(jobs, X, mb, ystride, k, total_rows, st, po);
    return launch_v16<MB, 8, SRC, P2P>(jobs, X, mb, ystride, k, total_rows, st, po);
  }
  // (rows of 129-160 chunks in one round of 5 chunks per lane measured the
  // same on the 4B lm_head, already at the copy rate)
  if (C >= 128 && MB <= 2) return launch_v16<MB, 32, SRC, P2P>(jobs, X, mb, ystride, k, total_rows, st, po);
  if constexpr (MB <= 2 && !P2P) {
    // A streamed set of narrow rows: enough chunks per lane that one round
    // of loads covers a row, so each row group waits on one DRAM round trip
    // (at four a 640-byte row took a second round for its last 8 chunks).
    const int lpr = C >= 64 ? 16 : 8;
    const int u = (C + lpr - 1) / lpr;
    if (u == 5)
      return lpr == 16 ? launch_v16<MB, 16, SRC, P2P, 5>(jobs, X, mb, ystride, k, total_rows, st, po)
                       : launch_v16<MB, 8, SRC, P2P, 5>(jobs, X, mb, ystride, k, total_rows, st, po);
    if (u > 5)
      return lpr == 16 ? launch_v16<MB, 16, SRC, P2P, 8>(jobs, X, mb, ystride, k, total_rows, st, po)
                       : launch_v16<MB, 8, SRC, P2P, 8>(jobs, X, mb, ystride, k, total_rows, st, po);
  }
  if (C >= 64) return launch_v16<MB, 16, SRC, P2P>(jobs, X, mb, ystride, k, total_rows, st, po);
  return launch_v16<MB, 8, SRC, P2P>(jobs, X, mb, ystride, k, total_rows, st, po);
}

template <int SRC>
int launch_vec(const GemvJobs &jobs, const GemvX &X, int mb, long ystride, int k, int total_rows,
               cudaStream_t st) {
  if (mb == 1) return launch_mb<1, SRC>(jobs, X, mb, ystride, k, total_rows, st);
  if (mb == 2) return launch_mb<2, SRC>(jobs, X, mb, ystride, k, total_rows, st);
  if (mb <= 4) return launch_mb<4, SRC>(jobs, X, mb, ystride, k, total_rows, st);
  return launch_mb<8, SRC>(jobs, X, mb, ystride, k, total_rows, st);
}

// One producer row staged in front of the GEMV (SRC_GEGLU / SRC_RESNORM):
// the lane split of launch_mb<1> for this k, VPT float4 of the row per thread.
template <int SRC, int VPT>
int launch_staged(const GemvJobs &jobs, const GemvX &X, int k, int total_rows, cudaStream_t st) {
  const int C = k / 16;
  if (C > 128 && (long)total_rows * k <= kPrefetchMaxBytes)
    return launch_fill<1, 32, SRC, false, 8, VPT>(jobs, X, 1, 0, k, total_rows, st);
  if constexpr (SRC == SRC_RESNORM) {
    // a streamed set of model-width rows (the 4B / 12B gate + up): one round
    // of loads per row group, 5 or 8 chunks per lane
    if (C > 128 && C <= 160) return launch_v16<1, 32, SRC, false, 5, VPT>(jobs, X, 1, 0, k, total_rows, st);
    if (C > 160 && C <= 256) return launch_v16<1, 32, SRC, false, 8, VPT>(jobs, X, 1, 0, k, total_rows, st);
  }
  if (C > 64) return launch_v16<1, 32, SRC, false, 4, VPT>(jobs, X, 1, 0, k, total_rows, st);
  if (C > 32) return launch_v16<1, 16, SRC, false, 4, VPT>(jobs, X, 1, 0, k, total_rows, st);
  return launch_v16<1, 8, SRC, false, 4, VPT>(jobs, X, 1, 0, k, total_rows, st);
}

}  // namespace

int launch_gemv(const GemvJobs &jobs, const int8_t *x, long xstride, const float *xs, int mb,
                long ystride, int k, cudaStream_t st) {
  if (jobs.njobs <= 0 || mb <= 0) return 0;
  if (mb > 8) return set_error("gemv: at most 8 activation rows (got %d)", mb);
  const int total_rows = jobs.row_end[jobs.njobs - 1];
  if (total_rows <= 0) return 0;
  if (k <= 0) return set_error("gemv: k must be positive (got %d)", k);
  const int mb_pad = mb == 1 ? 1 : mb == 2 ? 2 : mb <= 4 ? 4 : 8;
  bool vec = (k % 16 == 0) && ((uintptr_t)x % 16 == 0) && (mb == 1 || xstride % 16 == 0) &&
             (size_t)mb_pad * k <= 200 * 1024;
  for (int j = 0; j < jobs.njobs && vec; ++j) vec = ((uintptr_t)jobs.w[j] % 16 == 0);
  if (vec) {
    GemvX X{x, xstride, xs, nullptr, nullptr, nullptr};
    return launch_vec<SRC_I8>(jobs, X, mb, ystride, k, total_rows, st);
  }
  long need = ((long)total_rows + 7) / 8;
  long cap = (long)num_sms() * 8;
  const int grid = (int)(need < cap ? need : cap);
  GCU_CUDA(launch_k(k_gemv_any, grid, kThreads, 0, st, jobs, x, xstride, xs, mb, ystride, k, total_rows));
  GCU_CUDA(cudaGetLastError());
  return 0;
}

// Row-sharded GEMV with the all-gather fused into its epilogue (see PeerOut).
int launch_gemv_p2p(const GemvJobs &jobs, const int8_t *x, long xstride, const float *xs,
                    const float *xf, int8_t *qout, float *sout, int mb, int k, const PeerOut &po,
                    cudaStream_t st) {
  if (jobs.njobs <= 0 || jobs.njobs != po.njobs || mb <= 0 || mb > 8 || po.mb != mb)
    return set_error("gemv p2p: 1..%d jobs and 1..8 rows", GCU_MAX_JOBS);
  const int total_rows = jobs.row_end[jobs.njobs - 1];
  bool vec = (k % 16 == 0) && (size_t)8 * k <= 200 * 1024 && total_rows > 0;
  if (xf)
    vec = vec && ((uintptr_t)xf % 16 == 0) && (mb == 1 || xstride % 4 == 0) && ((uintptr_t)qout % 16 == 0);
  else
    vec = vec && ((uintptr_t)x % 16 == 0) && (mb == 1 || xstride % 16 == 0);
  for (int j = 0; j < jobs.njobs && vec; ++j)
    vec = ((uintptr_t)jobs.w[j] % 16 == 0) && ((uintptr_t)po.dst[j] % 16 == 0) && po.n_local[j] % 4 == 0;
  if (!vec) return set_error("gemv p2p: needs k %% 16 == 0, 16-byte aligned operands and outputs");
  if (xf) {
    GemvX X{nullptr, xstride, nullptr, xf, qout, sout};
    if (mb == 1) return launch_mb<1, SRC_QUANT, true>(jobs, X, mb, 0, k, total_rows, st, &po);
    if (mb == 2) return launch_mb<2, SRC_QUANT, true>(jobs, X, mb, 0, k, total_rows, st, &po);
    if (mb <= 4) return launch_mb<4, SRC_QUANT, true>(jobs, X, mb, 0, k, total_rows, st, &po);
    return launch_mb<8, SRC_QUANT, true>(jobs, X, mb, 0, k, total_rows, st, &po);
  }
  GemvX X{x, xstride, xs, nullptr, nullptr, nullptr};
  if (mb == 1) return launch_mb<1, SRC_I8, true>(jobs, X, mb, 0, k, total_rows, st, &po);
  if (mb == 2) return launch_mb<2, SRC_I8, true>(jobs, X, mb, 0, k, total_rows, st, &po);
  if (mb <= 4) return launch_mb<4, SRC_I8, true>(jobs, X, mb, 0, k, total_rows, st, &po);
  return launch_mb<8, SRC_I8, true>(jobs, X, mb, 0, k, total_rows, st, &po);
}

// Fused quantize_acts + GEMV: xf holds mb fp32 rows (row stride xfstride
// floats); the codes and scales are also written to qout / sout.
int launch_quantize_gemv(const GemvJobs &jobs, const float *xf, long xfstride, int8_t *qout,
                         float *sout, int mb, long ystride, int k, cudaStream_t st) {
  if (jobs.njobs <= 0 || mb <= 0) return 0;
  if (mb > 8) return set_error("quantize+gemv: at most 8 activation rows (got %d)", mb);
  const int total_rows = jobs.row_end[jobs.njobs - 1];
  const int mb_pad = mb == 1 ? 1 : mb == 2 ? 2 : mb <= 4 ? 4 : 8;
  bool vec = (k % 16 == 0) && ((uintptr_t)xf % 16 == 0) && (mb == 1 || xfstride % 4 == 0) &&
             ((uintptr_t)qout % 16 == 0) && (size_t)mb_pad * k <= 200 * 1024;
  for (int j = 0; j < jobs.njobs && vec; ++j) vec = ((uintptr_t)jobs.w[j] % 16 == 0);
  if (!vec) {
    // unaligned or odd k: the two kernels back to back
    if (launch_quantize_rows(qout, sout, xf, xfstride, mb, k, st)) return 1;
    return launch_gemv(jobs, qout, k, sout, mb, ystride, k, st);
  }
  if (total_rows <= 0) return launch_quantize_rows(qout, sout, xf, xfstride, mb, k, st);
  GemvX X{nullptr, xfstride, nullptr, xf, qout, sout};
  return launch_vec<SRC_QUANT>(jobs, X, mb, ystride, k, total_rows, st);
}

// Producer row + GEMV in one launch (decode, one token): the codes, scale and
// (SRC_RESNORM) the updated residual row are also written out, as the
// standalone producer kernels write them.
int launch_geglu_gemv(const GemvJobs &jobs, const float *gate, const float *up, int8_t *qout, float *sout,
                      int k, cudaStream_t st) {
  if (jobs.njobs <= 0 || jobs.njobs > GCU_MAX_JOBS) return set_error("geglu_quantize_gemv: 1..%d jobs", GCU_MAX_JOBS);
  const int total_rows = jobs.row_end[jobs.njobs - 1];
  if (total_rows <= 0 || k <= 0 || k % 16 || k > 16384)
    return set_error("geglu_quantize_gemv: k %d must be a positive multiple of 16 up to 16384", k);
  if (!gate || !up || (uintptr_t)gate % 16 || (uintptr_t)up % 16 || (uintptr_t)qout % 16)
    return set_error("geglu_quantize_gemv: gate, up and the codes must be 16-byte aligned");
  for (int j = 0; j < jobs.njobs; ++j)
    if ((uintptr_t)jobs.w[j] % 16) return set_error("geglu_quantize_gemv: weight rows must be 16-byte aligned");
  GemvX X{};
  X.xf = gate;
  X.xb = up;
  X.xstride = k;
  X.qout = qout;
  X.sout = sout;
  const int vpt = (k / 4 + kThreads - 1) / kThreads;
  if (vpt <= 2) return launch_staged<SRC_GEGLU, 2>(jobs, X, k, total_rows, st);
  if (vpt <= 4) return launch_staged<SRC_GEGLU, 4>(jobs, X, k, total_rows, st);
  if (vpt <= 8) return launch_staged<SRC_GEGLU, 8>(jobs, X, k, total_rows, st);
  return launch_staged<SRC_GEGLU, 16>(jobs, X, k, total_rows, st);
}

int launch_resnorm_gemv(const GemvJobs &jobs, const float *y, const float *resid, const float *w_post,
                        const float *w_next, float eps, float *xout, int8_t *qout, float *sout, int dim,
                        cudaStream_t st) {
  if (jobs.njobs <= 0 || jobs.njobs > GCU_MAX_JOBS)
    return set_error("residual_norm_quantize_gemv: 1..%d jobs", GCU_MAX_JOBS);
  const int total_rows = jobs.row_end[jobs.njobs - 1];
  if (total_rows <= 0 || dim <= 0 || dim % 16 || dim > 4096)
    return set_error("residual_norm_quantize_gemv: dim %d must be a positive multiple of 16 up to 4096", dim);
  if (!y || !resid || !w_next || !xout)
    return set_error("residual_norm_quantize_gemv: null pointer");
  if ((uintptr_t)y % 16 || (uintptr_t)resid % 16 || (uintptr_t)w_next % 16 || (w_post && (uintptr_t)w_post % 16) ||
      (uintptr_t)xout % 16 || (uintptr_t)qout % 16)
    return set_error("residual_norm_quantize_gemv: rows must be 16-byte aligned");
  // every CTA reads y and resid while CTA 0 writes x: x must be another buffer
  const char *xo = reinterpret_cast<const char *>(xout);
  const size_t bytes = (size_t)dim * sizeof(float);
  auto overlaps = [&](const float *p) {
    const char *c = reinterpret_cast<const char *>(p);
    return xo < c + bytes && c < xo + bytes;
  };
  if (overlaps(resid) || overlaps(y))
    return set_error("residual_norm_quantize_gemv: x must not overlap resid or y (every CTA reads them)");
  for (int j = 0; j < jobs.njobs; ++j)
    if ((uintptr_t)jobs.w[j] % 16)
      return set_error("residual_norm_quantize_gemv: weight rows must be 16-byte aligned");
  GemvX X{};
  X.xf = y;
  X.xb = resid;
  X.w_post = w_post;
  X.w_next = w_next;
  X.eps = eps;
  X.xout = xout;
  X.xstride = dim;
  X.qout = qout;
  X.sout = sout;
  const int nc = (dim / 4 + kThreads - 1) / kThreads;
  if (nc == 1) return launch_staged<SRC_RESNORM, 1>(jobs, X, dim, total_rows, st);
  if (nc == 2) return launch_staged<SRC_RESNORM, 2>(jobs, X, dim, total_rows, st);
  if (nc == 3) return launch_staged<SRC_RESNORM, 3>(jobs, X, dim, total_rows, st);
  return launch_staged<SRC_RESNORM, 4>(jobs, X, dim, total_rows, st);
}

}  // namespace gcu
