// k_chain.cu -- a chain of quantize_acts -> gemm_int8 steps in one launch.
//
// gemma.c's prefill runs every projection as a pair: quantize_acts over the
// block input, then gemm_int8 of one or more weights on the codes
// (gemma.c:5034-5091 Q/K/V, 5302-5304 O, 5365-5372 up/gate, 5389-5391 down;
// the vision tower at 4497-4633).  At M = 512 tokens each of those launches
// carries a few microseconds of fixed cost -- launch, barrier and TMEM set-up,
// the first operand tiles' trip from DRAM, the epilogue tail -- for well under
// a microsecond of HBM or tensor work.  This kernel runs a list of pairs as
// one persistent launch (one CTA per SM, cooperative so all CTAs are
// resident), in order, with the same arithmetic and bits as the separate
// calls (k_quant.cu, k_gemm.cu):
//
//   for each pair i:   (q_i, s_i) = quantize_acts(x_i)
//                      dst_ij     = gemm_int8(w_ij, q_i, s_i)   for each job j
//
// Every step may read what any earlier step wrote (x_i may be an earlier
// dst), so the steps are ordered by grid-wide hand-offs: a pair's quantize
// starts once every CTA has finished the previous pair's GEMM, and its GEMM
// reads the codes once every CTA has finished quantizing.  What the hand-offs
// do not order is what cannot depend on earlier steps: the weights.  The TMA
// producer streams the pair's weight tiles into the shared-memory ring (and
// prefetches the next pair's into L2) while the previous GEMM drains and the
// quantize runs; TMEM, barriers and tensor maps are set up once per launch.
//
// Warp roles (320 threads):
//   warp 0      TMA producer over a variable-size stage ring (each pair has its
//               own tile shape): B tiles as soon as ring space frees, A tiles
//               once the pair's codes are published
//   warp 1      TMEM owner and tcgen05.mma.kind::i8 issuer (one thread)
//   warps 2-9   quantize worker (rows of the pair's x), then GEMM epilogue:
//               tcgen05.ld, dequant (float)acc * (xs*ws), fp32 out by TMA store;
//               split-K partials and their reduction as in k_gemm.cu
// Every wait is bounded (cycle counter); a wait that has run long also gives up
// once any CTA has recorded an error; on error the kernel drains its copies,
// frees TMEM and returns.  Every TMA load reads this GPU's own memory into the
// issuing CTA.
#include "gcu_internal.cuh"

#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

namespace gcu {
namespace {

constexpr int BM = 128;
constexpr int BK = 128;  // K bytes per stage (one 128-byte swizzle row)
constexpr int kEpiWarps = 8;
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kThreads = 64 + kEpiThreads;
constexpr int kJobs = 4;                  // weights per pair
constexpr int kEpiStageBytes = 32 * 128;  // 32 rows x 32 fp32 per epilogue warp
constexpr int kEpiBytes = kEpiWarps * kEpiStageBytes;
constexpr int kNB = 16;                   // stage barrier slots (>= live stages)
constexpr int kRingBytes = 192 * 1024;    // operand stages
constexpr int kBarOff = kRingBytes + kEpiBytes;
constexpr int kBarBytes = 1024;
constexpr int kSmem = 1024 + kBarOff + kBarBytes;  // + alignment slack
constexpr int kMaxVpt = 16;               // float4 per lane of a quantized row
static_assert(kSmem <= 232448, "shared memory budget");

struct alignas(64) PairDesc {
  CUtensorMap tmA;          // codes q [m][k] int8, box 128 B x (128*mb) rows
  CUtensorMap tmB[kJobs];   // weights [n][k] int8, box 128 B x bn rows
  CUtensorMap tmD[kJobs];   // outputs [m][n] fp32, box 32 x 32
  const float *x;           // quantize input, [m][xstr] fp32
  int8_t *q;                // codes, dense [m][k]
  float *s;                 // scales [m]
  const float *matsc[kJobs];
  float *dst[kJobs];
  long xstr;
  long dstr[kJobs];
  int n[kJobs];
  int tn_begin[kJobs];      // first global n-tile of job j
  int tma_store[kJobs];
  int njobs, m, k;
  int bn, mb, splits, tiles_m, tiles_n, kb_total, kb_per_split, units, dist;
  int wpr, vpt;             // quantize: warps per row, float4 per lane
};

// The step descriptors travel as kernel parameters (a grid constant): their
// fields are read through the constant cache, and the TMA unit finds the
// tensor maps in the parameter bank.  (Descriptors in global memory cost a
// dependent L2 round trip per field read in the quantize and epilogue code,
// about a microsecond each.)  A launch therefore covers at most kParamPairs
// steps; a longer chain is several launches.
constexpr int kParamPairs = 22;

struct alignas(64) ChainParams {
  PairDesc pd[kParamPairs];
  int npairs;             // <= kParamPairs
  int *sync;       // counters kSyncStride ints apart: [2i] CTAs done quantizing pair i,
                   // [2i+1] done with its GEMM, [2n] exits
  int *abort;      // nonzero once a wait of this launch has given up (device memory)
  int32_t *ws;     // split-K partials (pairs run one after another and share it)
  int *counters;   // split-K tile counters (zero between launches)
  unsigned int *err;
};
static_assert(sizeof(ChainParams) <= 32764, "kernel parameter limit");

// Each hand-off counter sits in its own 128-byte line: the CTAs that count in
// and the threads that poll one counter then do not queue behind another's.
constexpr int kSyncStride = 32;
__device__ __forceinline__ int *slot(const ChainParams &p, int i) { return p.sync + i * kSyncStride; }

// A pair's geometry, copied to registers at the start of each pair.
struct Geo {
  int njobs, m, k, bn, mb, splits, tiles_m, tiles_n, kb_total, kb_per_split, units, dist;
  int tn1, tn2, tn3;  // tn_begin of jobs 1..3 (job 0 starts at 0)
  __device__ void load(const PairDesc &D) {
    njobs = D.njobs; m = D.m; k = D.k; bn = D.bn; mb = D.mb; splits = D.splits;
    tiles_m = D.tiles_m; tiles_n = D.tiles_n; kb_total = D.kb_total;
    kb_per_split = D.kb_per_split; units = D.units; dist = D.dist;
    tn1 = D.tn_begin[1]; tn2 = D.tn_begin[2]; tn3 = D.tn_begin[3];
  }
  __device__ int tile_m() const { return BM * mb; }
  __device__ uint32_t a_bytes() const { return (uint32_t)(BM * mb * BK); }
  __device__ uint32_t stage_bytes() const { return (uint32_t)((BM * mb + bn) * BK); }
};

struct Unit {
  int m_t, s, job, n_t, tile;
};

__device__ __forceinline__ Unit decode_unit(const Geo &g, int u) {
  Unit w;
  w.m_t = u % g.tiles_m;
  const int rest = u / g.tiles_m;
  w.s = rest % g.splits;
  const int ntg = rest / g.splits;
  int j = 0, tb = 0;
  if (g.njobs > 1 && ntg >= g.tn1) { j = 1; tb = g.tn1; }
  if (g.njobs > 2 && ntg >= g.tn2) { j = 2; tb = g.tn2; }
  if (g.njobs > 3 && ntg >= g.tn3) { j = 3; tb = g.tn3; }
  w.job = j;
  w.n_t = ntg - tb;
  w.tile = w.m_t * g.tiles_n + ntg;
  return w;
}

__device__ __forceinline__ float dequant(int acc, float xs, float ws) {
  return __fmul_rn(__int2float_rn(acc), __fmul_rn(xs, ws));
}

// Where a wait that gives up reports: the library's error word (which may be
// mapped host memory, so it is written once and never polled) and the
// launch's abort word in device memory, which the other waits poll.
struct Fail {
  unsigned int *err;
  int *abort;
};

// Waits are timed on the SM's cycle counter: reading %globaltimer costs
// about 0.1 us on B200, and a waiter that reads it between polls notices a
// landed stage that much later, on every stage.  A wait gives up after
// kBudgetCycles (2 s at 2 GHz, longer at lower clocks), or -- once it has
// waited kErrPollCycles -- as soon as another wait has given up.  The abort
// word is only read after that point: a load from global memory stalls the
// waiting thread for about a microsecond.  (Polling the error word itself
// was measured to stall whole launches: in mapped host memory each poll is a
// PCIe read, and hundreds of waiters flood the link.)
constexpr long long kBudgetCycles = 4000000000ll;
constexpr long long kErrPollCycles = 40000ll;

__device__ __forceinline__ bool give_up(long long t0, Fail f, unsigned int code) {
  const long long dt = clock64() - t0;
  if (dt < kErrPollCycles) return false;
  if (*reinterpret_cast<volatile int *>(f.abort) != 0) return true;
  if (dt > kBudgetCycles) {
    ptx::record_err(f.err, code);
    *reinterpret_cast<volatile int *>(f.abort) = 1;
    __threadfence();
    return true;
  }
  return false;
}

__device__ __forceinline__ int ld_relaxed_gpu(const int *p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until *flag >= target, then acquire at gpu scope; bounded.  The spin
// is relaxed loads with a short back-off; one acquire load at the end.
__device__ __forceinline__ bool chain_wait(const int *flag, int target, Fail err,
                                           unsigned int code = DEV_TIMEOUT_CHAIN) {
  if (ld_relaxed_gpu(flag) < target) {
    const long long t0 = clock64();
    int n = 0;
    int nap = 32;
    while (ld_relaxed_gpu(flag) < target) {
      __nanosleep(nap);
      if (nap < 256) nap += 16;  // long waits poll the shared line less often
      if ((++n & 15) == 0 && give_up(t0, err, code)) return false;
    }
  }
  (void)ptx::ld_acquire_gpu(flag);
  return true;
}

// mbarrier wait, bounded.  `nap` > 0: sleep that many ns between polls, for
// the 256 epilogue threads, whose spinning would otherwise take issue slots
// from the producer and MMA threads on the same SM sub-partitions.
__device__ __forceinline__ bool bar_wait(uint64_t *bar, uint32_t parity, Fail err,
                                         unsigned int code, int nap = 0) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    for (int i = 0; i < 16; ++i) {
      if (ptx::mbar_try_wait(bar, parity)) return true;
      if (nap) __nanosleep(nap);
    }
    if (give_up(t0, err, code)) return false;
  }
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void red_release_add(int *p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// K rotation: every CTA leaves a hand-off at the same moment, and the CTAs
// that share an operand tile (the N tiles of one M block, the M blocks of one
// N tile) would all request the same K block at once.  Each unit starts its K
// loop at block (tile % nk) and wraps around, so those requests spread over
// different L2 lines; the int32 sums are exact, so the order cannot change a
// bit.  (On the 1B prefill layer it measured no different from a common
// start: the per-stage cost is in the MMA issue, not in the operand reads.)
//
// The stage ring: stages are placed one after another, wrapping to offset 0
// when the next stage would run past the end.  The producer and the MMA warp
// step through the same sequence of stage sizes, so they agree on offsets.
__device__ __forceinline__ uint32_t ring_place(uint32_t &head, uint32_t bytes) {
  const uint32_t off = head + bytes > (uint32_t)kRingBytes ? 0u : head;
  head = off + bytes;
  return off;
}

// L2 prefetch of the rows of x this CTA will quantize.  A prefetch returns no
// data to the CTA, so it may run before the hand-off that orders the step
// after its producers: a line written later is read fresh from L2.
__device__ __forceinline__ void prefetch_x_rows(const PairDesc &D) {
  const int gpc = kEpiWarps / D.wpr;
  const int total = gridDim.x * gpc;
  const uint32_t bytes = (uint32_t)D.k * 4u;
  for (int grp = 0; grp < gpc; ++grp)
    for (int row = grp * gridDim.x + blockIdx.x; row < D.m; row += total)
      ptx::bulk_prefetch_l2(D.x + (size_t)row * D.xstr, bytes);
}

// ---- MMA issue of one stage --------------------------------------------------
// The K steps of a stage (4 x 32 bytes) go to `nc` accumulators round robin:
// consecutive tcgen05.mma into one accumulator wait for each other (~170
// cycles apiece on B200 for N <= 128, measured), while MMAs into different
// accumulators pipeline.  A one-M-block tile of bn <= 128 columns therefore
// keeps 256/bn accumulators side by side in its 256-column TMEM slot, and the
// epilogue adds them (exact int32 adds: the bits do not change).
template <int MB>
__device__ __forceinline__ void mma_stage(uint32_t d_tmem, uint32_t a0, uint32_t b0, uint32_t idesc,
                                          int bn, int nc, bool first) {
#pragma unroll
  for (int j = 0; j < BK / 32; ++j) {
    const int c = MB == 1 ? (j & (nc - 1)) : 0;
    const uint32_t acc = (!first || j >= (MB == 1 ? nc : 1)) ? 1u : 0u;
#pragma unroll
    for (int mb = 0; mb < MB; ++mb)
      ptx::mma_i8(d_tmem + (uint32_t)((c + mb) * bn), ptx::smem_desc_k128(a0 + mb * BM * BK + 32 * j),
                  ptx::smem_desc_k128(b0 + 32 * j), idesc, acc);
  }
}

// accumulators of a tile: 256/bn for one M block of bn <= 128, else 1
__device__ __forceinline__ int n_chains(int mb, int bn) { return mb == 1 && bn <= 128 ? 256 / bn : 1; }

// 32 columns of a warp's lane quarter, summed over the tile's nc accumulators
// (nc - 1 more loads bn columns apart)
__device__ __forceinline__ void tmem_ld_sum(uint32_t taddr, int bn, int nc, uint32_t (&r)[32]) {
  ptx::tmem_ld_32x32(taddr, r);
  ptx::tmem_ld_wait();
#pragma unroll 1
  for (int c = 1; c < nc; ++c) {
    uint32_t t[32];
    ptx::tmem_ld_32x32(taddr + (uint32_t)(c * bn), t);
    ptx::tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] += t[i];
  }
}

// ---- quantize step (epilogue warps of every CTA) ----------------------------
// Rows of x go to groups of `wpr` warps (8/wpr groups per CTA): row r to CTA
// r % grid, so every SM carries a share of the loads; lane `lane` of warp `wi`
// of a group holds float4s (i*wpr + wi)*32 + lane, i < vpt, so a warp load
// reads 512 contiguous bytes.  The arithmetic is k_quant.cu's
// (gemma.c:2586-2650 under -ffast-math).
// The cross-warp maxima go through red[2][8], alternating halves row by row;
// every step starts on the first half (a CTA-wide barrier separates steps, and
// the warp groups change with the step's row length).
__device__ __forceinline__ void quantize_rows(const PairDesc &D, float *red) {
  int rpar = 0;
  const int et = threadIdx.x - 64;
  const int ew = et >> 5, lane = et & 31;
  const int wpr = D.wpr, vpt = D.vpt;
  const int grp = ew / wpr, wi = ew - grp * wpr;
  const int gpc = kEpiWarps / wpr;
  const int total = gridDim.x * gpc;
  const int k4 = D.k >> 2;
  for (int row = grp * gridDim.x + blockIdx.x; row < D.m; row += total) {
    const float4 *x = reinterpret_cast<const float4 *>(D.x + (size_t)row * D.xstr);
    float4 v[kMaxVpt];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxVpt; ++i) {
      const int idx = (i * wpr + wi) * 32 + lane;
      if (i < vpt && idx < k4) {
        v[i] = __ldcg(x + idx);  // coherent: x may be an earlier step's output
        amax = ptx::absmax4(v[i], amax);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (wpr > 1) {
      float *r = red + rpar * kEpiWarps;
      if (lane == 0) r[ew] = amax;
      ptx::named_bar_sync(2 + grp, 32 * wpr);
      for (int w = 0; w < wpr; ++w) amax = fmaxf(amax, r[grp * wpr + w]);
      rpar ^= 1;
    }
    float scale, inv;
    ptx::quant_scale(amax, scale, inv);
    int *q = reinterpret_cast<int *>(D.q + (size_t)row * D.k);
#pragma unroll
    for (int i = 0; i < kMaxVpt; ++i) {
      const int idx = (i * wpr + wi) * 32 + lane;
      if (i < vpt && idx < k4) q[idx] = ptx::quant_pack4(v[i], inv);
    }
    if (wi == 0 && lane == 0) D.s[row] = scale;
  }
}

// ---- GEMM epilogue pieces (k_gemm.cu's, with the tile shape at run time) ----
__device__ __forceinline__ void emit_chunk(const PairDesc &D, const CUtensorMap *tmD, int job,
                                           const int (&acc)[32], float xs, float ws_lane, int row,
                                           int col0, int lane, uint8_t *stage, int tile_row0, int m) {
  float out[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) out[i] = dequant(acc[i], xs, __shfl_sync(0xffffffffu, ws_lane, i));
  if (D.tma_store[job]) {
    if (lane == 0) ptx::bulk_wait_read<0>();  // the previous store left this buffer
    __syncwarp();
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float4 v = make_float4(out[4 * c], out[4 * c + 1], out[4 * c + 2], out[4 * c + 3]);
      *reinterpret_cast<float4 *>(stage + lane * 128 + ((c ^ (lane & 7)) << 4)) = v;
    }
    ptx::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0 && tile_row0 < m) {
      ptx::tma_store_2d(tmD, stage, col0, tile_row0);
      ptx::bulk_commit();
    }
  } else if (row < m) {
    const int n = D.n[job];
    float *d = D.dst[job] + (size_t)row * D.dstr[job];
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (col0 + i < n) d[col0 + i] = out[i];
  }
}

// Split-K, every split resident: split w.s reduces the tile's 32x32 blocks
// b = w.s, w.s + splits, ... (k_gemm.cu's distributed reduction).
__device__ __forceinline__ void reduce_share(const ChainParams &p, const PairDesc &D, const Geo &g,
                                             const Unit &w, size_t part_int4) {
  const int nch = g.bn / 32;
  const int nb = g.tile_m() / 32 * nch;
  const int my_nb = (nb - w.s + g.splits - 1) / g.splits;
  const int et = threadIdx.x - 64;
  const int lane = et & 31, c = et >> 5;
  const int n = D.n[w.job];
  const int4 *tbase = reinterpret_cast<const int4 *>(p.ws) + (size_t)w.tile * g.splits * part_int4;
  for (int i = 0; i < my_nb; ++i) {
    const int b = w.s + i * g.splits;
    const int rb = b / nch, ch = b - rb * nch;
    const int row = w.m_t * g.tile_m() + rb * 32 + lane;
    const int col = w.n_t * g.bn + ch * 32 + 4 * c;
    const float xs = row < g.m ? __ldcg(D.s + row) : 0.0f;
    float wsc[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) wsc[e] = col + e < n ? __ldg(D.matsc[w.job] + col + e) : 0.0f;
    int4 acc = make_int4(0, 0, 0, 0);
    const size_t boff = (size_t)b * 256 + et;
    for (int sg = 0; sg < g.splits; sg += 4) {
      int4 v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        v[j] = sg + j < g.splits ? __ldcg(tbase + (size_t)(sg + j) * part_int4 + boff)
                                 : make_int4(0, 0, 0, 0);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc.x += v[j].x;
        acc.y += v[j].y;
        acc.z += v[j].z;
        acc.w += v[j].w;
      }
    }
    if (row >= g.m || col >= n) continue;
    const float4 o = make_float4(dequant(acc.x, xs, wsc[0]), dequant(acc.y, xs, wsc[1]),
                                 dequant(acc.z, xs, wsc[2]), dequant(acc.w, xs, wsc[3]));
    float *d = D.dst[w.job] + (size_t)row * D.dstr[w.job] + col;
    if (D.tma_store[w.job] && col + 3 < n) {
      *reinterpret_cast<float4 *>(d) = o;
    } else {
      d[0] = o.x;
      if (col + 1 < n) d[1] = o.y;
      if (col + 2 < n) d[2] = o.z;
      if (col + 3 < n) d[3] = o.w;
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1) k_chain(const __grid_constant__ ChainParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *ring = smem;
  uint8_t *epi = smem + kRingBytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kBarOff);
  uint64_t *full = bars;              // [kNB] stage landed
  uint64_t *empty = bars + kNB;       // [kNB] stage consumed by the MMAs
  uint64_t *tfull = bars + 2 * kNB;   // [2] accumulator slot ready
  uint64_t *tempty = tfull + 2;       // [2] accumulator slot drained
  uint64_t *mma_done = tempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
  int *s_last = reinterpret_cast<int *>(tmem_slot + 1);
  float *red = reinterpret_cast<float *>(tmem_slot + 4);  // [2][8]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const Fail fail{p.err, p.abort};

  if (threadIdx.x == 0) {
    for (int s = 0; s < kNB; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(&tfull[b], 1);
      ptx::mbar_init(&tempty[b], kEpiThreads);
    }
    ptx::mbar_init(mma_done, 1);
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, 512);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_a = ptx::policy_evict_last();
      const uint64_t pol_b = ptx::policy_evict_first();
      uint32_t head = 0;
      int it = 0, lo = 0;  // stages [lo, it) are issued and not yet known consumed
      prefetch_x_rows(p.pd[0]);
      // ring bookkeeping in shared memory (local memory would miss in the
      // small L1 this kernel leaves): stage offsets and sizes, and the A
      // coordinates of stages still waiting for their codes
      uint32_t *soff = reinterpret_cast<uint32_t *>(smem + kBarOff + 512);
      uint32_t *ssz = soff + kNB;
      int *pa_x = reinterpret_cast<int *>(ssz + kNB);
      int *pa_y = pa_x + kNB;
      bool ok = true;
      for (int pi = 0; pi < p.npairs && ok; ++pi) {
        const PairDesc &D = p.pd[pi];
        Geo g;
        g.load(D);
        const uint32_t S = g.stage_bytes(), AB = g.a_bytes();
        for (int j = 0; j < g.njobs; ++j) ptx::prefetch_tmap(&D.tmB[j]);
        ptx::prefetch_tmap(&D.tmA);
        bool dep = false;   // codes of pair pi published by every CTA
        int pend_lo = it;   // stages [pend_lo, it) wait for their A tile while !dep
        auto publish_wait = [&]() -> bool {
          if (!chain_wait(slot(p, 2 * pi), G, fail)) return false;
          fence_proxy_async_global();  // generic-proxy codes before async-proxy reads
          for (int j = pend_lo; j < it; ++j) {
            const int sl = j % kNB;
            ptx::tma_load_2d(&D.tmA, &full[sl], ring + soff[sl], pa_x[sl], pa_y[sl], pol_a);
          }
          return true;
        };
        for (int u = blockIdx.x; u < g.units && ok; u += G) {
          const Unit w = decode_unit(g, u);
          const int kb0 = w.s * g.kb_per_split;
          const int nk = min(kb0 + g.kb_per_split, g.kb_total) - kb0;
          const int rot = w.tile % nk;
          for (int i = 0; i < nk; ++i) {
            const int kb = kb0 + (rot + i) % nk;  // see k_rotation below
            uint32_t h2 = head;
            const uint32_t off = ring_place(h2, S);
            // free the stages this one would overwrite (and a barrier slot)
            while (lo < it) {
              bool clash = it - lo >= kNB;
              for (int j = lo; j < it && !clash; ++j) {
                const int sl = j % kNB;
                clash = off < soff[sl] + ssz[sl] && soff[sl] < off + S;
              }
              if (!clash) break;
              if (!dep && lo >= pend_lo) {  // the oldest stage still lacks its A tile
                if (!publish_wait()) {
                  ok = false;
                  break;
                }
                dep = true;
              }
              if (!bar_wait(&empty[lo % kNB], (lo / kNB) & 1, fail, DEV_TIMEOUT_EMPTY)) {
                ok = false;
                break;
              }
              ++lo;
            }
            if (!ok) break;
            head = h2;
            const int sl = it % kNB;
            soff[sl] = off;
            ssz[sl] = S;
            ptx::mbar_arrive_expect_tx(&full[sl], S);
            ptx::tma_load_2d(&D.tmB[w.job], &full[sl], ring + off + AB, kb * BK, w.n_t * g.bn, pol_b);
            if (dep) {
              ptx::tma_load_2d(&D.tmA, &full[sl], ring + off, kb * BK, w.m_t * g.tile_m(), pol_a);
            } else {
              pa_x[sl] = kb * BK;
              pa_y[sl] = w.m_t * g.tile_m();
            }
            ++it;
          }
        }
        if (!dep && ok) {
          if (it == pend_lo) dep = true;  // no tile of this pair here
          else if (publish_wait()) dep = true;
          else ok = false;
        }
        if (!dep) {
          // giving up: stages holding a B tile still need their A bytes so
          // that their barriers complete and the drain below sees them land
          for (int j = pend_lo; j < it; ++j) {
            const int sl = j % kNB;
            ptx::tma_load_2d(&D.tmA, &full[sl], ring + soff[sl], pa_x[sl], pa_y[sl], pol_a);
          }
          break;
        }
        // warm L2 with the next pair's activation rows and first weight tiles
        if (pi + 1 < p.npairs && ok) {
          prefetch_x_rows(p.pd[pi + 1]);
          Geo gn;
          gn.load(p.pd[pi + 1]);
          if ((int)blockIdx.x < gn.units) {
            const Unit w = decode_unit(gn, blockIdx.x);
            const int kb0 = w.s * gn.kb_per_split;
            const int nk = min(kb0 + gn.kb_per_split, gn.kb_total) - kb0;
            const int rot = w.tile % nk;
            const int kbn = min(nk, max(4, (64 * 1024) / (gn.bn * BK)));
            for (int i = 0; i < kbn; ++i)
              ptx::tma_prefetch_l2_2d(&p.pd[pi + 1].tmB[w.job], (kb0 + (rot + i) % nk) * BK,
                                      w.n_t * gn.bn);
          }
        }
      }
      // drain: every issued stage has landed before the CTA may exit
      for (int j = lo; j < it; ++j)
        ptx::mbar_wait(&full[j % kNB], (j / kNB) & 1, p.err, DEV_TIMEOUT_DRAIN);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t head = 0;
      int it = 0;
      int uses[2] = {0, 0};  // accumulator slot uses so far
      int nxt = 0;           // slot of the next narrow tile
      bool ok = true;
      for (int pi = 0; pi < p.npairs && ok; ++pi) {
        Geo g;
        g.load(p.pd[pi]);
        const uint32_t S = g.stage_bytes(), AB = g.a_bytes();
        const uint32_t idesc = ptx::idesc_i8(BM, g.bn);
        const bool wide = g.mb * g.bn > 256;
        const int nc = n_chains(g.mb, g.bn);
        for (int u = blockIdx.x; u < g.units && ok; u += G) {
          const Unit w = decode_unit(g, u);
          const int kb0 = w.s * g.kb_per_split;
          const int nk = min(kb0 + g.kb_per_split, g.kb_total) - kb0;
          int slot;
          if (wide) {  // the tile needs both 256-column slots
            slot = 0;
            if (!bar_wait(&tempty[0], (uses[0] & 1) ^ 1, fail, DEV_TIMEOUT_TMEM) ||
                !bar_wait(&tempty[1], (uses[1] & 1) ^ 1, fail, DEV_TIMEOUT_TMEM)) {
              ok = false;
              break;
            }
            ++uses[0];
            ++uses[1];
          } else {
            slot = nxt;
            nxt ^= 1;
            if (!bar_wait(&tempty[slot], (uses[slot] & 1) ^ 1, fail, DEV_TIMEOUT_TMEM)) {
              ok = false;
              break;
            }
            ++uses[slot];
          }
          ptx::tc_fence_after();
          const uint32_t d_tmem = tmem_base + (uint32_t)slot * 256u;
          for (int i = 0; i < nk; ++i, ++it) {
            const uint32_t off = ring_place(head, S);
            const int sl = it % kNB;
            if (!bar_wait(&full[sl], (it / kNB) & 1, fail, DEV_TIMEOUT_FULL)) {
              ok = false;
              break;
            }
            ptx::tc_fence_after();
            const uint32_t a0 = ptx::smem_u32(ring + off);
            const uint32_t b0 = ptx::smem_u32(ring + off + AB);
            if (g.mb == 1)
              mma_stage<1>(d_tmem, a0, b0, idesc, g.bn, nc, i == 0);
            else
              mma_stage<2>(d_tmem, a0, b0, idesc, g.bn, nc, i == 0);
            ptx::mma_commit(&empty[sl]);
          }
          if (!ok) break;
          ptx::mma_commit(&tfull[slot]);
        }
      }
      // every MMA of this CTA completes before TMEM may be freed
      ptx::mma_commit(mma_done);
      ptx::mbar_wait(mma_done, 0, p.err, DEV_TIMEOUT_DRAIN);
    }
  } else {
    // ------------------------------------------- quantize + GEMM epilogue
    const int et = threadIdx.x - 64;
    const int q = warp & 3;            // TMEM lane quarter this warp may read
    const int half = (warp - 2) >> 2;  // second warp of the quarter?
    uint8_t *stage = epi + (warp - 2) * kEpiStageBytes;
    int fills[2] = {0, 0};
    int nxt = 0;
    bool ok = true;
    for (int pi = 0; pi < p.npairs && ok; ++pi) {
      const PairDesc &D = p.pd[pi];
      Geo g;
      g.load(D);
      // 1. the previous pair's outputs are complete on every CTA
      if (pi > 0) {
        if (et == 0) *s_last = chain_wait(slot(p, 2 * pi - 1), G, fail) ? 1 : 0;
        ptx::named_bar_sync(1, kEpiThreads);
        if (!*s_last) {
          ok = false;
          break;
        }
      }
      // 2. quantize this CTA's rows of x_pi, then publish the codes
      quantize_rows(D, red);
      // publish: the CTA barrier orders every thread's stores before thread
      // 0's release at gpu scope (cumulative); the readers acquire, then
      // fence the async proxy before their TMA loads of the codes
      ptx::named_bar_sync(1, kEpiThreads);
      if (et == 0) red_release_add(slot(p, 2 * pi), 1);
      // the epilogue reads activation scales that other CTAs wrote: observe
      // their publication (long complete by the time a tile is ready)
      if ((int)blockIdx.x < g.units) {
        if (et == 0) *s_last = chain_wait(slot(p, 2 * pi), G, fail) ? 1 : 0;
        ptx::named_bar_sync(1, kEpiThreads);
        if (!*s_last) {
          ok = false;
          break;
        }
      }
      // 3. epilogue of this CTA's tiles
      const int mblk = g.mb == 2 ? half : 0;
      const int nch = g.bn / 32;
      const bool wide = g.mb * g.bn > 256;
      // this warp's 32-column chunks: all of them for two M blocks, every
      // other one when the quarter's two warps share the M block.  The chunk
      // loops stay rolled (one copy of the dequant and store code): unrolled,
      // the kernel outgrows the instruction cache and every phase slows down.
      const int ch0 = g.mb == 2 ? 0 : half;
      const int chs = g.mb == 2 ? 1 : 2;
      const int nc = n_chains(g.mb, g.bn);
      for (int u = blockIdx.x; u < g.units; u += G) {
        const Unit w = decode_unit(g, u);
        const int job = w.job;
        const int n = D.n[job];
        int slot;
        if (wide) {
          slot = 0;
        } else {
          slot = nxt;
          nxt ^= 1;
        }
        const int tile_row0 = w.m_t * g.tile_m() + mblk * BM + q * 32;
        const int row = tile_row0 + lane;
        const int n0 = w.n_t * g.bn;
        const float *wsc = D.matsc[job];
        auto ws_of = [&](int ch) {
          const int col = n0 + ch * 32 + lane;
          return ch < nch && col < n ? __ldg(wsc + col) : 0.0f;
        };
        // scales, fetched while the tile's MMAs run: the row's activation
        // scale (written by this launch: coherent load) and, in lane i, the
        // weight scale of column 32*ch + i of the first chunk (later ones one
        // chunk ahead)
        const float xs = row < g.m ? __ldcg(D.s + row) : 0.0f;
        float ws_cur = ws_of(ch0);
        if (!bar_wait(&tfull[slot], fills[slot] & 1, fail, DEV_TIMEOUT_TMEM, 100)) {
          ok = false;
          break;
        }
        ++fills[slot];
        ptx::tc_fence_after();
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)slot * 256u +
                               (uint32_t)(mblk * g.bn);
        if (g.splits == 1) {
#pragma unroll 1
          for (int ch = ch0; ch < nch; ch += chs) {
            const float ws_nxt = ws_of(ch + chs);
            __syncwarp();
            uint32_t r[32];
            tmem_ld_sum(taddr + ch * 32, g.bn, nc, r);
            const int col0 = n0 + ch * 32;
            if (col0 < n)
              emit_chunk(D, &D.tmD[job], job, reinterpret_cast<const int(&)[32]>(r), xs, ws_cur,
                         row, col0, lane, stage, tile_row0, g.m);
            ws_cur = ws_nxt;
          }
          ptx::tc_fence_before();
          ptx::mbar_arrive(&tempty[slot]);
          if (wide) ptx::mbar_arrive(&tempty[1]);
          continue;
        }
        // split K: this split's int32 partial, [M block][quarter][chunk][8 x int4][lane]
        const size_t part_int4 = (size_t)g.tile_m() * g.bn / 4;
        const size_t my_off = (size_t)(mblk * 4 + q) * nch * 8 * 32 + lane;
        int4 *part = reinterpret_cast<int4 *>(p.ws) + ((size_t)w.tile * g.splits + w.s) * part_int4 +
                     my_off;
#pragma unroll 1
        for (int ch = ch0; ch < nch; ch += chs) {
          __syncwarp();
          uint32_t r[32];
          tmem_ld_sum(taddr + ch * 32, g.bn, nc, r);
#pragma unroll
          for (int c = 0; c < 8; ++c)
            __stcg(part + (ch * 8 + c) * 32, make_int4(r[4 * c], r[4 * c + 1], r[4 * c + 2], r[4 * c + 3]));
        }
        ptx::tc_fence_before();
        ptx::mbar_arrive(&tempty[slot]);
        if (wide) ptx::mbar_arrive(&tempty[1]);
        __threadfence();
        ptx::named_bar_sync(1, kEpiThreads);
        if (g.dist) {
          // every split of the tile is resident: wait for all partials, then
          // each split reduces its share of the tile's 32x32 blocks
          if (et == 0) {
            atomicAdd(p.counters + w.tile, 1);
            *s_last = chain_wait(p.counters + w.tile, g.splits, fail, DEV_TIMEOUT_SPLIT) ? 1 : 0;
          }
          ptx::named_bar_sync(1, kEpiThreads);
          if (!*s_last) {
            ok = false;
            break;
          }
          reduce_share(p, D, g, w, part_int4);
          ptx::named_bar_sync(1, kEpiThreads);
          if (et == 0) {
            int *done = p.counters + g.tiles_m * g.tiles_n + w.tile;
            if (atomicAdd(done, 1) == g.splits - 1) {  // last reader resets both counters
              p.counters[w.tile] = 0;
              *done = 0;
            }
          }
          continue;
        }
        if (et == 0) *s_last = (atomicAdd(p.counters + w.tile, 1) == g.splits - 1);
        ptx::named_bar_sync(1, kEpiThreads);
        if (*s_last) {
          // the last split to finish sums every partial (exact integer adds)
          __threadfence();
          const int4 *base =
              reinterpret_cast<const int4 *>(p.ws) + (size_t)w.tile * g.splits * part_int4 + my_off;
#pragma unroll 1
          for (int ch = ch0; ch < nch; ch += chs) {
            const int col0 = n0 + ch * 32;
            if (col0 >= n) continue;
            const float ws_ch = ws_of(ch);
            int acc[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[i] = 0;
            for (int s = 0; s < g.splits; ++s) {
              const int4 *src = base + (size_t)s * part_int4 + ch * 8 * 32;
#pragma unroll
              for (int c = 0; c < 8; ++c) {
                const int4 v = __ldcg(src + c * 32);
                acc[4 * c] += v.x;
                acc[4 * c + 1] += v.y;
                acc[4 * c + 2] += v.z;
                acc[4 * c + 3] += v.w;
              }
            }
            __syncwarp();
            emit_chunk(D, &D.tmD[job], job, acc, xs, ws_ch, row, col0, lane, stage, tile_row0, g.m);
          }
          ptx::named_bar_sync(1, kEpiThreads);
          if (et == 0) p.counters[w.tile] = 0;  // ready for the next pair or launch
        }
      }
      if (!ok) break;
      // 4. this CTA's outputs of pair pi are written: publish (the TMA
      // stores complete, ordered before the generic release by a proxy fence)
      if (lane == 0) {
        ptx::bulk_wait<0>();
        fence_proxy_async_global();
      }
      __syncwarp();
      ptx::named_bar_sync(1, kEpiThreads);
      if (et == 0) red_release_add(slot(p, 2 * pi + 1), 1);
    }
    if (lane == 0) ptx::bulk_wait<0>();
    __syncwarp();
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, 512);
  }
  // the last CTA out resets the hand-off counters for the next launch (every
  // CTA has finished all of its waits before it counts itself out)
  if (threadIdx.x == 0) {
    __threadfence();
    int *exits = slot(p, 2 * p.npairs);
    if (atomicAdd(exits, 1) == G - 1) {
      for (int i = 0; i < 2 * p.npairs; ++i) *slot(p, i) = 0;
      *p.abort = 0;
      __threadfence();
      *exits = 0;
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct Chain {
  int device = -1;
  int npairs = 0;
  std::vector<PairDesc> h;  // descriptors (they go into each launch's parameters)
  int *d_sync = nullptr;
  int32_t *d_ws = nullptr;
  int *d_cnt = nullptr;
  std::vector<int> plan;  // bn, mb, splits per pair
};
std::mutex g_chain_mu;
std::map<int, Chain> g_chains;
int g_next_chain = 1;

void free_chain(Chain &c) {
  if (c.d_sync) cudaFree(c.d_sync);
  if (c.d_ws) cudaFree(c.d_ws);
  if (c.d_cnt) cudaFree(c.d_cnt);
  c = Chain{};
}

int set_smem_attr(int dev) {
  static std::mutex mu;
  static uint64_t done = 0;
  std::lock_guard<std::mutex> lk(mu);
  if (!(done & (1ull << (dev & 63)))) {
    GCU_CUDA(cudaFuncSetAttribute(k_chain, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    done |= 1ull << (dev & 63);
  }
  return 0;
}

int build_pair(const gcu_qgemm_step &st, int idx, int sms, const int *force, PairDesc &D,
               size_t &ws_need, int &cnt_need) {
  memset(&D, 0, sizeof(D));
  const int m = st.m, k = st.k;
  if (m < 1 || k < 16 || k % 16 != 0)
    return set_error("gemm chain step %d: needs m >= 1 and k a multiple of 16 (m %d, k %d)", idx, m, k);
  if (st.njobs < 1 || st.njobs > kJobs)
    return set_error("gemm chain step %d: 1..%d weights (got %d)", idx, kJobs, st.njobs);
  const long xstr = st.xstr ? st.xstr : k;
  if (!st.x || !st.q || !st.s || xstr < k || xstr % 4 || (uintptr_t)st.x % 16 ||
      (uintptr_t)st.q % 16 || (uintptr_t)st.s % 4)
    return set_error("gemm chain step %d: x, q, s must be device pointers with 16-byte aligned "
                     "rows (x row stride %ld floats)", idx, xstr);
  int ns[kJobs];
  for (int j = 0; j < st.njobs; ++j) {
    const gcu_gemv_job &J = st.jobs[j];
    if (!J.w || !J.sc || !J.dst || J.m < 1 || (uintptr_t)J.w % 16)
      return set_error("gemm chain step %d job %d: bad weight (rows %d)", idx, j, J.m);
    ns[j] = J.m;
  }
  int bn, mb, splits;
  if (force && force[0] > 0) {
    bn = force[0];
    mb = force[1] > 0 ? force[1] : 1;
    splits = force[2];
    if (!((mb == 1 && (bn == 64 || bn == 128 || bn == 256)) ||
          (mb == 2 && (bn == 128 || bn == 192 || bn == 256))))
      return set_error("gemm chain step %d: no %d x %d tile", idx, 128 * mb, bn);
  } else if (gemm_plan_one_cta(m, k, ns, st.njobs, sms, &bn, &mb, &splits)) {
    return 1;
  }
  const int tile_m = BM * mb;
  const int kb_total = (k + BK - 1) / BK;
  const int tiles_m = (m + tile_m - 1) / tile_m;
  int tn = 0;
  for (int j = 0; j < st.njobs; ++j) {
    D.tn_begin[j] = tn;
    tn += (ns[j] + bn - 1) / bn;
  }
  const int tiles = tiles_m * tn;
  if (splits <= 0) splits = gemm_split_for(tiles, k, sms);
  if (splits > kb_total) splits = kb_total;
  const int kb_per = (kb_total + splits - 1) / splits;
  splits = (kb_total + kb_per - 1) / kb_per;
  if (gemm_tmap_i8(&D.tmA, st.q, k, m, k, tile_m)) return 1;
  for (int j = 0; j < st.njobs; ++j) {
    const gcu_gemv_job &J = st.jobs[j];
    if (gemm_tmap_i8(&D.tmB[j], static_cast<const int8_t *>(J.w), k, ns[j], k, bn)) return 1;
    D.tma_store[j] = (uintptr_t)J.dst % 16 == 0 && ns[j] % 4 == 0;
    if (D.tma_store[j] && gemm_tmap_f32(&D.tmD[j], J.dst, ns[j], m, ns[j])) return 1;
    D.matsc[j] = J.sc;
    D.dst[j] = J.dst;
    D.dstr[j] = ns[j];
    D.n[j] = ns[j];
  }
  D.x = st.x;
  D.xstr = xstr;
  D.q = st.q;
  D.s = st.s;
  D.njobs = st.njobs;
  D.m = m;
  D.k = k;
  D.bn = bn;
  D.mb = mb;
  D.splits = splits;
  D.tiles_m = tiles_m;
  D.tiles_n = tn;
  D.kb_total = kb_total;
  D.kb_per_split = kb_per;
  D.units = tiles * splits;
  D.dist = splits > 1 && D.units <= sms;
  // The rows are latency-bound: at most 16 float4 per lane, and as many
  // warps per row as still leave a warp group for every row (all 8 warps of
  // every CTA loading).
  const int k4 = k / 4;
  int wpr = 1;
  while (wpr < 8 && (k4 > 32 * kMaxVpt * wpr ||
                     ((long)sms * (kEpiWarps / (2 * wpr)) >= m && k4 > 32 * 2 * wpr)))
    wpr *= 2;
  const int vpt = (k4 + 32 * wpr - 1) / (32 * wpr);
  if (vpt > kMaxVpt)
    return set_error("gemm chain step %d: k %d exceeds %d", idx, k, 32 * 8 * kMaxVpt * 4);
  D.wpr = wpr;
  D.vpt = vpt;
  if (splits > 1) {
    const size_t need = (size_t)tiles * splits * tile_m * bn * sizeof(int32_t);
    if (need > ws_need) ws_need = need;
    if (2 * tiles > cnt_need) cnt_need = 2 * tiles;
  }
  return 0;
}

}  // namespace
}  // namespace gcu

using namespace gcu;

#define GCU_EXPORT extern "C" __attribute__((visibility("default")))

GCU_EXPORT int gcu_gemm_chain_create(const gcu_qgemm_step *steps, int nsteps, const int *force,
                                     int *handle) {
  if (!handle) return set_error("gemm chain: null handle");
  *handle = 0;
  if (!steps || nsteps < 1) return set_error("gemm chain: no steps");
  const int dev = calling_device();
  GCU_CUDA(cudaSetDevice(dev));
  int coop = 0;
  GCU_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev));
  if (!coop) return set_error("gemm chain: device %d has no cooperative launch", dev);
  const int sms = num_sms();
  std::vector<PairDesc> h(nsteps);
  size_t ws_need = 0;
  int cnt_need = 0;
  Chain c;
  c.device = dev;
  c.npairs = nsteps;
  for (int i = 0; i < nsteps; ++i) {
    if (build_pair(steps[i], i, sms, force ? force + 3 * i : nullptr, h[i], ws_need, cnt_need)) return 1;
    c.plan.push_back(h[i].bn);
    c.plan.push_back(h[i].mb);
    c.plan.push_back(h[i].splits);
  }
  c.h = h;
  // [2 per step of a launch][exits], kSyncStride ints apart; then the abort word
  const int nsync = (2 * kParamPairs + 1) * kSyncStride + 1;
  cudaError_t e = cudaMalloc(&c.d_sync, sizeof(int) * nsync);
  if (e == cudaSuccess && ws_need) e = cudaMalloc(&c.d_ws, ws_need);
  if (e == cudaSuccess && cnt_need) e = cudaMalloc(&c.d_cnt, sizeof(int) * cnt_need);
  if (e == cudaSuccess) e = cudaMemset(c.d_sync, 0, sizeof(int) * nsync);
  if (e == cudaSuccess && cnt_need) e = cudaMemset(c.d_cnt, 0, sizeof(int) * cnt_need);
  if (e != cudaSuccess) {
    free_chain(c);
    return check_cuda(e, "gemm chain: device buffers");
  }
  if (set_smem_attr(dev)) {
    free_chain(c);
    return 1;
  }
  std::lock_guard<std::mutex> lk(g_chain_mu);
  *handle = g_next_chain++;
  g_chains[*handle] = std::move(c);
  return 0;
}

GCU_EXPORT int gcu_gemm_chain_run(int handle, void *stream) {
  // the launch parameters are built under the lock (the handle stays valid)
  static thread_local ChainParams p;
  std::lock_guard<std::mutex> lk(g_chain_mu);
  auto it = g_chains.find(handle);
  if (it == g_chains.end()) return set_error("gemm chain: unknown handle %d", handle);
  const Chain &c = it->second;
  if (c.device != calling_device())
    return set_error("gemm chain: handle %d belongs to device %d", handle, c.device);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms());
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // launches of at most kParamPairs steps, in order on the stream; the
  // hand-off counters are reset by each launch's last CTA, so they share them
  for (int b = 0; b < c.npairs; b += kParamPairs) {
    const int n = c.npairs - b < kParamPairs ? c.npairs - b : kParamPairs;
    memset(&p, 0, sizeof(p));
    for (int i = 0; i < n; ++i) p.pd[i] = c.h[b + i];
    p.npairs = n;
    p.sync = c.d_sync;
    p.ws = c.d_ws;
    p.counters = c.d_cnt;
    p.err = dev_error_word();
    p.abort = c.d_sync + (2 * kParamPairs + 1) * kSyncStride;
    GCU_CUDA(cudaLaunchKernelEx(&cfg, k_chain, p));
  }
  GCU_CUDA(cudaGetLastError());
  return 0;
}

GCU_EXPORT int gcu_gemm_chain_plan(int handle, int *plan, int nsteps) {
  std::lock_guard<std::mutex> lk(g_chain_mu);
  auto it = g_chains.find(handle);
  if (it == g_chains.end()) return set_error("gemm chain: unknown handle %d", handle);
  if (nsteps != it->second.npairs)
    return set_error("gemm chain: handle %d has %d steps", handle, it->second.npairs);
  for (int i = 0; i < 3 * nsteps; ++i) plan[i] = it->second.plan[i];
  return 0;
}

GCU_EXPORT int gcu_gemm_chain_destroy(int handle) {
  Chain c;
  {
    std::lock_guard<std::mutex> lk(g_chain_mu);
    auto it = g_chains.find(handle);
    if (it == g_chains.end()) return set_error("gemm chain: unknown handle %d", handle);
    c = std::move(it->second);
    g_chains.erase(it);
  }
  const int dev = c.device;
  int cur = -1;
  cudaGetDevice(&cur);
  if (cur != dev) cudaSetDevice(dev);
  free_chain(c);
  if (cur >= 0 && cur != dev) cudaSetDevice(cur);
  return 0;
}
