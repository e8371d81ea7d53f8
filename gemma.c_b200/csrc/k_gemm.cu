// k_gemm.cu -- K3: int8 NT GEMM on the 5th-generation tensor cores.
//
// Device restatement of gemm_int8 (gemma.c:3937-4054):
//   dst[i*dstr + j] = (float)(sum_l src[i,l] * mat[j,l]) * (ssc[i] * matsc[j])
// The int32 sums are exact, so the tiling, the split of K and the order of
// accumulation cannot change a bit; the epilogue is the reference -ffast-math
// build's (float)acc * (xs*ws) with round-to-nearest multiplies.
//
// Design (one CTA per SM, persistent over work units).  A CTA tile is
// (128*MB) x BN outputs, MB in {1, 2}: with MB = 2 every B stage feeds two
// M=128 MMAs, which halves the operand bytes each SM pulls per output --
// the limit for the small-M (prefill) shapes, whose A/B panels are re-read
// from L2 by every tile.
//   warp 0      TMA producer: 128-byte-swizzled A ((128*MB) x 128 B) and B
//               (BN x 128 B) tiles into a STAGES-deep shared-memory ring
//   warp 1      allocates TMEM, issues tcgen05.mma.cta_group::1.kind::i8
//               (M=128, N=BN, K=32) from one thread, commits stage releases
//   warps 2-9   epilogue, two warps per TMEM lane quarter: tcgen05.ld the
//               int32 accumulators (two TMEM buffers when they fit, so the
//               next tile's MMAs overlap this epilogue), dequantize, stage
//               through swizzled shared memory and TMA-store fp32 rows; or,
//               when K is split, write int32 partials and let the last split
//               of a tile reduce them
// Every TMA load reads this GPU's own memory into the CTA that issues it.
// Every wait is bounded (globaltimer); on timeout the kernel records an error
// code, drains its copies, frees TMEM and returns.
#include "gcu_internal.cuh"

#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

namespace gcu {
namespace {

constexpr int BM = 128;
constexpr int BK = 128;  // K bytes per stage (one 128-byte swizzle row)
constexpr int kEpiWarps = 8;  // two per TMEM lane quarter, each half the chunks
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kThreads = 64 + kEpiThreads;
constexpr int kMaxJobs = 4;
constexpr int kEpiStageBytes = 32 * 128;  // 32 rows x 32 fp32

constexpr int kSmemMax = 232448;  // opt-in shared memory per CTA on sm_100
constexpr int kPrefetchBytes = 256 * 1024;  // B bytes a CTA warms in L2 before its wait

__host__ __device__ constexpr int pow2_at_least(int v) {
  int p = 32;
  while (p < v) p <<= 1;
  return p;
}

// A stage holds KG consecutive 128-byte K blocks under one pair of
// barriers: the MMA issuer's wait on a landed stage and its commit cost a
// few hundred cycles apiece, so tiles small enough to keep three double
// stages resident take two K blocks per stage.
template <int BN, int MB>
struct Cfg {
  static constexpr int TILE_M = BM * MB;
  static constexpr int A_BYTES = TILE_M * BK;  // one K block
  static constexpr int B_BYTES = BN * BK;
  static constexpr int ACC_COLS = MB * BN;  // TMEM columns of one tile
  static constexpr int NBUF = 2 * ACC_COLS <= 512 ? 2 : 1;
  static constexpr int TMEM_COLS = pow2_at_least(NBUF * ACC_COLS);
  static constexpr int EPI_BYTES = kEpiWarps * kEpiStageBytes;
  static constexpr int FIXED = 1024 + EPI_BYTES + 512;
  static constexpr int KG = (kSmemMax - FIXED) / (2 * (A_BYTES + B_BYTES)) >= 3 ? 2 : 1;
  static constexpr int STAGE_BYTES = KG * (A_BYTES + B_BYTES);
  static constexpr int STAGES_FIT = (kSmemMax - FIXED) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int EPI_OFF = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = EPI_OFF + EPI_BYTES;
  static constexpr int NBARS = 2 * STAGES + 5;
  static constexpr int SMEM = 1024 + BAR_OFF + NBARS * 8 + 16;
  static_assert(STAGES >= 2, "tile too large for shared memory");
  static_assert(SMEM + 64 <= kSmemMax, "shared memory budget");
  static_assert(ACC_COLS <= 512 && BN % 32 == 0 && BN <= 256, "tile shape");
};

// A CTA pair (thread-block cluster of two) computes a 256 x BN tile with
// tcgen05.mma.cta_group::2: CTA r of the pair holds A rows [128r, 128r+128)
// and B rows [r*BN/2, (r+1)*BN/2) of every stage, and its TMEM holds the
// accumulator of its 128 rows x all BN columns.  Per output, each SM pulls
// a third less operand data than a one-CTA 128 x BN tile, and a 128 x BN
// accumulator leaves room for two TMEM buffers.
constexpr int kPairMB = 4;  // Plan::mb value of the pair kernel

template <int BN>
struct PairCfg {
  static constexpr int BH = BN / 2;  // B rows per CTA
  static constexpr int TILE_M = 2 * BM;
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BH * BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int ACC_COLS = BN;
  static constexpr int NBUF = 2 * ACC_COLS <= 512 ? 2 : 1;
  static constexpr int TMEM_COLS = pow2_at_least(NBUF * ACC_COLS);
  static constexpr int EPI_BYTES = kEpiWarps * kEpiStageBytes;
  static constexpr int FIXED = 1024 + EPI_BYTES + 512;
  static constexpr int STAGES_FIT = (kSmemMax - FIXED) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int EPI_OFF = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = EPI_OFF + EPI_BYTES;
  static constexpr int NBARS = 3 * STAGES + 5;
  static constexpr int SMEM = 1024 + BAR_OFF + NBARS * 8 + 16;
  static_assert(STAGES >= 2, "tile too large for shared memory");
  static_assert(SMEM + 64 <= kSmemMax, "shared memory budget");
  static_assert(BH % 8 == 0 && BN <= 256 && BN % 32 == 0, "pair tile shape");
};

struct alignas(64) TcJob {
  CUtensorMap tmB;  // weights [n][k] int8, box BN x 128
  CUtensorMap tmD;  // output [m][n] fp32 (row stride dstr), box 32 x 32
  const float *matsc;
  float *dst;
  long dstr;
  int n;
  int tn_begin;  // first global n-tile of this job
  int tma_store;
};

struct alignas(64) TcParams {
  CUtensorMap tmA;  // activations [m][k] int8, box 128 x 128
  TcJob jobs[kMaxJobs];
  int njobs;
  int m, k;
  int tiles_m, tiles_n, splits, kb_total, kb_per_split, units;
  const float *ssc;
  int32_t *ws;    // split-K partials [tile][split][TILE_M][BN]
  int *counters;  // split-K counters: arrivals [tile], then finished reductions [tile]
  int dist;       // split-K with every unit in one wave: the splits share the reduction
  unsigned int *err;
};

__device__ __forceinline__ float dequant(int acc, float xs, float ws) {
  return __fmul_rn(__int2float_rn(acc), __fmul_rn(xs, ws));
}

struct Unit {
  int m_t, s, job, n_t, tile;
};

__device__ __forceinline__ Unit decode_unit(const TcParams &p, int u) {
  Unit w;
  w.m_t = u % p.tiles_m;
  const int rest = u / p.tiles_m;
  w.s = rest % p.splits;
  const int ntg = rest / p.splits;
  int j = 0;
#pragma unroll
  for (int t = 1; t < kMaxJobs; ++t)
    if (t < p.njobs && ntg >= p.jobs[t].tn_begin) j = t;
  w.job = j;
  w.n_t = ntg - p.jobs[j].tn_begin;
  w.tile = w.m_t * p.tiles_n + ntg;
  return w;
}

// Dequantize 32 accumulators of one row and write them: either into the
// warp's swizzled staging buffer for a TMA store, or straight to global.
// Lane i of the warp holds the weight scale of column col0 + i in `ws_lane`
// (loaded before the accumulator was ready); shuffles broadcast it.
template <bool TMA, bool RAW = false>
__device__ __forceinline__ void emit_chunk(const TcParams &p, const TcJob &job, const int (&acc)[32],
                                           float xs, float ws_lane, int row, int col0, int lane,
                                           uint8_t *stage, int tile_row0) {
  float out[32];
#pragma unroll
  for (int i = 0; i < 32; ++i)
    out[i] = dequant(acc[i], xs, __shfl_sync(0xffffffffu, ws_lane, i));
  if (RAW) {  // the int32 sums themselves, as their bit patterns
#pragma unroll
    for (int i = 0; i < 32; ++i) out[i] = __int_as_float(acc[i]);
  }
  if (TMA) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float4 v = make_float4(out[4 * c], out[4 * c + 1], out[4 * c + 2], out[4 * c + 3]);
      *reinterpret_cast<float4 *>(stage + lane * 128 + ((c ^ (lane & 7)) << 4)) = v;
    }
    ptx::fence_proxy_async_smem();
    __syncwarp();
    // boxes starting below the last row (M tail) hold nothing to store
    if (lane == 0 && tile_row0 < p.m) {
      ptx::tma_store_2d(&job.tmD, stage, col0, tile_row0);
      ptx::bulk_commit();
    }
  } else {
    if (row < p.m) {
      float *d = job.dst + (size_t)row * job.dstr;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col0 + i < job.n) d[col0 + i] = out[i];
    }
  }
}

// Distributed split-K reduction, run by the 256 epilogue threads of split
// w.s once every split of tile w.tile has written its int32 partial.  The
// tile's 32x32 blocks b = w.s, w.s + splits, ... are this split's share;
// partials use the writer's layout [row block][chunk][8 x int4][lane], so
// thread `et` sums int4 `et` of a block (row 32*rb + lane, columns
// 32*ch + 4*(et/32) ...) across the splits and stores its four fp32 outputs
// directly.  Up to four blocks per round and four splits per load batch: at
// most 16 int4 loads in flight per thread.
struct ShareScales {
  float xs[4];
  float ws[4][4];
};

template <typename C, int BN, bool RAW = false>
__device__ __forceinline__ void share_scales(const TcParams &p, const TcJob &job, const Unit &w,
                                             int r0, int my_nb, ShareScales &sc) {
  constexpr int NCH = BN / 32;
  const int et = threadIdx.x - 64;
  const int lane = et & 31, c = et >> 5;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int b = w.s + (r0 + i) * p.splits;
    const int rb = b / NCH, ch = b - rb * NCH;
    const int row = w.m_t * C::TILE_M + rb * 32 + lane;
    const int col = w.n_t * BN + ch * 32 + 4 * c;
    const bool ok = r0 + i < my_nb;
    sc.xs[i] = ok && !RAW && row < p.m ? __ldg(p.ssc + row) : 0.0f;
#pragma unroll
    for (int e = 0; e < 4; ++e)
      sc.ws[i][e] = ok && !RAW && col + e < job.n ? __ldg(job.matsc + col + e) : 0.0f;
  }
}

template <typename C, int BN, bool RAW = false>
__device__ __forceinline__ void reduce_share(const TcParams &p, const TcJob &job, const Unit &w,
                                             size_t part_int4, int my_nb, ShareScales &sc) {
  constexpr int NCH = BN / 32;
  const int et = threadIdx.x - 64;
  const int lane = et & 31, c = et >> 5;
  const int4 *tbase = reinterpret_cast<const int4 *>(p.ws) + (size_t)w.tile * p.splits * part_int4;
  for (int r0 = 0; r0 < my_nb; r0 += 4) {
    if (r0 > 0) share_scales<C, BN, RAW>(p, job, w, r0, my_nb, sc);
    int4 acc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] = make_int4(0, 0, 0, 0);
    for (int sg = 0; sg < p.splits; sg += 4) {
      int4 v[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const size_t boff = (size_t)(w.s + (r0 + i) * p.splits) * 256 + et;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          v[i][j] = (r0 + i < my_nb && sg + j < p.splits)
                        ? __ldcg(tbase + (size_t)(sg + j) * part_int4 + boff)
                        : make_int4(0, 0, 0, 0);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[i].x += v[i][j].x;
          acc[i].y += v[i][j].y;
          acc[i].z += v[i][j].z;
          acc[i].w += v[i][j].w;
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (r0 + i >= my_nb) break;
      const int b = w.s + (r0 + i) * p.splits;
      const int rb = b / NCH, ch = b - rb * NCH;
      const int row = w.m_t * C::TILE_M + rb * 32 + lane;
      const int col = w.n_t * BN + ch * 32 + 4 * c;
      if (row >= p.m || col >= job.n) continue;
      const float4 o = RAW ? make_float4(__int_as_float(acc[i].x), __int_as_float(acc[i].y),
                                             __int_as_float(acc[i].z), __int_as_float(acc[i].w))
                               : make_float4(dequant(acc[i].x, sc.xs[i], sc.ws[i][0]),
                                             dequant(acc[i].y, sc.xs[i], sc.ws[i][1]),
                                             dequant(acc[i].z, sc.xs[i], sc.ws[i][2]),
                                             dequant(acc[i].w, sc.xs[i], sc.ws[i][3]));
      float *d = job.dst + (size_t)row * job.dstr + col;
      if (job.tma_store && col + 3 < job.n) {  // 16-byte aligned rows
        *reinterpret_cast<float4 *>(d) = o;
      } else {
        d[0] = o.x;
        if (col + 1 < job.n) d[1] = o.y;
        if (col + 2 < job.n) d[2] = o.z;
        if (col + 3 < job.n) d[3] = o.w;
      }
    }
  }
}

template <int BN, int MB, bool RAW = false>
__global__ void __launch_bounds__(kThreads, 1) k_gemm_i8_tc(const __grid_constant__ TcParams p) {
  using C = Cfg<BN, MB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *smA = smem;
  uint8_t *smB = smem + C::STAGES * C::KG * C::A_BYTES;
  uint8_t *epi = smem + C::EPI_OFF;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
  uint64_t *full = bars;
  uint64_t *empty = bars + C::STAGES;
  uint64_t *tfull = bars + 2 * C::STAGES;
  uint64_t *tempty = tfull + 2;
  uint64_t *mma_done = tempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
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
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&p.tmA);
    for (int j = 0; j < p.njobs; ++j) {
      ptx::prefetch_tmap(&p.jobs[j].tmB);
      if (p.jobs[j].tma_store) ptx::prefetch_tmap(&p.jobs[j].tmD);
    }
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, C::TMEM_COLS);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // The weights do not depend on the previous kernel on the stream: warm L2
  // with this CTA's first B tiles while that kernel finishes.  An L2 prefetch
  // brings nothing into the CTA, and L2 is where every write to device memory
  // lands, so it cannot expose a stale value.
  Unit w_first{};
  if (warp == 0 && lane == 0 && (int)blockIdx.x < p.units) {
    w_first = decode_unit(p, blockIdx.x);
    const int kb0 = w_first.s * p.kb_per_split;
    const int kb1 = min(kb0 + p.kb_per_split, p.kb_total);
    const int kbn = min(kb1 - kb0, max(C::STAGES, kPrefetchBytes / C::B_BYTES));
    for (int kb = kb0; kb < kb0 + kbn; ++kb)
      ptx::tma_prefetch_l2_2d(&p.jobs[w_first.job].tmB, kb * BK, w_first.n_t * BN);
  }
  // everything above overlapped the previous kernel; global memory from here
  ptx::griddep_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_a = ptx::policy_evict_last();
      const uint64_t pol_b = ptx::policy_evict_first();
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
        const Unit w = u == (int)blockIdx.x ? w_first : decode_unit(p, u);
        const int kb0 = w.s * p.kb_per_split;
        const int kb1 = min(kb0 + p.kb_per_split, p.kb_total);
        for (int kb = kb0; kb < kb1; kb += C::KG, ++it) {
          const int st = it % C::STAGES;
          const uint32_t round = it / C::STAGES;
          const int nk = min(C::KG, kb1 - kb);  // K blocks in this stage
          if (!ptx::mbar_wait(&empty[st], (round & 1) ^ 1, p.err, DEV_TIMEOUT_EMPTY)) {
            ok = false;
            break;
          }
          ptx::mbar_arrive_expect_tx(&full[st], (uint32_t)nk * (C::A_BYTES + C::B_BYTES));
#pragma unroll
          for (int g = 0; g < C::KG; ++g) {
            if (g >= nk) break;
            ptx::tma_load_2d(&p.tmA, &full[st], smA + (st * C::KG + g) * C::A_BYTES, (kb + g) * BK,
                             w.m_t * C::TILE_M, pol_a);
            ptx::tma_load_2d(&p.jobs[w.job].tmB, &full[st], smB + (st * C::KG + g) * C::B_BYTES,
                             (kb + g) * BK, w.n_t * BN, pol_b);
          }
        }
      }
      // drain: the last load issued into each stage must have landed before
      // the CTA may exit (immediate in normal operation)
      for (int d = 1; d <= C::STAGES && d <= it; ++d) {
        const int j = it - d;
        ptx::mbar_wait(&full[j % C::STAGES], (j / C::STAGES) & 1, p.err, DEV_TIMEOUT_DRAIN);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = ptx::idesc_i8(BM, BN);
      int it = 0, t = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++t) {
        const Unit w = decode_unit(p, u);
        const int kb0 = w.s * p.kb_per_split;
        const int kb1 = min(kb0 + p.kb_per_split, p.kb_total);
        const int buf = t % C::NBUF;
        const uint32_t use = t / C::NBUF;
        if (!ptx::mbar_wait(&tempty[buf], (use & 1) ^ 1, p.err, DEV_TIMEOUT_TMEM)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * C::ACC_COLS;
        for (int kb = kb0; kb < kb1; kb += C::KG, ++it) {
          const int st = it % C::STAGES;
          const uint32_t round = it / C::STAGES;
          const int nk = min(C::KG, kb1 - kb);
          if (!ptx::mbar_wait(&full[st], round & 1, p.err, DEV_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
#pragma unroll
          for (int g = 0; g < C::KG; ++g) {
            if (g >= nk) break;
            const uint32_t a0 = ptx::smem_u32(smA + (st * C::KG + g) * C::A_BYTES);
            const uint32_t b0 = ptx::smem_u32(smB + (st * C::KG + g) * C::B_BYTES);
#pragma unroll
            for (int j = 0; j < BK / 32; ++j)
#pragma unroll
              for (int mb = 0; mb < MB; ++mb)  // M block mb: A rows 128*mb.., TMEM columns BN*mb..
                ptx::mma_i8(d_tmem + mb * BN, ptx::smem_desc_k128(a0 + mb * BM * BK + 32 * j),
                            ptx::smem_desc_k128(b0 + 32 * j), idesc, (kb + g > kb0 || j > 0) ? 1u : 0u);
          }
          ptx::mma_commit(&empty[st]);
        }
        ptx::mma_commit(&tfull[buf]);
      }
      // the next kernel may start its prologue while our epilogue drains
      ptx::griddep_launch();
      // all MMAs of this CTA complete before TMEM may be freed
      ptx::mma_commit(mma_done);
      ptx::mbar_wait(mma_done, 0, p.err, DEV_TIMEOUT_DRAIN);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;  // second warp of the quarter?
    // MB == 2: the two warps of a quarter take one M block each, all chunks;
    // MB == 1: they share the M block and take alternate chunks
    const int mblk = MB == 2 ? half : 0;
    uint8_t *stage = epi + (warp - 2) * kEpiStageBytes;
    constexpr int NCH = BN / 32;  // 32-column chunks per tile
    auto mine = [&](int ch) { return MB == 2 || (ch & 1) == half; };
    int t = 0;
    for (int u = blockIdx.x; u < p.units; u += gridDim.x, ++t) {
      const Unit w = decode_unit(p, u);
      const TcJob &job = p.jobs[w.job];
      const int buf = t % C::NBUF;
      const uint32_t use = t / C::NBUF;
      const int tile_row0 = w.m_t * C::TILE_M + mblk * BM + q * 32;
      const int row = tile_row0 + lane;
      const int n0 = w.n_t * BN;
      // operand scales of this tile, fetched while its MMAs still run: the
      // row's activation scale, and lane i holds column (32*ch + i)'s weight
      // scale for chunk ch
      const float xs = !RAW && row < p.m ? __ldg(p.ssc + row) : 0.0f;
      float wsl[NCH];
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
        const int col = n0 + ch * 32 + lane;
        wsl[ch] = !RAW && col < job.n ? __ldg(job.matsc + col) : 0.0f;
      }
      if (!ptx::mbar_wait(&tfull[buf], use & 1, p.err, DEV_TIMEOUT_TMEM)) break;
      ptx::tc_fence_after();
      const uint32_t taddr =
          tmem_base + ((uint32_t)(q * 32) << 16) + buf * C::ACC_COLS + mblk * BN;
      if (p.splits == 1) {
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch) {
          if (!mine(ch)) continue;
          __syncwarp();
          uint32_t r[32];
          ptx::tmem_ld_32x32(taddr + ch * 32, r);
          ptx::tmem_ld_wait();
          const int col0 = n0 + ch * 32;
          if (col0 >= job.n) continue;
          if (job.tma_store) {
            if (lane == 0) ptx::bulk_wait_read<0>();
            __syncwarp();
            emit_chunk<true, RAW>(p, job, reinterpret_cast<const int(&)[32]>(r), xs, wsl[ch], row, col0,
                             lane, stage, tile_row0);
          } else {
            emit_chunk<false, RAW>(p, job, reinterpret_cast<const int(&)[32]>(r), xs, wsl[ch], row, col0,
                              lane, nullptr, tile_row0);
          }
        }
        ptx::tc_fence_before();
        ptx::mbar_arrive(&tempty[buf]);
      } else {
        // split K: this split's int32 partial goes to the workspace in a
        // layout where each warp store is 512 contiguous bytes:
        // [M block][quarter q][chunk][8 x int4][lane]
        constexpr size_t kPartInt4 = (size_t)C::TILE_M * BN / 4;
        const size_t my_off = (size_t)(mblk * 4 + q) * NCH * 8 * 32 + lane;
        int4 *part = reinterpret_cast<int4 *>(p.ws) + ((size_t)w.tile * p.splits + w.s) * kPartInt4 +
                     my_off;
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch) {
          if (!mine(ch)) continue;
          __syncwarp();
          uint32_t r[32];
          ptx::tmem_ld_32x32(taddr + ch * 32, r);
          ptx::tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 8; ++c)
            __stcg(part + (ch * 8 + c) * 32,
                   make_int4(r[4 * c], r[4 * c + 1], r[4 * c + 2], r[4 * c + 3]));
        }
        ptx::tc_fence_before();
        ptx::mbar_arrive(&tempty[buf]);
        __threadfence();
        ptx::named_bar_sync(1, kEpiThreads);
        if (p.dist) {
          // Every unit runs in this one wave, so all splits of the tile are
          // resident: wait until each has published its partial, then every
          // split reduces its own share of the tile's 32x32 blocks.  The
          // scales of the first round are fetched before the wait.
          constexpr int NB = C::TILE_M / 32 * NCH;
          const int my_nb = (NB - w.s + p.splits - 1) / p.splits;
          ShareScales sc;
          share_scales<C, BN, RAW>(p, job, w, 0, my_nb, sc);
          if (threadIdx.x == 64) {
            atomicAdd(p.counters + w.tile, 1);
            ptx::flag_wait_geq<false>(p.counters + w.tile, p.splits, ptx::globaltimer(), p.err,
                                      DEV_TIMEOUT_SPLIT);
          }
          ptx::named_bar_sync(1, kEpiThreads);
          reduce_share<C, BN, RAW>(p, job, w, kPartInt4, my_nb, sc);
          ptx::named_bar_sync(1, kEpiThreads);
          if (threadIdx.x == 64) {
            // the last split done reading resets both counters for the next launch
            int *done = p.counters + p.tiles_m * p.tiles_n + w.tile;
            if (atomicAdd(done, 1) == p.splits - 1) {
              p.counters[w.tile] = 0;
              *done = 0;
            }
          }
          continue;
        }
        if (threadIdx.x == 64) {
          const int prev = atomicAdd(p.counters + w.tile, 1);
          s_last = (prev == p.splits - 1);
        }
        ptx::named_bar_sync(1, kEpiThreads);
        if (s_last) {
          // the last split to finish sums every partial (integer adds are
          // exact, so the order of arrival does not matter)
          __threadfence();
          const int4 *base =
              reinterpret_cast<const int4 *>(p.ws) + (size_t)w.tile * p.splits * kPartInt4 + my_off;
#pragma unroll
          for (int ch = 0; ch < NCH; ++ch) {
            if (!mine(ch)) continue;
            const int col0 = n0 + ch * 32;
            if (col0 >= job.n) continue;
            int acc[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[i] = 0;
            for (int s = 0; s < p.splits; ++s) {
              const int4 *src = base + (size_t)s * kPartInt4 + ch * 8 * 32;
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
            if (job.tma_store) {
              if (lane == 0) ptx::bulk_wait_read<0>();
              __syncwarp();
              emit_chunk<true, RAW>(p, job, acc, xs, wsl[ch], row, col0, lane, stage, tile_row0);
            } else {
              emit_chunk<false, RAW>(p, job, acc, xs, wsl[ch], row, col0, lane, nullptr, tile_row0);
            }
          }
          ptx::named_bar_sync(1, kEpiThreads);
          if (threadIdx.x == 64) p.counters[w.tile] = 0;  // ready for the next launch
        }
      }
    }
    if (lane == 0) ptx::bulk_wait<0>();
    __syncwarp();
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// The CTA-pair kernel.  Warp roles as in k_gemm_i8_tc; in addition the
// second CTA's warp 1 forwards "my stage is full" to the first CTA (a remote
// mbarrier arrival), whose warp 1 issues the pair's MMAs once both halves of
// a stage have landed.  Commits arrive on the stage and accumulator barriers
// of both CTAs; each CTA's epilogue reads its own TMEM rows and hands the
// buffer back to the first CTA.  No split K.
template <int BN>
__global__ void __launch_bounds__(kThreads, 1) k_gemm_i8_pair(const __grid_constant__ TcParams p) {
  using C = PairCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *smA = smem;
  uint8_t *smB = smem + C::STAGES * C::A_BYTES;
  uint8_t *epi = smem + C::EPI_OFF;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
  uint64_t *full = bars;                    // this CTA's half of a stage landed
  uint64_t *empty = bars + C::STAGES;       // the pair's MMAs are done with a stage
  uint64_t *pfull = bars + 2 * C::STAGES;   // first CTA: the second CTA's half landed
  uint64_t *tfull = bars + 3 * C::STAGES;   // accumulator buffer ready (both CTAs)
  uint64_t *tempty = tfull + 2;             // first CTA: buffer drained by both CTAs
  uint64_t *mma_done = tempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = ptx::cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
      ptx::mbar_init(&pfull[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(&tfull[b], 1);
      ptx::mbar_init(&tempty[b], 2 * kEpiWarps);
    }
    ptx::mbar_init(mma_done, 1);
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&p.tmA);
    for (int j = 0; j < p.njobs; ++j) {
      ptx::prefetch_tmap(&p.jobs[j].tmB);
      if (p.jobs[j].tma_store) ptx::prefetch_tmap(&p.jobs[j].tmD);
    }
  }
  if (warp == 1) {
    ptx::tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    ptx::tmem_relinquish_pair();
  }
  ptx::tc_fence_before();
  ptx::cluster_sync();  // both CTAs' barriers exist before any remote arrival
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // warm L2 with this CTA's first B half-tiles (see k_gemm_i8_tc)
  Unit w_first{};
  if (warp == 0 && lane == 0 && pair < p.units) {
    w_first = decode_unit(p, pair);
    const int kbn = min(p.kb_total, max(C::STAGES, kPrefetchBytes / C::B_BYTES));
    for (int kb = 0; kb < kbn; ++kb)
      ptx::tma_prefetch_l2_2d(&p.jobs[w_first.job].tmB, kb * BK, w_first.n_t * BN + crank * C::BH);
  }
  ptx::griddep_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_a = ptx::policy_evict_last();
      const uint64_t pol_b = ptx::policy_evict_first();
      int it = 0;
      bool ok = true;
      for (int u = pair; u < p.units && ok; u += npairs) {
        const Unit w = u == pair ? w_first : decode_unit(p, u);
        for (int kb = 0; kb < p.kb_total; ++kb, ++it) {
          const int st = it % C::STAGES;
          const uint32_t round = it / C::STAGES;
          if (!ptx::mbar_wait(&empty[st], (round & 1) ^ 1, p.err, DEV_TIMEOUT_EMPTY)) {
            ok = false;
            break;
          }
          ptx::mbar_arrive_expect_tx(&full[st], C::STAGE_BYTES);
          ptx::tma_load_2d(&p.tmA, &full[st], smA + st * C::A_BYTES, kb * BK,
                           w.m_t * C::TILE_M + crank * BM, pol_a);
          ptx::tma_load_2d(&p.jobs[w.job].tmB, &full[st], smB + st * C::B_BYTES, kb * BK,
                           w.n_t * BN + crank * C::BH, pol_b);
        }
      }
      for (int d = 1; d <= C::STAGES && d <= it; ++d) {
        const int j = it - d;
        ptx::mbar_wait(&full[j % C::STAGES], (j / C::STAGES) & 1, p.err, DEV_TIMEOUT_DRAIN);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && crank == 0) {
      // -------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc = ptx::idesc_i8(2 * BM, BN);
      int it = 0, t = 0;
      bool ok = true;
      for (int u = pair; u < p.units && ok; u += npairs, ++t) {
        const int buf = t % C::NBUF;
        const uint32_t use = t / C::NBUF;
        if (!ptx::mbar_wait_cluster(&tempty[buf], (use & 1) ^ 1, p.err, DEV_TIMEOUT_TMEM)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * C::ACC_COLS;
        for (int kb = 0; kb < p.kb_total; ++kb, ++it) {
          const int st = it % C::STAGES;
          const uint32_t round = it / C::STAGES;
          if (!ptx::mbar_wait(&full[st], round & 1, p.err, DEV_TIMEOUT_FULL) ||
              !ptx::mbar_wait_cluster(&pfull[st], round & 1, p.err, DEV_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t a0 = ptx::smem_u32(smA + st * C::A_BYTES);
          const uint32_t b0 = ptx::smem_u32(smB + st * C::B_BYTES);
#pragma unroll
          for (int j = 0; j < BK / 32; ++j)
            ptx::mma_i8_pair(d_tmem, ptx::smem_desc_k128(a0 + 32 * j), ptx::smem_desc_k128(b0 + 32 * j),
                             idesc, (kb > 0 || j > 0) ? 1u : 0u);
          ptx::mma_commit_pair(&empty[st]);
        }
        ptx::mma_commit_pair(&tfull[buf]);
      }
      ptx::griddep_launch();
      ptx::mma_commit_pair(mma_done);
      ptx::mbar_wait(mma_done, 0, p.err, DEV_TIMEOUT_DRAIN);
    } else if (lane == 0) {
      // ------------------------------------------- forwarder (second CTA)
      const uint32_t pfull0 = ptx::mapa(ptx::smem_u32(pfull), 0);
      int it = 0;
      bool ok = true;
      for (int u = pair; u < p.units && ok; u += npairs) {
        for (int kb = 0; kb < p.kb_total; ++kb, ++it) {
          const int st = it % C::STAGES;
          if (!ptx::mbar_wait(&full[st], (it / C::STAGES) & 1, p.err, DEV_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          ptx::mbar_arrive_remote_relaxed(pfull0 + st * 8);
        }
      }
      ptx::griddep_launch();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    uint8_t *stage = epi + (warp - 2) * kEpiStageBytes;
    constexpr int NCH = BN / 32;
    const uint32_t tempty0 = ptx::mapa(ptx::smem_u32(tempty), 0);
    int t = 0;
    for (int u = pair; u < p.units; u += npairs, ++t) {
      const Unit w = decode_unit(p, u);
      const TcJob &job = p.jobs[w.job];
      const int buf = t % C::NBUF;
      const uint32_t use = t / C::NBUF;
      const int tile_row0 = w.m_t * C::TILE_M + crank * BM + q * 32;
      const int row = tile_row0 + lane;
      const int n0 = w.n_t * BN;
      const float xs = row < p.m ? __ldg(p.ssc + row) : 0.0f;
      float wsl[NCH];
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
        const int col = n0 + ch * 32 + lane;
        wsl[ch] = col < job.n ? __ldg(job.matsc + col) : 0.0f;
      }
      if (!ptx::mbar_wait(&tfull[buf], use & 1, p.err, DEV_TIMEOUT_TMEM)) break;
      ptx::tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + buf * C::ACC_COLS;
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
        if ((ch & 1) != half) continue;
        __syncwarp();
        uint32_t r[32];
        ptx::tmem_ld_32x32(taddr + ch * 32, r);
        ptx::tmem_ld_wait();
        const int col0 = n0 + ch * 32;
        if (col0 >= job.n) continue;
        if (job.tma_store) {
          if (lane == 0) ptx::bulk_wait_read<0>();
          __syncwarp();
          emit_chunk<true>(p, job, reinterpret_cast<const int(&)[32]>(r), xs, wsl[ch], row, col0, lane,
                           stage, tile_row0);
        } else {
          emit_chunk<false>(p, job, reinterpret_cast<const int(&)[32]>(r), xs, wsl[ch], row, col0,
                            lane, nullptr, tile_row0);
        }
      }
      // this warp's TMEM reads are done: hand its part of the buffer back
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (crank == 0)
          ptx::mbar_arrive(&tempty[buf]);
        else
          ptx::mbar_arrive_remote(tempty0 + buf * 8);
      }
    }
    if (lane == 0) ptx::bulk_wait<0>();
    __syncwarp();
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync();  // the other CTA is done with this CTA's barriers and TMEM
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int get_encode() {
  std::call_once(g_encode_once, [] {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return set_error("cuTensorMapEncodeTiled unavailable");
  return 0;
}

int make_map_i8(CUtensorMap *m, const int8_t *base, int k, int rows, long stride, int box_rows) {
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)stride};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t *>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error("tensor map (int8 %dx%d stride %ld) failed: %d", rows, k, stride, (int)r);
  return 0;
}

int make_map_f32(CUtensorMap *m, float *base, int n, int rows, long stride_elems) {
  cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)stride_elems * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error("tensor map (f32 %dx%d) failed: %d", rows, n, (int)r);
  return 0;
}

template <int BN, int MB, bool RAW = false>
int launch_cfg(TcParams &p, cudaStream_t st) {
  using C = Cfg<BN, MB>;
  // the shared-memory opt-in is per device; set it once, outside any capture
  static std::mutex mu;
  static uint64_t done_mask = 0;
  int dev = 0;
  GCU_CUDA(cudaGetDevice(&dev));
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!(done_mask & (1ull << (dev & 63)))) {
      GCU_CUDA(cudaFuncSetAttribute(k_gemm_i8_tc<BN, MB, RAW>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
      done_mask |= 1ull << (dev & 63);
    }
  }
  int grid = p.units < num_sms() ? p.units : num_sms();
  GCU_CUDA(launch_k(k_gemm_i8_tc<BN, MB, RAW>, grid, kThreads, C::SMEM, st, p));
  GCU_CUDA(cudaGetLastError());
  return 0;
}

template <int BN>
int launch_pair(TcParams &p, cudaStream_t st) {
  using C = PairCfg<BN>;
  static std::mutex mu;
  static uint64_t done_mask = 0;
  int dev = 0;
  GCU_CUDA(cudaGetDevice(&dev));
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!(done_mask & (1ull << (dev & 63)))) {
      GCU_CUDA(cudaFuncSetAttribute(k_gemm_i8_pair<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    C::SMEM));
      done_mask |= 1ull << (dev & 63);
    }
  }
  const int max_pairs = num_sms() / 2;
  const int pairs = p.units < max_pairs ? p.units : max_pairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  GCU_CUDA(cudaLaunchKernelEx(&cfg, k_gemm_i8_pair<BN>, p));
  GCU_CUDA(cudaGetLastError());
  return 0;
}

// Tile shapes the kernel is instantiated for: BN x (128*MB).
struct Shape {
  int bn, mb;
};
constexpr Shape kShapes[] = {{64, 1},        {128, 1},       {256, 1},      {128, 2}, {192, 2},
                             {256, 2},       {128, kPairMB}, {192, kPairMB}, {256, kPairMB}};

// rows of one tile: 128*mb for one CTA, 256 for a CTA pair
constexpr int tile_rows(int mb) { return mb == kPairMB ? 2 * BM : BM * mb; }

int split_for(int tiles, int kb_total, int sms) {
  // split K only when the tiles cannot occupy the SMs and K is long, keeping
  // at least 8 K blocks per split so the partial round trip stays small
  if (tiles * 2 > sms || kb_total < 16) return 1;
  int s = sms / tiles;
  if (s > kb_total / 8) s = kb_total / 8;
  if (s > 16) s = 16;
  return s < 1 ? 1 : s;
}

// Estimated microseconds of one launch with this tile shape.  The constants
// were fitted to per-CTA timelines (globaltimer / clock64 stamps) and to a
// sweep of every tile shape and split over the BASELINE shapes on B200:
//   - a CTA's TMA ring ingests ~100 GB/s from L2; all SMs together ~12 TB/s
//   - kind::i8 MMA sustains ~22 TOPS per SM (clocks drop under load)
//   - a CTA pair's ring moves ~78 GB/s per CTA (each stage waits for the
//     other CTA's half to be forwarded), plus ~3 us of pair set-up and tail
//   - the fp32 epilogue drains ~70 GB/s per CTA after ~0.5 us of latency
//   - a split-K round trip costs about half a partial write per split
// With two TMEM accumulators the epilogue of a tile overlaps the next tile's
// main loop; with one (MB*BN > 256) it does not.
double estimate_us(int m, int ntn, int kb_total, int bn, int mb, int splits, int sms) {
  if (mb == kPairMB) {
    // per CTA of a pair: 128 rows x bn outputs from 128 + bn/2 operand rows
    const long tiles = (long)((m + 255) / 256) * ntn;
    const double stage = (128.0 + bn / 2) * 128.0;
    const double t_load = kb_total * stage / 0.78e5;
    const double t_mma = kb_total * 2.0 * 128.0 * bn * 128.0 / 2.2e7;
    const double t_unit = t_load > t_mma ? t_load : t_mma;
    const long waves = (tiles + sms / 2 - 1) / (sms / 2);
    const double t_drain = 128.0 * bn * 4.0 / 7.0e4;
    double t_main = waves * (t_unit > t_drain ? t_unit : t_drain);
    const double t_l2 = (double)tiles * 2 * kb_total * stage / 1.2e7;
    if (t_l2 > t_main) t_main = t_l2;
    return t_main + 3.0 + t_drain;
  }
  const double tile_m = 128.0 * mb;
  const long tiles = (long)((m + 128 * mb - 1) / (128 * mb)) * ntn;
  const long units = tiles * splits;
  const int kb_unit = (kb_total + splits - 1) / splits;
  const double stage = (tile_m + bn) * 128.0;
  const double t_load = kb_unit * stage / 1.0e5;
  const double t_mma = kb_unit * 2.0 * tile_m * bn * 128.0 / 2.2e7;
  const double t_unit = t_load > t_mma ? t_load : t_mma;
  const long waves = (units + sms - 1) / sms;
  const double out_bytes = tile_m * bn * 4.0;
  const double t_drain = out_bytes / 7.0e4;
  const double t_out = 0.5 + t_drain;
  const bool two_acc = 2 * mb * bn <= 512;
  double t_main = two_acc ? waves * (t_unit > t_drain ? t_unit : t_drain) : waves * (t_unit + t_out);
  const double t_l2 = (double)units * kb_unit * stage / 1.2e7;
  if (t_l2 > t_main) t_main = t_l2;
  const double t_split = splits > 1 ? 0.5 * out_bytes * splits / 7.0e4 : 0.0;
  return t_main + (two_acc ? t_out : 0.0) + t_split;
}

}  // namespace

namespace {

struct Plan {
  int bn, mb, splits;  // CTA tile (128*mb) x bn, K split
};

int ntiles_n(const GemmArgs *jobs, int njobs, int bn) {
  int t = 0;
  for (int j = 0; j < njobs; ++j) t += (jobs[j].n + bn - 1) / bn;
  return t;
}

// Enqueue one launch of plan `pl` (everything after the tile choice).
int run_plan(const Plan &pl, const int8_t *src, long sstr, const float *ssc, int m, int k,
             const GemmArgs *jobs, int njobs, cudaStream_t st, const ExtWorkspace *ext);

// Planner's pick without running anything: the cost model above.
Plan model_plan(int m, int k, const GemmArgs *jobs, int njobs, int sms, bool allow_pair = true) {
  const int kb_total = (k + BK - 1) / BK;
  Plan best{128, 1, 1};
  double best_t = 1e30;
  for (const Shape &sh : kShapes) {
    if (!allow_pair && sh.mb == kPairMB) continue;
    const int tiles = (m + tile_rows(sh.mb) - 1) / tile_rows(sh.mb) * ntiles_n(jobs, njobs, sh.bn);
    const int sp = sh.mb == kPairMB ? 1 : split_for(tiles, kb_total, sms);
    const double t = estimate_us(m, ntiles_n(jobs, njobs, sh.bn), kb_total, sh.bn, sh.mb, sp, sms);
    if (t < best_t - 1e-9) {
      best_t = t;
      best = Plan{sh.bn, sh.mb, sp};
    }
  }
  return best;
}

// Measured pick (opt-in, GCU_AUTOTUNE=1): the first call of a shape
// (outside stream capture) times every tile shape, with and without a K
// split, on the caller's stream and caches the fastest per device.  Every
// candidate computes the same exact int32 sums, so the output is the same
// whichever wins.  It times repeated calls on the same operands, i.e. with
// the weights warm in L2, which misjudges a model whose weights stream from
// HBM once per token; the calibrated cost model is therefore the default.
struct TuneKey {
  int dev, m, k, njobs, n[kMaxJobs];
  bool operator<(const TuneKey &o) const {
    return std::tie(dev, m, k, njobs, n[0], n[1], n[2], n[3]) <
           std::tie(o.dev, o.m, o.k, o.njobs, o.n[0], o.n[1], o.n[2], o.n[3]);
  }
};
std::mutex g_tune_mu;
std::map<TuneKey, Plan> g_tune;

bool autotune_enabled() {
  static const bool on = [] {
    const char *e = getenv("GCU_AUTOTUNE");
    return e && e[0] == '1';
  }();
  return on;
}

int tuned_plan(Plan *out, const int8_t *src, long sstr, const float *ssc, int m, int k,
               const GemmArgs *jobs, int njobs, cudaStream_t st, int sms) {
  TuneKey key{};
  GCU_CUDA(cudaGetDevice(&key.dev));
  key.m = m;
  key.k = k;
  key.njobs = njobs;
  for (int j = 0; j < njobs; ++j) key.n[j] = jobs[j].n;
  {
    std::lock_guard<std::mutex> lk(g_tune_mu);
    auto it = g_tune.find(key);
    if (it != g_tune.end()) {
      *out = it->second;
      return 0;
    }
  }
  const int kb_total = (k + BK - 1) / BK;
  Plan cand[2 * sizeof(kShapes) / sizeof(kShapes[0])];
  int nc = 0;
  for (const Shape &sh : kShapes) {
    const int tiles = (m + tile_rows(sh.mb) - 1) / tile_rows(sh.mb) * ntiles_n(jobs, njobs, sh.bn);
    const int sp = split_for(tiles, kb_total, sms);
    cand[nc++] = Plan{sh.bn, sh.mb, 1};
    if (sp > 1 && sh.mb != kPairMB) cand[nc++] = Plan{sh.bn, sh.mb, sp};
  }
  cudaEvent_t e0, e1;
  GCU_CUDA(cudaEventCreate(&e0));
  if (cudaEventCreate(&e1) != cudaSuccess) {
    cudaEventDestroy(e0);
    return set_error("gemm autotune: cudaEventCreate failed");
  }
  float best_ms = 1e30f;
  Plan best = model_plan(m, k, jobs, njobs, sms);
  int rc = 0;
  for (int c = 0; c < nc && rc == 0; ++c) {
    rc = run_plan(cand[c], src, sstr, ssc, m, k, jobs, njobs, st, nullptr);  // warm
    if (rc) break;
    cudaEventRecord(e0, st);
    for (int r = 0; r < 3 && rc == 0; ++r)
      rc = run_plan(cand[c], src, sstr, ssc, m, k, jobs, njobs, st, nullptr);
    cudaEventRecord(e1, st);
    if (cudaEventSynchronize(e1) != cudaSuccess) {
      rc = set_error("gemm autotune: event synchronize failed");
      break;
    }
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e0, e1);
    if (ms < best_ms) {
      best_ms = ms;
      best = cand[c];
    }
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (rc) return rc;
  {
    std::lock_guard<std::mutex> lk(g_tune_mu);
    g_tune[key] = best;
  }
  if (getenv("GCU_DEBUG"))
    fprintf(stderr, "gcu: gemm m=%d k=%d n0=%d jobs=%d -> tile %dx%d split %d (%.2f us)\n", m, k,
            key.n[0], njobs, tile_rows(best.mb), best.bn, best.splits, best_ms * 1000.0f / 3.0f);
  *out = best;
  return 0;
}

}  // namespace

// Multi-job entry: jobs share A (src); job j has its own weights and output.
int launch_gemm_tc_jobs(const int8_t *src, long sstr, const float *ssc, int m, int k,
                        const GemmArgs *jobs, int njobs, cudaStream_t st, int force_bn,
                        int force_split, const ExtWorkspace *ext, int force_mb) {
  if (njobs < 1 || njobs > kMaxJobs) return set_error("gemm: 1..%d jobs (got %d)", kMaxJobs, njobs);
  if (m <= 0 || k <= 0) return 0;
  if (get_encode()) return 1;
  if ((uintptr_t)src % 16 || sstr % 16)
    return set_error("gemm: activation rows must be 16-byte aligned (stride %ld)", sstr);
  const int sms = num_sms();
  for (int j = 0; j < njobs; ++j)
    if ((uintptr_t)jobs[j].mat % 16 || jobs[j].mstr % 16)
      return set_error("gemm: weight rows must be 16-byte aligned (stride %ld)", jobs[j].mstr);
  const int kb_total = (k + BK - 1) / BK;
  Plan pl;
  if (force_bn > 0) {
    pl.bn = force_bn;
    pl.mb = force_mb > 0 ? force_mb : 1;
    bool known = false;
    for (const Shape &sh : kShapes) known |= (sh.bn == pl.bn && sh.mb == pl.mb);
    if (!known) return set_error("gemm: no %d x %d tile variant", tile_rows(pl.mb), pl.bn);
    const int tiles = (m + tile_rows(pl.mb) - 1) / tile_rows(pl.mb) * ntiles_n(jobs, njobs, pl.bn);
    pl.splits = force_split > 0 ? force_split : split_for(tiles, kb_total, sms);
    if (pl.mb == kPairMB && pl.splits > 1) return set_error("gemm: the CTA-pair tiles take no K split");
    return run_plan(pl, src, sstr, ssc, m, k, jobs, njobs, st, ext);
  }
  // int32-sum output exists for the one-CTA tiles only
  const bool raw = jobs[0].raw != 0;
  pl = model_plan(m, k, jobs, njobs, sms, !raw);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  GCU_CUDA(cudaStreamIsCapturing(st, &cap));
  if (!ext && !raw && autotune_enabled() && cap == cudaStreamCaptureStatusNone &&
      tuned_plan(&pl, src, sstr, ssc, m, k, jobs, njobs, st, sms))
    return 1;
  if (force_split > 0) pl.splits = force_split;
  return run_plan(pl, src, sstr, ssc, m, k, jobs, njobs, st, ext);
}

namespace {

int run_plan(const Plan &pl, const int8_t *src, long sstr, const float *ssc, int m, int k,
             const GemmArgs *jobs, int njobs, cudaStream_t st, const ExtWorkspace *ext) {
  const int bn = pl.bn, mb = pl.mb;
  const bool pair = mb == kPairMB;
  for (int j = 1; j < njobs; ++j)
    if (jobs[j].raw != jobs[0].raw) return set_error("gemm: int32-sum output is all jobs or none");
  if (jobs[0].raw && pair) return set_error("gemm: int32-sum output has no CTA-pair tile");
  const int kb_total = (k + BK - 1) / BK;
  const int tile_m = tile_rows(mb);
  const int tiles_m = (m + tile_m - 1) / tile_m;
  const int tiles_n = ntiles_n(jobs, njobs, bn);
  const int tiles = tiles_m * tiles_n;
  int splits = pl.splits < 1 || pair ? 1 : pl.splits;
  if (splits > kb_total) splits = kb_total;
  const int kb_per = (kb_total + splits - 1) / splits;
  splits = (kb_total + kb_per - 1) / kb_per;

  static_assert(sizeof(TcParams) <= 4096, "kernel parameters exceed 4 KB");
  TcParams p;
  memset(&p, 0, sizeof(p));
  // a pair's CTAs each load 128 A rows and bn/2 B rows per stage
  if (make_map_i8(&p.tmA, src, k, m, sstr, pair ? BM : tile_m)) return 1;
  int tn = 0;
  for (int j = 0; j < njobs; ++j) {
    TcJob &J = p.jobs[j];
    if (make_map_i8(&J.tmB, jobs[j].mat, k, jobs[j].n, jobs[j].mstr, pair ? bn / 2 : bn)) return 1;
    J.tma_store = ((uintptr_t)jobs[j].dst % 16 == 0) && (jobs[j].dstr % 4 == 0);
    if (J.tma_store && make_map_f32(&J.tmD, jobs[j].dst, jobs[j].n, m, jobs[j].dstr)) return 1;
    J.matsc = jobs[j].matsc;
    J.dst = jobs[j].dst;
    J.dstr = jobs[j].dstr;
    J.n = jobs[j].n;
    J.tn_begin = tn;
    tn += (jobs[j].n + bn - 1) / bn;
  }
  p.njobs = njobs;
  p.m = m;
  p.k = k;
  p.tiles_m = tiles_m;
  p.tiles_n = tiles_n;
  p.splits = splits;
  p.kb_total = kb_total;
  p.kb_per_split = kb_per;
  p.units = tiles * splits;
  p.ssc = ssc;
  p.err = dev_error_word();
  if (splits > 1) {
    const size_t need = (size_t)tiles * splits * tile_m * bn * sizeof(int32_t);
    void *ws = nullptr;
    int *cnt = nullptr;
    if (ext) {
      if (need > ext->ws_bytes || 2 * tiles > ext->ncounters)
        return set_error("gemm: split-K needs %zu bytes of scratch and %d counters; the caller's "
                         "scratch holds %zu bytes and %d counters",
                         need, 2 * tiles, ext->ws_bytes, ext->ncounters);
      GCU_CUDA(cudaMemsetAsync(ext->counters, 0, (size_t)2 * tiles * sizeof(int), st));
      ws = ext->ws;
      cnt = ext->counters;
    } else if (gemm_workspace(need, &ws, &cnt, 2 * tiles, st)) {
      return 1;
    }
    p.ws = static_cast<int32_t *>(ws);
    p.counters = cnt;
    // one wave (grid = min(units, SMs), one CTA per SM): every split of a
    // tile is resident together and they can share the reduction
    p.dist = p.units <= num_sms();
  }
  if (pair) {
    if (bn == 128) return launch_pair<128>(p, st);
    if (bn == 192) return launch_pair<192>(p, st);
    return launch_pair<256>(p, st);
  }
  if (jobs[0].raw) {  // int32 sums out (one-CTA tiles only)
    if (mb == 2) {
      if (bn == 128) return launch_cfg<128, 2, true>(p, st);
      if (bn == 192) return launch_cfg<192, 2, true>(p, st);
      return launch_cfg<256, 2, true>(p, st);
    }
    if (bn == 256) return launch_cfg<256, 1, true>(p, st);
    if (bn == 128) return launch_cfg<128, 1, true>(p, st);
    return launch_cfg<64, 1, true>(p, st);
  }
  if (mb == 2) {
    if (bn == 128) return launch_cfg<128, 2>(p, st);
    if (bn == 192) return launch_cfg<192, 2>(p, st);
    return launch_cfg<256, 2>(p, st);
  }
  if (bn == 256) return launch_cfg<256, 1>(p, st);
  if (bn == 128) return launch_cfg<128, 1>(p, st);
  return launch_cfg<64, 1>(p, st);
}

}  // namespace

int launch_gemm_tc(const GemmArgs &a, cudaStream_t st, int force_bn, int force_split,
                   int force_mb) {
  return launch_gemm_tc_jobs(a.src, a.sstr, a.ssc, a.m, a.k, &a, 1, st, force_bn, force_split,
                             nullptr, force_mb);
}

// ---- helpers shared with the chain kernel (k_chain.cu) ----------------------
int gemm_tmap_i8(CUtensorMap *m, const int8_t *base, int k, int rows, long stride, int box_rows) {
  if (get_encode()) return 1;
  return make_map_i8(m, base, k, rows, stride, box_rows);
}

int gemm_tmap_f32(CUtensorMap *m, float *base, int n, int rows, long stride_elems) {
  if (get_encode()) return 1;
  return make_map_f32(m, base, n, rows, stride_elems);
}

int gemm_plan_one_cta(int m, int k, const int *n, int njobs, int sms, int *bn, int *mb, int *splits) {
  if (njobs < 1 || njobs > kMaxJobs) return set_error("gemm plan: 1..%d jobs (got %d)", kMaxJobs, njobs);
  GemmArgs jobs[kMaxJobs] = {};
  for (int j = 0; j < njobs; ++j) jobs[j].n = n[j];
  const Plan pl = model_plan(m, k, jobs, njobs, sms, false);
  *bn = pl.bn;
  *mb = pl.mb;
  *splits = pl.splits;
  return 0;
}

int gemm_split_for(int tiles, int k, int sms) { return split_for(tiles, (k + BK - 1) / BK, sms); }

}  // namespace gcu

// Test hook (not in the public header): gemm_int8's int32 sums themselves,
// dst[i][j] = sum_l src[i][l] * mat[j][l] as int32 bit patterns, with a forced
// tile shape and K split -- the mode the sharded FFN's down projection uses.
extern "C" __attribute__((visibility("default"))) int gcu_dev_gemm_int8_raw_tuned(
    int32_t *dst, const int8_t *mat, const int8_t *src, int m, int n, int k, int bn, int split, int mb,
    void *stream) {
  using namespace gcu;
  if (m <= 8) return set_error("gemm_int8_raw: m > 8 only (tensor-core path)");
  GemmArgs a{reinterpret_cast<float *>(dst), n, mat, k, nullptr, src, k, nullptr, m, n, k};
  a.raw = 1;
  return launch_gemm_tc_jobs(src, k, nullptr, m, k, &a, 1, static_cast<cudaStream_t>(stream), bn, split,
                             nullptr, mb);
}
