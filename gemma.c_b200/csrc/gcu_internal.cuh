// gcu_internal.cuh -- shared declarations of the gemma.c W8A8 CUDA library.
//
// Everything here is internal to libgcu.so: launch helpers, the device
// error word, and inline-PTX wrappers for the sm_100a features the kernels
// use (mbarrier, TMA tensor copies, tcgen05 / TMEM).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/gcu.h"

namespace gcu {

// ---------------------------------------------------------------------------
// host-side error reporting (thread local, like gemma.c's g_err, gemma.c:577)
// ---------------------------------------------------------------------------
int set_error(const char *fmt, ...);
int check_cuda(cudaError_t e, const char *what);
#define GCU_CUDA(call)                                                        \
  do {                                                                        \
    cudaError_t e__ = (call);                                                 \
    if (e__ != cudaSuccess)                                                   \
      return ::gcu::check_cuda(e__, #call);                                   \
  } while (0)

int num_sms();

// Programmatic dependent launch: every kernel is launched with programmatic
// stream serialization, does its setup (barrier init, TMEM allocation,
// descriptor prefetch), then waits on griddepcontrol.wait before touching
// global memory, so its prologue overlaps the previous kernel's tail.
// GCU_PDL=0 in the environment turns the attribute off.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                            cudaStream_t st, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------------------
// device error word.  Kernels never trap: a bounded wait that gives up sets
// a code here and the kernel returns; the host reads it after synchronising.
// ---------------------------------------------------------------------------
enum DevErr : unsigned int {
  DEV_OK = 0,
  DEV_TIMEOUT_FULL = 1,   // MMA warp waited too long for a TMA stage
  DEV_TIMEOUT_EMPTY = 2,  // producer waited too long for a free stage
  DEV_TIMEOUT_TMEM = 3,   // accumulator hand-off between MMA and epilogue
  DEV_TIMEOUT_DRAIN = 4,  // draining in-flight copies after an error
  DEV_TIMEOUT_PEER = 6,   // a rank of a fused all-gather never signalled
  DEV_TIMEOUT_SPLIT = 7,  // a split-K CTA waited too long for the other splits
  DEV_TIMEOUT_SELFTEST = 8,  // gcu_selftest_bounded_wait's wait (nothing ever completes it)
  DEV_TIMEOUT_CHAIN = 9,     // a chain launch's grid-wide hand-off between two steps
};
unsigned int *dev_error_word();  // device address of the error word
// Bit mask of the device error codes the host has observed since start-up
// (1u << code), including a code now sitting in the error word unread;
// forget_error_code clears one (after the state it poisoned is rebuilt).
unsigned int error_codes_seen();
void forget_error_code(unsigned int code);

// ---------------------------------------------------------------------------
// weight registry (gcu_api.cu)
// ---------------------------------------------------------------------------
int calling_device();  // the calling thread's device (gcu_init)
// a weight whose device copy lives at byte offsets dq_off / ds_off of an arena
struct RegRec {
  uintptr_t q, s;  // host int8 values / scales
  int rows, k;
  size_t dq_off, ds_off;
};
// Register n weights held by the device allocation `base` (`bytes`), which
// the registry then owns; fails, owning nothing, if any overlaps a weight
// already registered.
int registry_add_arena(const RegRec *recs, int n, void *base, size_t bytes, int *arena_id);
void release_staging();  // free the model uploader's pinned slots (gcu_model.cu)

// ---------------------------------------------------------------------------
// kernel launchers (defined in k_*.cu)
// ---------------------------------------------------------------------------
int launch_quantize_rows(int8_t *dst, float *dsc, const float *src, long sstr,
                         int m, int n, cudaStream_t st);

struct GemvJobs {
  const int8_t *w[GCU_MAX_JOBS];
  const float *ws[GCU_MAX_JOBS];
  float *y[GCU_MAX_JOBS];
  int row_end[GCU_MAX_JOBS];  // exclusive prefix sums of job rows
  int njobs;
};
// y_j[b*ystride + i] = (float)dot(w_j row i, x row b) * (xs[b] * ws_j[i])
// for b < mb (mb <= 8) over all jobs' rows.
int launch_gemv(const GemvJobs &jobs, const int8_t *x, long xstride,
                const float *xs, int mb, long ystride, int k,
                cudaStream_t st);

// Row-sharded GEMV whose epilogue is the all-gather.  Every rank holds a
// symmetric buffer (two halves, mapped by every peer through CUDA IPC) laid
// out identically: job j's (mb, n_j) output at float offset off[j] of a half,
// rank r's column slice at r * n_local[j].  Each rank stores its slices into
// half (epoch & 1) of its own buffer; the last CTA of the grid to finish
// signals every rank ("slices ready"); every CTA waits, bounded, until all
// ranks have signalled for this launch, then pulls its share of every rank's
// slices over NVLink (16-byte loads from the peers' mappings) into the
// caller's dst.  The halves alternate by a device-side launch epoch: a rank
// one launch ahead writes the other half, and it cannot get two ahead before
// this rank has finished pulling.
struct PeerOut {
  long long delta[8];  // bytes from this rank's symmetric buffer to rank p's
  int *flag_peer[8];   // rank p's arrival counter
  int *flag_local;     // [0] arrivals (world per launch), [1] launch epoch,
                       // [2] finished CTAs of this launch
  float *sym;          // this rank's symmetric buffer (two halves)
  long half_elems;     // floats per half
  long off[GCU_MAX_JOBS];                    // job region offsets in a half
  int n[GCU_MAX_JOBS], n_local[GCU_MAX_JOBS];  // full / per-rank columns (n_local % 4 == 0)
  float *dst[GCU_MAX_JOBS];                  // caller's outputs, [mb][n_j] dense
  int njobs, mb, rank, world;
  unsigned int *err;
};
// x/xs: quantized activations, or xf (fp32, quantized in the launch into
// qout/sout as quantize_acts would) when xf is not null.
int launch_gemv_p2p(const GemvJobs &jobs, const int8_t *x, long xstride, const float *xs,
                    const float *xf, int8_t *qout, float *sout, int mb, int k,
                    const PeerOut &po, cudaStream_t st);

// GeGLU over a slice of the hidden dimension (k_producers.cu): h and each
// row's |max| over the slice; then the codes of h given each row's max over
// every slice (scales as quantize_acts writes them).  Rows 16-byte aligned,
// n % 4 == 0.
int launch_geglu_amax(float *h, float *amax, const float *gate, const float *up, int m, int n,
                      cudaStream_t st);
int launch_quantize_given_amax(int8_t *q, float *s, const float *h, const float *amax, int m, int n,
                               cudaStream_t st);

// quantize_acts + GEMV in one launch (mb <= 8 rows of fp32 xf); writes the
// codes (qout, dense [mb][k]) and scales (sout) as quantize_acts would.
int launch_quantize_gemv(const GemvJobs &jobs, const float *xf, long xfstride,
                         int8_t *qout, float *sout, int mb, long ystride, int k,
                         cudaStream_t st);

// A producer row + GEMV in one launch (one token): h = gelu(gate) * up, or
// x = clamp(resid + rmsnorm(y, w_post)) then rmsnorm(x, w_next), quantized
// and multiplied; codes, scale and (residual form) x are written out.
int launch_geglu_gemv(const GemvJobs &jobs, const float *gate, const float *up, int8_t *qout, float *sout,
                      int k, cudaStream_t st);
int launch_resnorm_gemv(const GemvJobs &jobs, const float *y, const float *resid, const float *w_post,
                        const float *w_next, float eps, float *xout, int8_t *qout, float *sout, int dim,
                        cudaStream_t st);

struct GemmArgs {
  float *dst;
  long dstr;
  const int8_t *mat;
  long mstr;
  const float *matsc;
  const int8_t *src;
  long sstr;
  const float *ssc;
  int m, n, k;
  int raw = 0;  // 1: dst receives the int32 sums (as their bit patterns), scales unused
};
// force_bn / force_mb / force_split = 0 let the planner choose the tile
// shape ((128*mb) x bn) and the K split.
int launch_gemm_tc(const GemmArgs &a, cudaStream_t st, int force_bn,
                   int force_split, int force_mb = 0);

// Caller-owned split-K scratch: when given, the launcher uses it instead of
// the runtime's allocated workspace, fails if the plan needs more than
// ws_bytes / ncounters, and zeroes the counters it uses on `st` first.
struct ExtWorkspace {
  void *ws;
  size_t ws_bytes;
  int *counters;
  int ncounters;
};
// Tensor-core GEMM over up to 4 jobs sharing the A operand `src`.
int launch_gemm_tc_jobs(const int8_t *src, long sstr, const float *ssc, int m,
                        int k, const GemmArgs *jobs, int njobs, cudaStream_t st,
                        int force_bn, int force_split,
                        const ExtWorkspace *ext = nullptr, int force_mb = 0);

// split-K workspace and tile counters (device memory owned by the runtime)
int gemm_workspace(size_t bytes, void **ws, int **counters, int ncounters,
                   cudaStream_t st);

// Shared with the chain kernel (k_chain.cu): TMA tensor maps of the GEMM's
// operand layouts (int8 [rows][k], box 128 B x box_rows, 128-byte swizzle;
// fp32 [rows][n], box 32 x 32), and the one-CTA tile planner ((128*mb) x bn
// tiles, K split) over the cost model of the GEMM launcher.
int gemm_tmap_i8(CUtensorMap *m, const int8_t *base, int k, int rows, long stride, int box_rows);
int gemm_tmap_f32(CUtensorMap *m, float *base, int n, int rows, long stride_elems);
int gemm_plan_one_cta(int m, int k, const int *n, int njobs, int sms, int *bn, int *mb,
                      int *splits);
int gemm_split_for(int tiles, int k, int sms);

}  // namespace gcu

// ===========================================================================
// device-side PTX helpers
// ===========================================================================
#if defined(__CUDACC__)
namespace gcu {
namespace ptx {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// wait until the grids this one depends on have completed and their memory
// is visible (no-op without a programmatic dependency)
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
// allow the dependent grid to be scheduled (it still waits for our completion
// in its griddep_wait before reading anything we write)
__device__ __forceinline__ void griddep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Record a device-side error code.  The word may live in mapped pinned host
// memory (the host entry points read it there after their stream wait, with
// no copy), so it is written with a plain store rather than an atomic: any
// nonzero code reports the failure, and the first writer usually wins.
__device__ __forceinline__ void record_err(unsigned int *err, unsigned int code) {
  volatile unsigned int *e = err;
  if (*e == 0u) *e = code;
  __threadfence_system();
}

__device__ __forceinline__ int ld_acquire_sys(const int *p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_acquire_gpu(const int *p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Spin until *flag >= target, acquiring at system scope (SYS: the flag is
// written by other GPUs) or gpu scope, for at most budget_ns after t0.
// Returns false, with `code` recorded in the error word, on timeout.
template <bool SYS>
__device__ __forceinline__ bool flag_wait_geq(const int *flag, int target, uint64_t t0,
                                              unsigned int *err, unsigned int code,
                                              uint64_t budget_ns = 2000000000ull) {
  while ((SYS ? ld_acquire_sys(flag) : ld_acquire_gpu(flag)) < target) {
    if (globaltimer() - t0 > budget_ns) {
      record_err(err, code);
      return false;
    }
    __nanosleep(32);
  }
  return true;
}

// ---- mbarrier --------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar,
                                                      uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar` to complete, for at most `budget_ns`.
// Returns false (and records `code` in the device error word) on timeout.
// as mbar_try_wait, acquiring at cluster scope (arrivals from the other CTA
// of a pair)
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity,
                                                  unsigned int *err, unsigned int code,
                                                  uint64_t budget_ns = 2000000000ull) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait_cluster(bar, parity)) return true;
    if (globaltimer() - t0 > budget_ns) {
      record_err(err, code);
      return false;
    }
  }
}
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity,
                                          unsigned int *err, unsigned int code,
                                          uint64_t budget_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > budget_ns) {
      record_err(err, code);
      return false;
    }
  }
}

// ---- TMA: each load lands in the issuing CTA's own shared memory ------------
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(m) : "memory");
}
__device__ __forceinline__ void tma_load_2d(const CUtensorMap *m,
                                            uint64_t *bar, void *dst, int x,
                                            int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::"
      "bytes.L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(m), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
// L2 prefetch of one tile through a tensor map (no data reaches the CTA)
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap *m, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(m), "r"(x),
               "r"(y)
               : "memory");
}
// 1D bulk copy of `bytes` (a multiple of 16) from a 16-byte aligned global
// address into this CTA's shared memory (16-byte aligned), completing on
// `bar` (complete_tx); only the issuing CTA receives the bytes.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// L2 prefetch of `bytes` (a multiple of 16) from a 16-byte aligned address
__device__ __forceinline__ void bulk_prefetch_l2(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *m,
                                             const void *src, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], "
      "[%1];" ::"l"(m),
      "r"(smem_u32(src)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;"
               : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;"
               : "=l"(p));
  return p;
}

// ---- tcgen05 / TMEM ----------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(slot)),
      "r"(ncols)
      : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(
                   taddr),
               "r"(ncols)
               : "memory");
}
// ---- CTA pairs (thread-block clusters of two) ------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// every thread of both CTAs; orders each CTA's earlier memory operations
// (remote mbarrier arrivals included) before the other's later ones
__device__ __forceinline__ void cluster_sync() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}
// shared::cluster address of this CTA's shared variable `saddr` in CTA `rank`
__device__ __forceinline__ uint32_t mapa(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// arrive (release at cluster scope) on an mbarrier of the other CTA
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
// the same without the release fence (~0.7 us cheaper per arrival on B200):
// for signalling that an asynchronous copy into this CTA's shared memory has
// completed (its mbarrier phase was observed), where the reader is the other
// CTA's tensor core and no generic-proxy write needs ordering
__device__ __forceinline__ void mbar_arrive_remote_relaxed(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// D[tmem of both CTAs] (+)= A[smem of both] * B[smem of both]^T: M = 256 rows
// (128 in each CTA), N columns (N/2 rows of B in each CTA); issued by one
// thread of the pair's first CTA
__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on `bar` (same offset) in both CTAs of the pair once every tcgen05
// operation issued so far has completed
__device__ __forceinline__ void mma_commit_pair(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32, one CTA.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc,
                                       uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on `bar` once all tcgen05 operations issued so far have completed
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(smem_u32(bar))
      : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns -> 32 registers per thread
__device__ __forceinline__ void tmem_ld_32x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
        "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzle: rows of 128 bytes, 8-row swizzle atoms 1024 bytes
// apart (stride byte offset), leading byte offset unused (1), descriptor
// version 1 (tcgen05), layout type 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t smem_desc_k128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor, kind::i8: D = s32, A = B = signed int8, both
// K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- quantize arithmetic of gemma.c:2586-2650 under -ffast-math ------------
// scale = amax * (1/127), inv = 127 / amax (IEEE division); 1, 1 for amax 0;
// q = trunc(x*inv + copysign(0.5, x*inv)) clamped to [-127, 127].  Explicit
// round-to-nearest intrinsics keep nvcc from contracting into FMAs.
__device__ __forceinline__ int quant_one(float x, float inv) {
  const float t = __fmul_rn(x, inv);
  const float s = __fadd_rn(t, copysignf(0.5f, t));
  int q = __float2int_rz(s);
  q = q > 127 ? 127 : q;
  q = q < -127 ? -127 : q;
  return q;
}
__device__ __forceinline__ void quant_scale(float amax, float &scale, float &inv) {
  if (amax > 0.0f) {
    scale = __fmul_rn(amax, 1.0f / 127.0f);
    inv = __fdiv_rn(127.0f, amax);
  } else {
    scale = 1.0f;
    inv = 1.0f;
  }
}
__device__ __forceinline__ float absmax4(const float4 &v, float m) {
  return fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
}
// four quantized values packed little-endian into one 32-bit word
__device__ __forceinline__ int quant_pack4(const float4 &v, float inv) {
  return (quant_one(v.x, inv) & 0xff) | ((quant_one(v.y, inv) & 0xff) << 8) |
         ((quant_one(v.z, inv) & 0xff) << 16) | ((quant_one(v.w, inv) & 0xff) << 24);
}

// streaming 16-byte global load that does not allocate in L1
__device__ __forceinline__ int4 ld_stream_v4(const void *p) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

}  // namespace ptx
}  // namespace gcu
#endif
