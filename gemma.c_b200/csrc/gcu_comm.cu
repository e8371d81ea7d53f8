// gcu_comm.cu -- row-sharded W8A8 matmul across the GPUs of one node.
//
// The reference is single-process (README.md:614); this is the one place the
// library adds communication.  Every output row of gemm_int8 / gemv_int8 is
// independent, so rank r computes rows [r*n/world, (r+1)*n/world) of the
// output from its slice of the weight and the slices are all-gathered over
// NVLink.  For the decode shapes (m <= 8) the all-gather is fused into the
// GEMV: each rank stores its outputs straight into every rank's symmetric
// buffer (CUDA IPC mappings exchanged at gcu_comm_init) and a bounded
// flag barrier ends the launch (see PeerOut).  Larger m, or a node without
// peer access, uses an NCCL all-gather.  NCCL is opened with dlopen on first
// use so the single-GPU entry points never depend on it.
#include "gcu_internal.cuh"

#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#define GCU_EXPORT extern "C" __attribute__((visibility("default")))

namespace gcu {
namespace {

struct Nccl {
  void *lib = nullptr;
  ncclResult_t (*getUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*commInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*allGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*allReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
  const char *(*getErrorString)(ncclResult_t) = nullptr;
};
Nccl g_nccl;
std::once_flag g_nccl_once;

int nccl() {
  std::call_once(g_nccl_once, [] {
    const char *names[] = {"libnccl.so.2", "libnccl.so"};
    for (const char *n : names) {
      g_nccl.lib = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
      if (g_nccl.lib) break;
    }
    if (!g_nccl.lib) return;
    g_nccl.getUniqueId = (decltype(g_nccl.getUniqueId))dlsym(g_nccl.lib, "ncclGetUniqueId");
    g_nccl.commInitRank = (decltype(g_nccl.commInitRank))dlsym(g_nccl.lib, "ncclCommInitRank");
    g_nccl.allGather = (decltype(g_nccl.allGather))dlsym(g_nccl.lib, "ncclAllGather");
    g_nccl.allReduce = (decltype(g_nccl.allReduce))dlsym(g_nccl.lib, "ncclAllReduce");
    g_nccl.commDestroy = (decltype(g_nccl.commDestroy))dlsym(g_nccl.lib, "ncclCommDestroy");
    g_nccl.getErrorString = (decltype(g_nccl.getErrorString))dlsym(g_nccl.lib, "ncclGetErrorString");
  });
  if (!g_nccl.lib || !g_nccl.getUniqueId || !g_nccl.commInitRank || !g_nccl.allGather ||
      !g_nccl.allReduce || !g_nccl.commDestroy)
    return set_error("NCCL (libnccl.so.2) could not be loaded");
  return 0;
}

int nccl_err(ncclResult_t r, const char *what) {
  return set_error("%s: %s", what, g_nccl.getErrorString ? g_nccl.getErrorString(r) : "nccl error");
}

// symmetric buffer: two halves of kSymHalf bytes, plus 4 flag words
constexpr size_t kSymHalf = (size_t)8 << 20;

struct Comm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  bool p2p = false;
  float *sym = nullptr;
  int *flags = nullptr;
  void *peer_sym[8] = {};
  int *peer_flags[8] = {};
};
Comm g_comm;
std::mutex g_comm_mu;

// Allocate this rank's symmetric buffer, exchange IPC handles over NCCL and
// map every peer's.  Any failure leaves p2p off on all ranks (they agree
// through a second all-gather), and the NCCL all-gather path is used.
int setup_p2p(Comm &c) {
  if (c.world < 2 || c.world > 8) return 0;
  cudaIpcMemHandle_t h[2];
  int ok = 1;
  if (cudaMalloc(&c.sym, 2 * kSymHalf) != cudaSuccess ||
      cudaMalloc(&c.flags, 256) != cudaSuccess || cudaMemset(c.flags, 0, 256) != cudaSuccess ||
      cudaIpcGetMemHandle(&h[0], c.sym) != cudaSuccess ||
      cudaIpcGetMemHandle(&h[1], c.flags) != cudaSuccess)
    ok = 0;
  cudaGetLastError();
  // all-gather {ok, handles} through NCCL
  const size_t rec = sizeof(int) * 4 + sizeof(h);
  unsigned char *dbuf = nullptr;
  cudaStream_t st = nullptr;
  std::vector<unsigned char> hbuf(rec * c.world);
  memcpy(hbuf.data() + rec * c.rank, &ok, sizeof(int));
  memcpy(hbuf.data() + rec * c.rank + 4 * sizeof(int), h, sizeof(h));
  GCU_CUDA(cudaMalloc(&dbuf, rec * c.world));
  GCU_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  GCU_CUDA(cudaMemcpy(dbuf + rec * c.rank, hbuf.data() + rec * c.rank, rec, cudaMemcpyHostToDevice));
  ncclResult_t r = g_nccl.allGather(dbuf + rec * c.rank, dbuf, rec, ncclUint8, c.comm, st);
  if (r != ncclSuccess) {
    cudaFree(dbuf);
    cudaStreamDestroy(st);
    return nccl_err(r, "ncclAllGather (ipc handles)");
  }
  GCU_CUDA(cudaStreamSynchronize(st));
  GCU_CUDA(cudaMemcpy(hbuf.data(), dbuf, rec * c.world, cudaMemcpyDeviceToHost));
  int all_ok = 1;
  for (int p = 0; p < c.world; ++p) {
    int okp;
    memcpy(&okp, hbuf.data() + rec * p, sizeof(int));
    all_ok &= okp;
  }
  for (int p = 0; p < c.world && all_ok; ++p) {
    if (p == c.rank) {
      c.peer_sym[p] = c.sym;
      c.peer_flags[p] = c.flags;
      continue;
    }
    cudaIpcMemHandle_t hp[2];
    memcpy(hp, hbuf.data() + rec * p + 4 * sizeof(int), sizeof(hp));
    void *a = nullptr, *b = nullptr;
    if (cudaIpcOpenMemHandle(&a, hp[0], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess ||
        cudaIpcOpenMemHandle(&b, hp[1], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      all_ok = 0;
      break;
    }
    c.peer_sym[p] = a;
    c.peer_flags[p] = static_cast<int *>(b);
  }
  // agree: p2p only if every rank mapped every peer
  memcpy(hbuf.data() + rec * c.rank, &all_ok, sizeof(int));
  GCU_CUDA(cudaMemcpy(dbuf + rec * c.rank, hbuf.data() + rec * c.rank, sizeof(int), cudaMemcpyHostToDevice));
  r = g_nccl.allGather(dbuf + rec * c.rank, dbuf, rec, ncclUint8, c.comm, st);
  if (r == ncclSuccess) {
    GCU_CUDA(cudaStreamSynchronize(st));
    GCU_CUDA(cudaMemcpy(hbuf.data(), dbuf, rec * c.world, cudaMemcpyDeviceToHost));
    for (int p = 0; p < c.world; ++p) {
      int okp;
      memcpy(&okp, hbuf.data() + rec * p, sizeof(int));
      all_ok &= okp;
    }
  } else {
    all_ok = 0;
  }
  cudaFree(dbuf);
  cudaStreamDestroy(st);
  c.p2p = all_ok != 0;
  return 0;
}

void teardown_p2p(Comm &c) {
  for (int p = 0; p < c.world && p < 8; ++p) {
    if (p != c.rank) {
      if (c.peer_sym[p]) cudaIpcCloseMemHandle(c.peer_sym[p]);
      if (c.peer_flags[p]) cudaIpcCloseMemHandle(c.peer_flags[p]);
    }
    c.peer_sym[p] = nullptr;
    c.peer_flags[p] = nullptr;
  }
  if (c.sym) cudaFree(c.sym);
  if (c.flags) cudaFree(c.flags);
  c.sym = nullptr;
  c.flags = nullptr;
  c.p2p = false;
}

}  // namespace
}  // namespace gcu

using namespace gcu;

GCU_EXPORT int gcu_comm_unique_id(unsigned char id[128]) {
  if (nccl()) return 1;
  ncclUniqueId u;
  ncclResult_t r = g_nccl.getUniqueId(&u);
  if (r != ncclSuccess) return nccl_err(r, "ncclGetUniqueId");
  memcpy(id, u.internal, 128);
  return 0;
}

GCU_EXPORT int gcu_comm_init(int rank, int world, const unsigned char id[128]) {
  if (nccl()) return 1;
  if (world < 1 || rank < 0 || rank >= world)
    return set_error("gcu_comm_init: rank %d of %d", rank, world);
  std::lock_guard<std::mutex> lk(g_comm_mu);
  if (g_comm.comm) return set_error("gcu_comm_init: already initialised");
  ncclUniqueId u;
  memcpy(u.internal, id, 128);
  ncclComm_t c = nullptr;
  ncclResult_t r = g_nccl.commInitRank(&c, world, u, rank);
  if (r != ncclSuccess) return nccl_err(r, "ncclCommInitRank");
  g_comm.comm = c;
  g_comm.rank = rank;
  g_comm.world = world;
  // all ranks synchronise here anyway (the NCCL init above is collective)
  if (setup_p2p(g_comm)) return 1;
  forget_error_code(DEV_TIMEOUT_PEER);  // fresh buffers and counters
  return 0;
}

// 1 if the row-shard entry point runs its all-gather as peer stores fused
// into the GEMV (every rank mapped every other rank's buffer), else 0.
GCU_EXPORT int gcu_comm_fused_allgather(void) { return g_comm.p2p ? 1 : 0; }

GCU_EXPORT int gcu_comm_destroy(void) {
  std::lock_guard<std::mutex> lk(g_comm_mu);
  if (!g_comm.comm) return 0;
  cudaDeviceSynchronize();
  teardown_p2p(g_comm);
  ncclResult_t r = g_nccl.commDestroy(g_comm.comm);
  g_comm.comm = nullptr;
  if (r != ncclSuccess) return nccl_err(r, "ncclCommDestroy");
  return 0;
}

// A rank whose fused all-gather gave up waiting for its peers (device code
// 6) leaves the arrival counters of every rank out of step: a late arrival
// would count toward the next launch, which could then read a half of a
// peer's buffer that is not yet written.  Row-sharded calls are therefore
// refused from then on, until gcu_comm_destroy and gcu_comm_init (on every
// rank) rebuild the buffers and counters.  They are refused rather than sent
// to NCCL: ranks that disagree on the path would wait for each other forever.
static int refuse_after_peer_timeout(const char *what) {
  if (error_codes_seen() & (1u << DEV_TIMEOUT_PEER))
    return set_error("%s: refused after a fused all-gather gave up waiting for a peer (device code %d); "
                     "call gcu_comm_destroy and gcu_comm_init on every rank",
                     what, (int)DEV_TIMEOUT_PEER);
  return 0;
}

// The fused all-gather's view of this rank's symmetric buffer and flags.
static PeerOut peer_out(int m) {
  PeerOut po{};
  for (int p = 0; p < g_comm.world; ++p) {
    po.delta[p] = (long long)((char *)g_comm.peer_sym[p] - (char *)g_comm.sym);
    po.flag_peer[p] = g_comm.peer_flags[p];
  }
  po.flag_local = g_comm.flags;
  po.sym = g_comm.sym;
  po.half_elems = (long)(kSymHalf / sizeof(float));
  po.mb = m;
  po.rank = g_comm.rank;
  po.world = g_comm.world;
  po.err = dev_error_word();
  return po;
}

GCU_EXPORT int gcu_dev_gemm_int8_rowshard(float *dst, float *work, const int8_t *mat_local,
                                          const float *matsc_local, const int8_t *src,
                                          const float *ssc, int m, int n, int k, void *stream) {
  if (!g_comm.comm) return set_error("gcu_dev_gemm_int8_rowshard: gcu_comm_init first");
  if (refuse_after_peer_timeout("gcu_dev_gemm_int8_rowshard")) return 1;
  const int world = g_comm.world, rank = g_comm.rank;
  if (n % world) return set_error("rowshard: n %d not divisible by world %d", n, world);
  if (m <= 0) return 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nl = n / world;
  if (m <= 8 && g_comm.p2p && (size_t)m * n * sizeof(float) <= kSymHalf && nl % 4 == 0 &&
      (uintptr_t)dst % 16 == 0) {
    // GEMV with the all-gather fused into it (NVLink loads from the peers)
    GemvJobs J{};
    J.w[0] = mat_local;
    J.ws[0] = matsc_local;
    J.row_end[0] = nl;
    J.njobs = 1;
    PeerOut po = peer_out(m);
    po.njobs = 1;
    po.n[0] = n;
    po.n_local[0] = nl;
    po.dst[0] = dst;
    return launch_gemv_p2p(J, src, k, ssc, nullptr, nullptr, nullptr, m, k, po, st);
  }
  // this rank's (m, nl) block, at its slot of the gather buffer
  float *mine = (m == 1 ? dst : work) + (size_t)rank * m * nl;
  if (m <= 8) {
    GemvJobs J{};
    J.w[0] = mat_local;
    J.ws[0] = matsc_local;
    J.y[0] = mine;
    J.row_end[0] = nl;
    J.njobs = 1;
    if (launch_gemv(J, src, k, ssc, m, nl, k, st)) return 1;
  } else {
    GemmArgs a{mine, nl, mat_local, k, matsc_local, src, k, ssc, m, nl, k};
    if (launch_gemm_tc(a, st, 0, 0)) return 1;
  }
  float *gather = m == 1 ? dst : work;
  ncclResult_t r = g_nccl.allGather(mine, gather, (size_t)m * nl, ncclFloat32, g_comm.comm, st);
  if (r != ncclSuccess) return nccl_err(r, "ncclAllGather");
  if (m > 1) {
    // [world][m][nl] -> [m][n]
    for (int g = 0; g < world; ++g)
      GCU_CUDA(cudaMemcpy2DAsync(dst + (size_t)g * nl, (size_t)n * 4, work + (size_t)g * m * nl,
                                 (size_t)nl * 4, (size_t)nl * 4, m, cudaMemcpyDeviceToDevice, st));
  }
  return 0;
}

GCU_EXPORT int gcu_dev_quantize_gemm_int8_rowshard_multi(const gcu_gemv_job *jobs, int njobs,
                                                         int8_t *q, float *s, const float *x,
                                                         int xstr, int m, int k, float *work,
                                                         void *stream) {
  if (!g_comm.comm) return set_error("gcu_dev_quantize_gemm_int8_rowshard_multi: gcu_comm_init first");
  if (refuse_after_peer_timeout("gcu_dev_quantize_gemm_int8_rowshard_multi")) return 1;
  if (njobs < 1 || njobs > GCU_MAX_JOBS)
    return set_error("quantize_gemm_rowshard_multi: 1..%d jobs (got %d)", GCU_MAX_JOBS, njobs);
  if (m <= 0) return 0;
  if (k <= 0) return set_error("quantize_gemm_rowshard_multi: k must be positive (got %d)", k);
  if (xstr == 0) xstr = k;
  const int world = g_comm.world;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  size_t total = 0;
  bool fused = m <= 8 && g_comm.p2p && k % 16 == 0;
  for (int j = 0; j < njobs; ++j) {
    const int n = jobs[j].m;
    if (n <= 0 || n % world) return set_error("quantize_gemm_rowshard_multi: job %d rows %d not a positive "
                                              "multiple of world %d", j, n, world);
    total += (size_t)m * n * sizeof(float);
    fused = fused && (n / world) % 4 == 0 && (uintptr_t)jobs[j].dst % 16 == 0;
  }
  fused = fused && total <= kSymHalf;
  if (fused) {
    GemvJobs J{};
    PeerOut po = peer_out(m);
    long off = 0;
    int rows = 0;
    for (int j = 0; j < njobs; ++j) {
      const int n = jobs[j].m, nl = n / world;
      J.w[j] = static_cast<const int8_t *>(jobs[j].w);
      J.ws[j] = jobs[j].sc;
      rows += nl;
      J.row_end[j] = rows;
      po.off[j] = off;
      po.n[j] = n;
      po.n_local[j] = nl;
      po.dst[j] = jobs[j].dst;
      off += (long)m * n;
    }
    J.njobs = njobs;
    po.njobs = njobs;
    return launch_gemv_p2p(J, nullptr, xstr, nullptr, x, q, s, m, k, po, st);
  }
  // quantize once, then every job through the row-shard entry point
  if (launch_quantize_rows(q, s, x, xstr, m, k, st)) return 1;
  for (int j = 0; j < njobs; ++j)
    if (gcu_dev_gemm_int8_rowshard(jobs[j].dst, work, static_cast<const int8_t *>(jobs[j].w), jobs[j].sc,
                                   q, s, m, jobs[j].m, k, stream))
      return 1;
  return 0;
}

// ---------------------------------------------------------------------------
// Gemma's feed-forward block over a hidden dimension sharded across the ranks
// ---------------------------------------------------------------------------
namespace gcu {
namespace {

// out[r][c] = (float)acc[r][c] * (hs[r] * ws[c]): the dequant of gemm_int8
// (gemma.c:3859-3862 under -ffast-math), on int32 sums summed over the ranks
__global__ void k_dequant_i32(float *__restrict__ out, const int *__restrict__ acc,
                              const float *__restrict__ hs, const float *__restrict__ ws, int m, int n) {
  const long total = (long)m * n;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int r = (int)(i / n), c = (int)(i - (long)r * n);
    out[i] = __fmul_rn(__int2float_rn(acc[i]), __fmul_rn(__ldg(hs + r), __ldg(ws + c)));
  }
}

// per-device scratch of the FFN entry point (grown, never shrunk)
struct FfnScratch {
  void *p = nullptr;
  size_t cap = 0;
};
std::mutex g_ffn_mu;
FfnScratch g_ffn[64];

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

}  // namespace
}  // namespace gcu

// Gemma's FFN for m > 8 tokens (gemma.c:5365-5391 and the GeGLU between,
// 4139-4170), the hidden dimension `ffn` split over the ranks of gcu_comm_init:
// rank r holds rows [r*fl, (r+1)*fl) of the up and gate weights (fl =
// ffn/world) and the same columns of the down weight (a [dim][fl] slice with
// row stride w_down_stride bytes).  Every rank computes its slice of up and
// gate, h = gelu(gate)*up on it, and the row maxima of h over its slice; an
// all-reduce(max) gives every rank the maxima of the full rows, so each
// quantizes its slice into exactly the codes and scales of the unsharded
// quantize_acts; its K slice of the down projection gives int32 partial sums,
// an all-reduce(sum) adds them -- integer addition is exact -- and one
// dequant forms out [m][dim], the same on every rank and bit for bit the
// unsharded block's.  The collectives move m floats and m*dim int32 values
// instead of the 2*m*ffn floats of gathering up and gate.  With one rank (or
// none initialised) the same block runs unsharded.
GCU_EXPORT int gcu_dev_ffn_rowshard(float *out, const int8_t *xq, const float *xs, int m, int dim,
                                    int ffn, const int8_t *w_up, const float *s_up,
                                    const int8_t *w_gate, const float *s_gate,
                                    const int8_t *w_down, int w_down_stride, const float *s_down,
                                    void *stream) {
  const int world = g_comm.comm ? g_comm.world : 1;
  if (g_comm.comm && refuse_after_peer_timeout("gcu_dev_ffn_rowshard")) return 1;
  if (m <= 8) return set_error("gcu_dev_ffn_rowshard: m %d (needs m > 8: tensor-core path)", m);
  if (dim <= 0 || ffn <= 0 || ffn % world)
    return set_error("gcu_dev_ffn_rowshard: ffn %d not a positive multiple of world %d", ffn, world);
  const int fl = ffn / world;
  if (fl % 16 || dim % 16) return set_error("gcu_dev_ffn_rowshard: ffn/world %d and dim %d must be multiples of 16", fl, dim);
  if (w_down_stride == 0) w_down_stride = fl;
  if (w_down_stride < fl || w_down_stride % 16) return set_error("gcu_dev_ffn_rowshard: bad down stride %d", w_down_stride);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int dev = calling_device();
  if (dev < 0 || dev >= 64) return set_error("gcu_dev_ffn_rowshard: device %d", dev);
  // scratch: up, h (over gate), row maxima, codes, scales, int32 sums
  const size_t b_up = align256((size_t)m * fl * 4), b_amax = align256((size_t)m * 4),
               b_q = align256((size_t)m * fl), b_acc = align256((size_t)m * dim * 4);
  const size_t need = 2 * b_up + 2 * b_amax + b_q + b_acc;
  char *base;
  {
    std::lock_guard<std::mutex> lk(g_ffn_mu);
    FfnScratch &fs = g_ffn[dev];
    if (fs.cap < need) {
      if (fs.p) {
        GCU_CUDA(cudaStreamSynchronize(st));
        cudaFree(fs.p);
      }
      fs.p = nullptr;
      fs.cap = 0;
      GCU_CUDA(cudaMalloc(&fs.p, need));
      fs.cap = need;
    }
    base = static_cast<char *>(fs.p);
  }
  float *up = reinterpret_cast<float *>(base);
  float *gate = reinterpret_cast<float *>(base + b_up);
  float *amax = reinterpret_cast<float *>(base + 2 * b_up);
  float *hs = reinterpret_cast<float *>(base + 2 * b_up + b_amax);
  int8_t *hq = reinterpret_cast<int8_t *>(base + 2 * b_up + 2 * b_amax);
  int *acc = reinterpret_cast<int *>(base + 2 * b_up + 2 * b_amax + b_q);
  // 1. this rank's slice of up (w1) and gate (w2), one launch
  GemmArgs jobs[2] = {};
  jobs[0] = GemmArgs{up, fl, w_up, dim, s_up, xq, dim, xs, m, fl, dim};
  jobs[1] = GemmArgs{gate, fl, w_gate, dim, s_gate, xq, dim, xs, m, fl, dim};
  if (launch_gemm_tc_jobs(xq, dim, xs, m, dim, jobs, 2, st, 0, 0)) return 1;
  if (world == 1) {
    // 2-4 unsharded: the fused GeGLU + quantize, the down projection with its dequant
    if (gcu_dev_geglu_quantize(hq, hs, nullptr, gate, up, m, fl, stream)) return 1;
    GemmArgs a{out, dim, w_down, w_down_stride, s_down, hq, fl, hs, m, dim, fl};
    return launch_gemm_tc(a, st, 0, 0);
  }
  // 2. h = gelu(gate)*up over the slice (in place of gate), row maxima of the slice
  if (launch_geglu_amax(gate, amax, gate, up, m, fl, st)) return 1;
  // 3. maxima of the full rows: every rank now forms the unsharded codes
  ncclResult_t r = g_nccl.allReduce(amax, amax, (size_t)m, ncclFloat32, ncclMax, g_comm.comm, st);
  if (r != ncclSuccess) return nccl_err(r, "ncclAllReduce (row maxima)");
  if (launch_quantize_given_amax(hq, hs, gate, amax, m, fl, st)) return 1;
  // 4. this rank's K slice of down: int32 partial sums, summed over the ranks
  GemmArgs d{reinterpret_cast<float *>(acc), dim, w_down, w_down_stride, nullptr, hq, fl, nullptr, m, dim, fl};
  d.raw = 1;
  if (launch_gemm_tc_jobs(hq, fl, nullptr, m, fl, &d, 1, st, 0, 0)) return 1;
  r = g_nccl.allReduce(acc, acc, (size_t)m * dim, ncclInt32, ncclSum, g_comm.comm, st);
  if (r != ncclSuccess) return nccl_err(r, "ncclAllReduce (int32 partial sums)");
  // 5. one dequant of the summed int32 values
  const long total = (long)m * dim;
  const int grid = (int)std::min<long>((total + 255) / 256, (long)num_sms() * 8);
  k_dequant_i32<<<grid, 256, 0, st>>>(out, acc, hs, s_down, m, dim);
  GCU_CUDA(cudaGetLastError());
  return 0;
}
