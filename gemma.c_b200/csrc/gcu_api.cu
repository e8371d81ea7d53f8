// gcu_api.cu -- runtime of libgcu.so: errors, per-thread streams and staging,
// the weight registry, and the exported host- and device-pointer entry points
// declared in include/gcu.h.
//
// The host entry points keep gemma.c's calling convention: host pointers in,
// results in host memory on return (gemma.c:2590, 2656, 2770, 2818, 3943).
// Weights are uploaded once at registration; any interior pointer of a
// registered range (gemma.c:5080-5086 passes w->i8.q + hd*hdim*dim) maps to
// the same offset of the device copy.
#include "gcu_internal.cuh"

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <atomic>
#include <mutex>
#include <shared_mutex>
#include <unordered_map>
#include <vector>

#define GCU_EXPORT extern "C" __attribute__((visibility("default")))

namespace gcu {

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------
static thread_local char t_err[256] = {0};

int set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
  return 1;
}

int check_cuda(cudaError_t e, const char *what) {
  return set_error("%s: %s", what, cudaGetErrorString(e));
}

// ---------------------------------------------------------------------------
// per-device state
// ---------------------------------------------------------------------------
__device__ unsigned int g_dev_err;

static thread_local int t_device = -1;

static int current_device() {
  if (t_device < 0) {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) d = 0;
    t_device = d;
  }
  return t_device;
}

// The device error word.  Two homes: a __device__ variable (looked up with no
// allocation, for callers that never set up the library), and once gcu_init
// or a host entry point has run on the device, a word of mapped pinned host
// memory, which kernels write directly and host calls read after their
// stream wait without a device-to-host copy (each copy costs ~10 us here).
struct DeviceInfo {
  int sms = 0;
  unsigned int *err_sym = nullptr;              // device variable
  unsigned int *err_map = nullptr;              // mapped host word, device view
  volatile unsigned int *err_host = nullptr;    // the same word, host view
};
static std::mutex g_dev_mu;
static std::unordered_map<int, DeviceInfo> g_dev;

static DeviceInfo &device_info() {
  const int d = current_device();
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo &di = g_dev[d];
  if (di.sms == 0) {
    cudaDeviceGetAttribute(&di.sms, cudaDevAttrMultiProcessorCount, d);
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_dev_err) == cudaSuccess) di.err_sym = (unsigned int *)p;
  }
  return di;
}

// Create the mapped host error word of the calling thread's device (once).
static int map_error_word() {
  const int d = current_device();
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo &di = g_dev[d];
  if (di.err_map) return 0;
  void *h = nullptr, *dp = nullptr;
  GCU_CUDA(cudaHostAlloc(&h, 64, cudaHostAllocMapped | cudaHostAllocPortable));
  memset(h, 0, 64);
  if (cudaHostGetDevicePointer(&dp, h, 0) != cudaSuccess) {
    cudaFreeHost(h);
    return set_error("cudaHostGetDevicePointer failed for the error word");
  }
  di.err_host = static_cast<volatile unsigned int *>(h);
  di.err_map = static_cast<unsigned int *>(dp);
  return 0;
}

// Every nonzero code the host has observed (bit `code`), whoever read it:
// a call that must not run after a given failure checks this.
static std::atomic<unsigned int> g_codes_seen{0};

unsigned int error_codes_seen() {
  DeviceInfo &di = device_info();
  if (di.err_host) {
    const unsigned int code = *di.err_host;  // peek: a later check still reports it
    if (code && code < 32) g_codes_seen.fetch_or(1u << code);
  }
  return g_codes_seen.load();
}

void forget_error_code(unsigned int code) {
  if (code < 32) g_codes_seen.fetch_and(~(1u << code));
}

// Read and clear every home of the error word (device variable by copy).
static unsigned int take_error_code(bool read_symbol) {
  DeviceInfo &di = device_info();
  unsigned int code = 0;
  if (di.err_host) {
    code = *di.err_host;
    if (code) *di.err_host = 0;
  }
  if (read_symbol && di.err_sym) {
    unsigned int c2 = 0;
    if (cudaMemcpy(&c2, di.err_sym, sizeof(c2), cudaMemcpyDeviceToHost) == cudaSuccess && c2) {
      unsigned int zero = 0;
      cudaMemcpy(di.err_sym, &zero, sizeof(zero), cudaMemcpyHostToDevice);
      if (!code) code = c2;
    }
  }
  if (code && code < 32) g_codes_seen.fetch_or(1u << code);
  return code;
}

int num_sms() { return device_info().sms; }

bool pdl_enabled() {
  static const bool on = [] {
    const char *e = getenv("GCU_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}
unsigned int *dev_error_word() {
  DeviceInfo &di = device_info();
  return di.err_map ? di.err_map : di.err_sym;
}

// ---------------------------------------------------------------------------
// per-thread context: stream and device buffers for the host entry points
// ---------------------------------------------------------------------------
struct DevBuf {
  void *p = nullptr;
  size_t cap = 0;
  int get(size_t bytes, void **out) {
    if (bytes > cap) {
      if (p) cudaFree(p);
      p = nullptr;
      cap = 0;
      size_t want = bytes + bytes / 4 + 256;
      GCU_CUDA(cudaMalloc(&p, want));
      cap = want;
    }
    *out = p;
    return 0;
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
  }
};

// Mapped pinned host memory that kernels read or write directly over PCIe
// (zero-copy).  The host entry points pass per-row scales this way: a 2 KB
// vector costs a host memcpy instead of a copy-engine transfer, and every
// transfer costs ~10 us of fixed latency on these machines.
struct MappedBuf {
  void *h = nullptr;  // host view
  void *d = nullptr;  // device view
  size_t cap = 0;
  int get(size_t bytes) {
    if (bytes <= cap) return 0;
    if (h) cudaFreeHost(h);
    h = d = nullptr;
    cap = 0;
    const size_t want = bytes + bytes / 4 + 256;
    GCU_CUDA(cudaHostAlloc(&h, want, cudaHostAllocMapped | cudaHostAllocPortable));
    if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess) {
      cudaFreeHost(h);
      h = nullptr;
      return set_error("cudaHostGetDevicePointer failed for a scale buffer");
    }
    cap = want;
    return 0;
  }
  void release() {
    if (h) cudaFreeHost(h);
    h = d = nullptr;
    cap = 0;
  }
};

// Host entry points that move several MB split their rows into chunks and
// pipeline them: chunk i's host->device copy (stream s_in), its kernel
// (stream), and its device->host copy (s_out) overlap chunk i+1's, so the
// two PCIe directions and the GPU work at the same time.
constexpr int kMaxChunks = 4;
// smaller transfers go in one piece: every transfer or launch costs ~10 us
// of fixed latency on these machines, more than overlapping saves below this
constexpr size_t kChunkMinBytes = 4u << 20;

struct ThreadCtx {
  int device = -1;
  cudaStream_t stream = nullptr;  // kernels (and everything of unchunked calls)
  cudaStream_t s_in = nullptr, s_out = nullptr;
  cudaEvent_t ev_in[kMaxChunks] = {}, ev_done[kMaxChunks] = {};
  DevBuf in, in2, out, sc, sc2, wtmp, wstmp;
  MappedBuf hs;  // per-row scales, read or written by the kernels in place
  ~ThreadCtx() {
    // process teardown may already have unloaded the driver: leak quietly
  }
};
static thread_local ThreadCtx t_ctx;

static int ctx(ThreadCtx **out) {
  const int d = current_device();
  ThreadCtx &c = t_ctx;
  if (c.device != d || c.stream == nullptr) {
    GCU_CUDA(cudaSetDevice(d));
    GCU_CUDA(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking));
    GCU_CUDA(cudaStreamCreateWithFlags(&c.s_in, cudaStreamNonBlocking));
    GCU_CUDA(cudaStreamCreateWithFlags(&c.s_out, cudaStreamNonBlocking));
    for (int i = 0; i < kMaxChunks; ++i) {
      GCU_CUDA(cudaEventCreateWithFlags(&c.ev_in[i], cudaEventDisableTiming));
      GCU_CUDA(cudaEventCreateWithFlags(&c.ev_done[i], cudaEventDisableTiming));
    }
    if (map_error_word()) return 1;
    c.device = d;
  }
  *out = &c;
  return 0;
}

// Copy `height` rows of `width` bytes between pitched buffers; one linear
// copy when both sides are dense (a pitched copy may be run row by row).
static cudaError_t copy_rows(void *dst, size_t dpitch, const void *src, size_t spitch, size_t width,
                             size_t height, cudaMemcpyKind kind, cudaStream_t st) {
  if (height == 1 || (dpitch == width && spitch == width))
    return cudaMemcpyAsync(dst, src, width * height, kind, st);
  return cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, height, kind, st);
}

// Rows per pipeline chunk for a call moving `bytes_per_row` bytes per row in
// its larger direction: one chunk below kChunkMinBytes, else up to
// kMaxChunks chunks, rounded up to a multiple of `align` rows.
static int chunk_rows(int m, size_t bytes_per_row, int align) {
  const size_t total = (size_t)m * bytes_per_row;
  if (total < kChunkMinBytes || m < 2 * align) return m;
  size_t chunks = total / (kChunkMinBytes / 4);
  if (chunks > (size_t)kMaxChunks) chunks = kMaxChunks;
  int rows = (int)((m + chunks - 1) / chunks);
  rows = (rows + align - 1) / align * align;
  return rows < m ? rows : m;
}

// ---------------------------------------------------------------------------
// split-K workspace, one per (device, stream): launches on one stream are
// ordered, so they can share it; different streams never do.
// ---------------------------------------------------------------------------
struct Workspace {
  void *ws = nullptr;
  size_t ws_cap = 0;
  int *cnt = nullptr;
  int cnt_cap = 0;
};
static std::mutex g_ws_mu;
static std::map<std::pair<int, cudaStream_t>, Workspace> g_ws;

int gemm_workspace(size_t bytes, void **ws, int **counters, int ncounters, cudaStream_t st) {
  std::lock_guard<std::mutex> lk(g_ws_mu);
  Workspace &w = g_ws[{current_device(), st}];
  if (bytes > w.ws_cap) {
    if (w.ws) {
      GCU_CUDA(cudaStreamSynchronize(st));
      cudaFree(w.ws);
    }
    w.ws = nullptr;
    w.ws_cap = 0;
    size_t want = bytes < ((size_t)16 << 20) ? ((size_t)16 << 20) : bytes;
    GCU_CUDA(cudaMalloc(&w.ws, want));
    w.ws_cap = want;
  }
  if (ncounters > w.cnt_cap) {
    if (w.cnt) {
      GCU_CUDA(cudaStreamSynchronize(st));
      cudaFree(w.cnt);
    }
    w.cnt = nullptr;
    w.cnt_cap = 0;
    int want = ncounters < 4096 ? 4096 : ncounters;
    GCU_CUDA(cudaMalloc(&w.cnt, (size_t)want * sizeof(int)));
    GCU_CUDA(cudaMemsetAsync(w.cnt, 0, (size_t)want * sizeof(int), st));
    w.cnt_cap = want;
  }
  *ws = w.ws;
  *counters = w.cnt;
  return 0;
}

// ---------------------------------------------------------------------------
// weight registry
// ---------------------------------------------------------------------------
struct WeightEntry {
  uintptr_t q0, q1;  // host range of the int8 values
  uintptr_t s0, s1;  // host range of the scales
  int8_t *dq;
  float *ds;
  int rows, k;
  int arena;  // 0: dq/ds are the entry's own allocations; else the arena holding them
};
// one device allocation holding many registered weights (gcu_register_qtensors)
struct Arena {
  int device;
  void *base;
  size_t bytes;
  std::vector<uintptr_t> keys;  // q begins of its entries
};
static std::shared_mutex g_reg_mu;
// keyed by (device, host begin)
static std::map<std::pair<int, uintptr_t>, WeightEntry> g_q;
static std::map<std::pair<int, uintptr_t>, uintptr_t> g_s;  // scales begin -> q begin
static std::map<int, Arena> g_arenas;
static int g_next_arena = 1;
static size_t g_reg_bytes = 0;

int calling_device() { return current_device(); }

// true if [p, p+bytes) meets a registered range of kind Q (int8) or S
// (scales) on device d; the caller holds g_reg_mu
static bool overlaps_locked(int d, uintptr_t a, size_t bytes, bool q) {
  if (q) {
    auto it = g_q.lower_bound({d, a + bytes});
    if (it == g_q.begin()) return false;
    --it;
    return it->first.first == d && it->second.q1 > a;
  }
  auto it = g_s.lower_bound({d, a + bytes});
  if (it == g_s.begin()) return false;
  --it;
  return it->first.first == d && g_q.at({d, it->second}).s1 > a;
}

int registry_add_arena(const RegRec *recs, int n, void *base, size_t bytes, int *arena_id) {
  const int d = current_device();
  std::unique_lock<std::shared_mutex> lk(g_reg_mu);
  for (int i = 0; i < n; ++i) {
    const size_t qb = (size_t)recs[i].rows * recs[i].k, sb = (size_t)recs[i].rows * sizeof(float);
    if (overlaps_locked(d, recs[i].q, qb, true) || overlaps_locked(d, recs[i].s, sb, false))
      return set_error("register_qtensors: tensor %d overlaps a registered weight", i);
  }
  const int id = g_next_arena++;
  Arena &ar = g_arenas[id];
  ar = Arena{d, base, bytes, {}};
  for (int i = 0; i < n; ++i) {
    const RegRec &r = recs[i];
    const size_t qb = (size_t)r.rows * r.k, sb = (size_t)r.rows * sizeof(float);
    WeightEntry e{r.q, r.q + qb, r.s, r.s + sb, (int8_t *)base + r.dq_off,
                  (float *)((char *)base + r.ds_off), r.rows, r.k, id};
    g_q[{d, e.q0}] = e;
    g_s[{d, e.s0}] = e.q0;
    ar.keys.push_back(e.q0);
  }
  g_reg_bytes += bytes;
  if (arena_id) *arena_id = id;
  return 0;
}

// device address for host range [p, p+bytes) inside a registered weight
static const void *lookup_q(const void *p, size_t bytes) {
  const int d = current_device();
  const uintptr_t a = (uintptr_t)p;
  std::shared_lock<std::shared_mutex> lk(g_reg_mu);
  auto it = g_q.upper_bound({d, a});
  if (it == g_q.begin()) return nullptr;
  --it;
  if (it->first.first != d) return nullptr;
  const WeightEntry &e = it->second;
  if (a < e.q0 || a + bytes > e.q1) return nullptr;
  return e.dq + (a - e.q0);
}
static const float *lookup_s(const float *p, size_t count) {
  const int d = current_device();
  const uintptr_t a = (uintptr_t)p;
  std::shared_lock<std::shared_mutex> lk(g_reg_mu);
  auto it = g_s.upper_bound({d, a});
  if (it == g_s.begin()) return nullptr;
  --it;
  if (it->first.first != d) return nullptr;
  const WeightEntry &e = g_q.at({d, it->second});
  if (a < e.s0 || a + count * sizeof(float) > e.s1) return nullptr;
  return e.ds + (a - e.s0) / sizeof(float);
}

// Device pointer of a weight operand: registered copy, else a transient
// upload into the thread's buffer (correct, but pays the copy every call).
static int weight_dev(ThreadCtx *c, DevBuf &buf, const void *host, size_t bytes,
                      const void **dev) {
  if ((*dev = lookup_q(host, bytes)) != nullptr) return 0;
  void *p;
  if (buf.get(bytes, &p)) return 1;
  GCU_CUDA(cudaMemcpyAsync(p, host, bytes, cudaMemcpyHostToDevice, c->stream));
  *dev = p;
  return 0;
}
static int scales_dev(ThreadCtx *c, DevBuf &buf, const float *host, size_t count,
                      const float **dev) {
  if ((*dev = lookup_s(host, count)) != nullptr) return 0;
  void *p;
  if (buf.get(count * sizeof(float), &p)) return 1;
  GCU_CUDA(cudaMemcpyAsync(p, host, count * sizeof(float), cudaMemcpyHostToDevice, c->stream));
  *dev = (const float *)p;
  return 0;
}

// Wait for `st`, the last stream of a host call, and report a device-side
// error word set by its kernels.  The host entry points run with the mapped
// error word (ctx() creates it), which the kernels wrote before the stream's
// work completed: reading it after the wait needs no copy.
static int sync_and_check(ThreadCtx *c, cudaStream_t st) {
  (void)c;
  GCU_CUDA(cudaStreamSynchronize(st));
  const unsigned int code = take_error_code(false);
  if (code) return set_error("device-side wait gave up (code %u)", code);
  return 0;
}
static int sync_and_check(ThreadCtx *c) { return sync_and_check(c, c->stream); }

static inline cudaStream_t as_stream(void *s) { return static_cast<cudaStream_t>(s); }

// Enqueue y = gemm on device operands, choosing the kernel by m.
static int dev_gemm(float *dst, long dstr, const int8_t *mat, long mstr, const float *matsc,
                    const int8_t *src, long sstr, const float *ssc, int m, int n, int k,
                    cudaStream_t st) {
  if (m <= 8) {
    if (mstr != k)
      return set_error("gemm: m <= 8 needs dense weight rows (mstr %ld, k %d)", mstr, k);
    GemvJobs jobs{};
    jobs.w[0] = mat;
    jobs.ws[0] = matsc;
    jobs.y[0] = dst;
    jobs.row_end[0] = n;
    jobs.njobs = 1;
    return launch_gemv(jobs, src, sstr, ssc, m, dstr, k, st);
  }
  GemmArgs a{dst, dstr, mat, mstr, matsc, src, sstr, ssc, m, n, k};
  return launch_gemm_tc(a, st, 0, 0);
}

}  // namespace gcu

using namespace gcu;

// ===========================================================================
// exported entry points
// ===========================================================================
GCU_EXPORT const char *gcu_version(void) { return "gcu 0.1 sm_100a"; }

GCU_EXPORT const char *gcu_last_error(void) { return t_err; }

GCU_EXPORT int gcu_init(int device) {
  int n = 0;
  GCU_CUDA(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n) return set_error("gcu_init: device %d of %d", device, n);
  GCU_CUDA(cudaSetDevice(device));
  t_device = device;
  device_info();
  return map_error_word();
}

GCU_EXPORT int gcu_check_device(void) {
  GCU_CUDA(cudaDeviceSynchronize());
  const unsigned int code = take_error_code(true);
  if (code) {
    set_error("device-side wait gave up (code %u)", code);
    return 1;
  }
  return 0;
}

GCU_EXPORT int gcu_register_weight(const int8_t *q, const float *scales, int rows, int k) {
  if (!q || !scales || rows <= 0 || k <= 0) return set_error("gcu_register_weight: bad arguments");
  const int d = current_device();
  GCU_CUDA(cudaSetDevice(d));
  {
    std::shared_lock<std::shared_mutex> lk(g_reg_mu);
    if (g_q.count({d, (uintptr_t)q})) return 0;  // already registered
  }
  const size_t qb = (size_t)rows * k, sb = (size_t)rows * sizeof(float);
  {
    std::shared_lock<std::shared_mutex> lk(g_reg_mu);
    if (overlaps_locked(d, (uintptr_t)q, qb, true) || overlaps_locked(d, (uintptr_t)scales, sb, false))
      return set_error("gcu_register_weight: overlaps a registered weight");
  }
  WeightEntry e{(uintptr_t)q, (uintptr_t)q + qb, (uintptr_t)scales, (uintptr_t)scales + sb,
                nullptr, nullptr, rows, k, 0};
  GCU_CUDA(cudaMalloc(&e.dq, qb));
  if (cudaMalloc(&e.ds, sb) != cudaSuccess) {
    cudaFree(e.dq);
    return set_error("gcu_register_weight: out of device memory");
  }
  cudaError_t r1 = cudaMemcpy(e.dq, q, qb, cudaMemcpyHostToDevice);
  cudaError_t r2 = cudaMemcpy(e.ds, scales, sb, cudaMemcpyHostToDevice);
  if (r1 != cudaSuccess || r2 != cudaSuccess) {
    cudaFree(e.dq);
    cudaFree(e.ds);
    return check_cuda(r1 != cudaSuccess ? r1 : r2, "gcu_register_weight upload");
  }
  std::unique_lock<std::shared_mutex> lk(g_reg_mu);
  g_q[{d, e.q0}] = e;
  g_s[{d, e.s0}] = e.q0;
  g_reg_bytes += qb + sb;
  return 0;
}

GCU_EXPORT int gcu_unregister_weight(const int8_t *q) {
  const int d = current_device();
  std::unique_lock<std::shared_mutex> lk(g_reg_mu);
  auto it = g_q.find({d, (uintptr_t)q});
  if (it == g_q.end()) return set_error("gcu_unregister_weight: not registered");
  if (it->second.arena)
    return set_error("gcu_unregister_weight: part of arena %d (gcu_unregister_arena)", it->second.arena);
  WeightEntry e = it->second;
  g_q.erase(it);
  g_s.erase({d, e.s0});
  g_reg_bytes -= (size_t)e.rows * e.k + (size_t)e.rows * sizeof(float);
  cudaDeviceSynchronize();
  cudaFree(e.dq);
  cudaFree(e.ds);
  return 0;
}

GCU_EXPORT int gcu_unregister_arena(int arena) {
  std::unique_lock<std::shared_mutex> lk(g_reg_mu);
  auto it = g_arenas.find(arena);
  if (it == g_arenas.end()) return set_error("gcu_unregister_arena: no arena %d", arena);
  Arena ar = it->second;
  g_arenas.erase(it);
  for (uintptr_t key : ar.keys) {
    auto e = g_q.find({ar.device, key});
    if (e == g_q.end()) continue;
    g_s.erase({ar.device, e->second.s0});
    g_q.erase(e);
  }
  g_reg_bytes -= ar.bytes;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(ar.device);
  cudaDeviceSynchronize();
  cudaFree(ar.base);
  cudaSetDevice(prev);
  return 0;
}

GCU_EXPORT size_t gcu_registered_bytes(void) {
  std::shared_lock<std::shared_mutex> lk(g_reg_mu);
  return g_reg_bytes;
}

GCU_EXPORT int gcu_shutdown(void) {
  cudaDeviceSynchronize();
  {
    std::unique_lock<std::shared_mutex> lk(g_reg_mu);
    for (auto &kv : g_q) {
      if (kv.second.arena) continue;
      cudaFree(kv.second.dq);
      cudaFree(kv.second.ds);
    }
    for (auto &kv : g_arenas) cudaFree(kv.second.base);
    g_q.clear();
    g_s.clear();
    g_arenas.clear();
    g_reg_bytes = 0;
  }
  {
    std::lock_guard<std::mutex> lk(g_ws_mu);
    for (auto &kv : g_ws) {
      cudaFree(kv.second.ws);
      cudaFree(kv.second.cnt);
    }
    g_ws.clear();
  }
  release_staging();
  ThreadCtx &c = t_ctx;
  c.in.release();
  c.in2.release();
  c.out.release();
  c.sc.release();
  c.sc2.release();
  c.wtmp.release();
  c.wstmp.release();
  c.hs.release();
  if (c.stream) {
    cudaStreamDestroy(c.stream);
    cudaStreamDestroy(c.s_in);
    cudaStreamDestroy(c.s_out);
    for (int i = 0; i < kMaxChunks; ++i) {
      cudaEventDestroy(c.ev_in[i]);
      cudaEventDestroy(c.ev_done[i]);
    }
  }
  c.stream = c.s_in = c.s_out = nullptr;
  c.device = -1;
  return 0;
}

// ---- host-pointer entry points ---------------------------------------------

GCU_EXPORT int gcu_quantize_acts(int8_t *dst, float *dsc, const float *src, int sstr, int m,
                                 int n) {
  if (m <= 0 || n <= 0) return 0;
  if (!dst || !dsc || !src) return set_error("gcu_quantize_acts: null pointer");
  if (sstr == 0) sstr = n;
  if (sstr < n) return set_error("gcu_quantize_acts: sstr %d < n %d", sstr, n);
  ThreadCtx *c;
  if (ctx(&c)) return 1;
  const size_t in_elems = (size_t)(m - 1) * sstr + n;
  // (the scales come back by a transfer too: kernel writes into mapped host
  // memory would queue behind the previous chunk's copy and delay the kernel)
  void *din, *dout, *dsc_v;
  if (c->in.get(in_elems * 4, &din) || c->out.get((size_t)m * n, &dout) ||
      c->sc.get((size_t)m * 4, &dsc_v))
    return 1;
  float *dsc_d = static_cast<float *>(dsc_v);
  const int rows = chunk_rows(m, (size_t)sstr * 4, 1);
  const bool piped = rows < m;
  cudaStream_t s_in = piped ? c->s_in : c->stream, s_out = piped ? c->s_out : c->stream;
  for (int r0 = 0, i = 0; r0 < m; r0 += rows, ++i) {
    const int mr = m - r0 < rows ? m - r0 : rows;
    const size_t off = (size_t)r0 * sstr;
    const size_t elems = (size_t)(mr - 1) * sstr + n;
    GCU_CUDA(cudaMemcpyAsync((float *)din + off, src + off, elems * 4, cudaMemcpyHostToDevice, s_in));
    if (piped) {
      GCU_CUDA(cudaEventRecord(c->ev_in[i], s_in));
      GCU_CUDA(cudaStreamWaitEvent(c->stream, c->ev_in[i], 0));
    }
    if (launch_quantize_rows((int8_t *)dout + (size_t)r0 * n, dsc_d + r0,
                             (const float *)din + off, sstr, mr, n, c->stream))
      return 1;
    if (piped) {
      GCU_CUDA(cudaEventRecord(c->ev_done[i], c->stream));
      GCU_CUDA(cudaStreamWaitEvent(s_out, c->ev_done[i], 0));
    }
    GCU_CUDA(cudaMemcpyAsync(dst + (size_t)r0 * n, (int8_t *)dout + (size_t)r0 * n, (size_t)mr * n,
                             cudaMemcpyDeviceToHost, s_out));
    GCU_CUDA(cudaMemcpyAsync(dsc + r0, dsc_d + r0, (size_t)mr * 4, cudaMemcpyDeviceToHost, s_out));
  }
  GCU_CUDA(cudaStreamSynchronize(s_out));
  return 0;
}

GCU_EXPORT float gcu_quantize_act(int8_t *dst, const float *vec, int dim) {
  float sc = NAN;
  if (gcu_quantize_acts(dst, &sc, vec, 0, 1, dim)) return NAN;
  return sc;
}

static int host_gemv_jobs(const gcu_gemv_job *jobs, int njobs, const int8_t *vec, float vsc,
                          int n) {
  if (njobs <= 0) return 0;
  if (njobs > GCU_MAX_JOBS) return set_error("gemv_int8_multi: at most %d jobs", GCU_MAX_JOBS);
  if (!vec || n <= 0) return set_error("gemv_int8: bad vector");
  ThreadCtx *c;
  if (ctx(&c)) return 1;
  GemvJobs J{};
  int rows = 0;
  size_t out_elems = 0;
  for (int j = 0; j < njobs; ++j) out_elems += jobs[j].m > 0 ? jobs[j].m : 0;
  void *dx, *dy;
  if (c->in.get((size_t)n + 16, &dx) || c->out.get(out_elems * 4 + 16, &dy) || c->hs.get(16))
    return 1;
  *static_cast<float *>(c->hs.h) = vsc;  // read by the kernel in place
  const void *dxs = c->hs.d;
  // weights of unregistered jobs share one transient buffer: size it once
  size_t wt = 0, st = 0;
  for (int j = 0; j < njobs; ++j) {
    if (!lookup_q(jobs[j].w, (size_t)jobs[j].m * n)) wt += (size_t)jobs[j].m * n + 16;
    if (!lookup_s(jobs[j].sc, (size_t)jobs[j].m)) st += (size_t)jobs[j].m * 4 + 16;
  }
  void *wbase = nullptr, *sbase = nullptr;
  if (wt && c->wtmp.get(wt, &wbase)) return 1;
  if (st && c->wstmp.get(st, &sbase)) return 1;
  size_t woff = 0, soff = 0, yoff = 0;
  for (int j = 0; j < njobs; ++j) {
    const int m = jobs[j].m;
    if (m <= 0) continue;
    const void *dw = lookup_q(jobs[j].w, (size_t)m * n);
    if (!dw) {
      void *p = (char *)wbase + woff;
      GCU_CUDA(cudaMemcpyAsync(p, jobs[j].w, (size_t)m * n, cudaMemcpyHostToDevice, c->stream));
      woff += ((size_t)m * n + 15) / 16 * 16;
      dw = p;
    }
    const float *ds = lookup_s(jobs[j].sc, (size_t)m);
    if (!ds) {
      void *p = (char *)sbase + soff;
      GCU_CUDA(cudaMemcpyAsync(p, jobs[j].sc, (size_t)m * 4, cudaMemcpyHostToDevice, c->stream));
      soff += ((size_t)m * 4 + 15) / 16 * 16;
      ds = (const float *)p;
    }
    J.w[J.njobs] = (const int8_t *)dw;
    J.ws[J.njobs] = ds;
    J.y[J.njobs] = (float *)dy + yoff;
    rows += m;
    J.row_end[J.njobs] = rows;
    J.njobs++;
    yoff += m;
  }
  GCU_CUDA(cudaMemcpyAsync(dx, vec, (size_t)n, cudaMemcpyHostToDevice, c->stream));
  if (launch_gemv(J, (const int8_t *)dx, 0, (const float *)dxs, 1, 0, n, c->stream)) return 1;
  yoff = 0;
  for (int j = 0; j < njobs; ++j) {
    if (jobs[j].m <= 0) continue;
    GCU_CUDA(cudaMemcpyAsync(jobs[j].dst, (float *)dy + yoff, (size_t)jobs[j].m * 4,
                             cudaMemcpyDeviceToHost, c->stream));
    yoff += jobs[j].m;
  }
  // the outputs are host memory the caller owns: wait for them
  GCU_CUDA(cudaStreamSynchronize(c->stream));
  return 0;
}

GCU_EXPORT int gcu_gemv_int8(float *dst, const int8_t *mat, const float *matsc, const int8_t *vec,
                             float vsc, int m, int n) {
  gcu_gemv_job j{mat, matsc, dst, m};
  return host_gemv_jobs(&j, 1, vec, vsc, n);
}

GCU_EXPORT int gcu_gemv_int8_multi(const gcu_gemv_job *jobs, int njobs, const int8_t *vec,
                                   float vsc, int n) {
  return host_gemv_jobs(jobs, njobs, vec, vsc, n);
}

GCU_EXPORT int gcu_gemm_int8(float *dst, int dstr, const int8_t *mat, int mstr,
                             const float *matsc, const int8_t *src, int sstr, const float *ssc,
                             int m, int n, int k) {
  if (m <= 0 || n <= 0) return 0;
  if (k <= 0 || !dst || !mat || !matsc || !src || !ssc) return set_error("gemm_int8: bad arguments");
  if (dstr == 0) dstr = n;
  if (mstr == 0) mstr = k;
  if (sstr == 0) sstr = k;
  ThreadCtx *c;
  if (ctx(&c)) return 1;
  const int k16 = (k + 15) / 16 * 16;  // device row stride of packed operands
  const int n4 = (n + 3) / 4 * 4;      // device row stride of the output
  // activations: pack to rows of k16 bytes (TMA wants 16-byte strides)
  void *dsrc, *dout, *dssc;
  if (c->in.get((size_t)m * k16, &dsrc) || c->out.get((size_t)m * n4 * 4, &dout)) return 1;
  // Activation scales: small outputs read them in place from mapped host
  // memory (no transfer); every N tile reads each row's scale, so large ones
  // (over ~16k PCIe reads) get them by a transfer like the activations.
  const bool scales_in_place = (size_t)m * n <= ((size_t)1 << 20);
  if (scales_in_place) {
    if (c->hs.get((size_t)m * 4)) return 1;
    memcpy(c->hs.h, ssc, (size_t)m * 4);
    dssc = c->hs.d;
  } else if (c->sc.get((size_t)m * 4, &dssc)) {
    return 1;
  }
  // row chunks of whole 128-row tiles when the output is large: chunk i's
  // output copy overlaps the GEMM and input copy of chunk i+1
  const int rows = m <= 8 ? m : chunk_rows(m, (size_t)n * 4, 128);
  const bool piped = rows < m;
  if (!piped) {
    GCU_CUDA(copy_rows(dsrc, k16, src, sstr, k, m, cudaMemcpyHostToDevice, c->stream));
    if (!scales_in_place)
      GCU_CUDA(cudaMemcpyAsync(dssc, ssc, (size_t)m * 4, cudaMemcpyHostToDevice, c->stream));
  }
  // weights: registered copy if the whole strided range is inside one
  const size_t wbytes = (size_t)(n - 1) * mstr + k;
  const void *dmat = lookup_q(mat, wbytes);
  const float *dms = nullptr;
  if (scales_dev(c, c->wstmp, matsc, (size_t)n, &dms)) return 1;
  long dmstr = mstr;
  // the GEMV kernel (m <= 8) reads dense rows; the tensor-core kernel any
  // 16-byte-aligned stride
  const bool dense_ok = dmat && (m <= 8 ? mstr == k
                                        : ((uintptr_t)dmat % 16 == 0) && (mstr % 16 == 0));
  if (!dense_ok) {
    // pack the weight rows into a dense, 16-byte-strided device buffer
    void *p;
    const int ws = (m <= 8) ? k : k16;
    if (c->wtmp.get((size_t)n * ws, &p)) return 1;
    if (dmat) {
      GCU_CUDA(copy_rows(p, ws, dmat, mstr, k, n, cudaMemcpyDeviceToDevice, c->stream));
    } else {
      GCU_CUDA(copy_rows(p, ws, mat, mstr, k, n, cudaMemcpyHostToDevice, c->stream));
    }
    dmat = p;
    dmstr = ws;
  }
  if (m <= 8) {
    // the GEMV kernel reads x rows at stride k16 and k-length weight rows
    if (dev_gemm((float *)dout, n4, (const int8_t *)dmat, dmstr, dms, (const int8_t *)dsrc, k16,
                 (const float *)dssc, m, n, k, c->stream))
      return 1;
    GCU_CUDA(copy_rows(dst, (size_t)dstr * 4, dout, (size_t)n4 * 4, (size_t)n * 4, m,
                               cudaMemcpyDeviceToHost, c->stream));
    return sync_and_check(c);
  }
  if (k16 != k && dmstr % 16 != 0) return set_error("gemm_int8: internal stride error");
  cudaStream_t s_out = piped ? c->s_out : c->stream;
  for (int r0 = 0, i = 0; r0 < m; r0 += rows, ++i) {
    const int mr = m - r0 < rows ? m - r0 : rows;
    if (piped) {
      // this chunk's activation rows, on the input stream
      GCU_CUDA(copy_rows((int8_t *)dsrc + (size_t)r0 * k16, k16, src + (size_t)r0 * sstr,
                                 sstr, k, mr, cudaMemcpyHostToDevice, c->s_in));
      if (!scales_in_place)
        GCU_CUDA(cudaMemcpyAsync((float *)dssc + r0, ssc + r0, (size_t)mr * 4,
                                 cudaMemcpyHostToDevice, c->s_in));
      GCU_CUDA(cudaEventRecord(c->ev_in[i], c->s_in));
      GCU_CUDA(cudaStreamWaitEvent(c->stream, c->ev_in[i], 0));
    }
    GemmArgs a{(float *)dout + (size_t)r0 * n4, n4, (const int8_t *)dmat, dmstr, dms,
               (const int8_t *)dsrc + (size_t)r0 * k16, k16, (const float *)dssc + r0, mr, n, k};
    if (launch_gemm_tc(a, c->stream, 0, 0)) return 1;
    if (piped) {
      GCU_CUDA(cudaEventRecord(c->ev_done[i], c->stream));
      GCU_CUDA(cudaStreamWaitEvent(s_out, c->ev_done[i], 0));
    }
    GCU_CUDA(copy_rows(dst + (size_t)r0 * dstr, (size_t)dstr * 4,
                               (float *)dout + (size_t)r0 * n4, (size_t)n4 * 4, (size_t)n * 4, mr,
                               cudaMemcpyDeviceToHost, s_out));
  }
  return sync_and_check(c, s_out);
}

// ---- device-pointer entry points ---------------------------------------------

GCU_EXPORT int gcu_dev_quantize_acts(int8_t *dst, float *dsc, const float *src, int sstr, int m,
                                     int n, void *stream) {
  if (sstr == 0) sstr = n;
  return launch_quantize_rows(dst, dsc, src, sstr, m, n, as_stream(stream));
}

GCU_EXPORT int gcu_dev_gemv_int8(float *dst, const int8_t *mat, const float *matsc,
                                 const int8_t *vec, const float *vsc, int m, int n, void *stream) {
  GemvJobs J{};
  J.w[0] = mat;
  J.ws[0] = matsc;
  J.y[0] = dst;
  J.row_end[0] = m;
  J.njobs = 1;
  return launch_gemv(J, vec, 0, vsc, 1, 0, n, as_stream(stream));
}

GCU_EXPORT int gcu_dev_gemv_int8_multi(const gcu_gemv_job *jobs, int njobs, const int8_t *vec,
                                       const float *vsc, int n, void *stream) {
  if (njobs > GCU_MAX_JOBS) return set_error("gemv_int8_multi: at most %d jobs", GCU_MAX_JOBS);
  GemvJobs J{};
  int rows = 0;
  for (int j = 0; j < njobs; ++j) {
    if (jobs[j].m <= 0) continue;
    J.w[J.njobs] = (const int8_t *)jobs[j].w;
    J.ws[J.njobs] = jobs[j].sc;
    J.y[J.njobs] = jobs[j].dst;
    rows += jobs[j].m;
    J.row_end[J.njobs] = rows;
    J.njobs++;
  }
  return launch_gemv(J, vec, 0, vsc, 1, 0, n, as_stream(stream));
}

GCU_EXPORT int gcu_dev_gemm_int8(float *dst, int dstr, const int8_t *mat, int mstr,
                                 const float *matsc, const int8_t *src, int sstr,
                                 const float *ssc, int m, int n, int k, void *stream) {
  if (m <= 0 || n <= 0) return 0;
  if (dstr == 0) dstr = n;
  if (mstr == 0) mstr = k;
  if (sstr == 0) sstr = k;
  return dev_gemm(dst, dstr, mat, mstr, matsc, src, sstr, ssc, m, n, k, as_stream(stream));
}

GCU_EXPORT int gcu_dev_gemm_int8_multi(const gcu_gemv_job *jobs, int njobs, const int8_t *src,
                                       int sstr, const float *ssc, int m, int k, void *stream) {
  if (m <= 0) return 0;
  if (sstr == 0) sstr = k;
  if (njobs <= 0) return 0;
  if (m <= 8) {
    if (njobs > GCU_MAX_JOBS) return set_error("gemm_int8_multi: at most %d jobs", GCU_MAX_JOBS);
    GemvJobs J{};
    int rows = 0;
    for (int j = 0; j < njobs; ++j) {
      J.w[j] = (const int8_t *)jobs[j].w;
      J.ws[j] = jobs[j].sc;
      J.y[j] = jobs[j].dst;
      rows += jobs[j].m;
      J.row_end[j] = rows;
    }
    J.njobs = njobs;
    if (njobs > 1) {
      // each job's output is (m, rows_j): one launch per job keeps the
      // per-job row stride
      for (int j = 0; j < njobs; ++j) {
        GemvJobs one{};
        one.w[0] = J.w[j];
        one.ws[0] = J.ws[j];
        one.y[0] = J.y[j];
        one.row_end[0] = jobs[j].m;
        one.njobs = 1;
        if (launch_gemv(one, src, sstr, ssc, m, jobs[j].m, k, as_stream(stream))) return 1;
      }
      return 0;
    }
    return launch_gemv(J, src, sstr, ssc, m, jobs[0].m, k, as_stream(stream));
  }
  if (njobs > 4) return set_error("gemm_int8_multi: at most 4 jobs on the tensor-core path");
  GemmArgs a[4];
  for (int j = 0; j < njobs; ++j)
    a[j] = GemmArgs{jobs[j].dst, jobs[j].m, (const int8_t *)jobs[j].w, k, jobs[j].sc,
                    src, sstr, ssc, m, jobs[j].m, k};
  return launch_gemm_tc_jobs(src, sstr, ssc, m, k, a, njobs, as_stream(stream), 0, 0);
}

GCU_EXPORT int gcu_dev_quantize_gemm_int8_multi(const gcu_gemv_job *jobs, int njobs, int8_t *q,
                                                float *s, const float *x, int xstr, int m, int k,
                                                void *stream) {
  if (m <= 0) return 0;
  if (k <= 0 || !q || !s || !x) return set_error("quantize_gemm_int8: bad arguments");
  if (xstr == 0) xstr = k;
  if (njobs <= 0) return launch_quantize_rows(q, s, x, xstr, m, k, as_stream(stream));
  cudaStream_t st = as_stream(stream);
  if (m <= 8) {
    if (njobs > GCU_MAX_JOBS) return set_error("quantize_gemm_int8: at most %d jobs", GCU_MAX_JOBS);
    GemvJobs J{};
    int rows = 0;
    for (int j = 0; j < njobs; ++j) {
      J.w[j] = (const int8_t *)jobs[j].w;
      J.ws[j] = jobs[j].sc;
      J.y[j] = jobs[j].dst;
      rows += jobs[j].m;
      J.row_end[j] = rows;
    }
    J.njobs = njobs;
    if (m == 1 || njobs == 1)
      return launch_quantize_gemv(J, x, xstr, q, s, m, njobs == 1 ? jobs[0].m : 0, k, st);
    // several rows and several jobs: each job's output has its own row stride
    if (launch_quantize_rows(q, s, x, xstr, m, k, st)) return 1;
    for (int j = 0; j < njobs; ++j) {
      GemvJobs one{};
      one.w[0] = J.w[j];
      one.ws[0] = J.ws[j];
      one.y[0] = J.y[j];
      one.row_end[0] = jobs[j].m;
      one.njobs = 1;
      if (launch_gemv(one, q, k, s, m, jobs[j].m, k, st)) return 1;
    }
    return 0;
  }
  if (njobs > 4) return set_error("quantize_gemm_int8: at most 4 jobs on the tensor-core path");
  GemmArgs a[4];
  for (int j = 0; j < njobs; ++j)
    a[j] = GemmArgs{jobs[j].dst, jobs[j].m, (const int8_t *)jobs[j].w, k, jobs[j].sc,
                    q, k, s, m, jobs[j].m, k};
  if (k % 16 || (uintptr_t)q % 16)
    return set_error("quantize_gemm_int8: m > 8 needs k %% 16 == 0 and a 16-byte aligned q "
                     "(the tensor-core kernel reads q with TMA); got k = %d", k);
  // Quantize kernel then tensor-core GEMM: the GEMM's prologue overlaps the
  // quantize kernel through programmatic dependent launch.  (Quantizing
  // inside the GEMM, one warp per row behind a grid barrier, measured slower
  // on B200 for the prefill shapes: a 148-CTA grid cannot keep enough loads
  // in flight for 512 rows.)
  if (launch_quantize_rows(q, s, x, xstr, m, k, st)) return 1;
  return launch_gemm_tc_jobs(q, k, s, m, k, a, njobs, st, 0, 0);
}

static int gemv_jobs_of(const gcu_gemv_job *jobs, int njobs, GemvJobs &J, const char *what) {
  if (!jobs || njobs <= 0 || njobs > GCU_MAX_JOBS) return set_error("%s: 1..%d jobs", what, GCU_MAX_JOBS);
  J = GemvJobs{};
  int rows = 0;
  for (int j = 0; j < njobs; ++j) {
    if (!jobs[j].w || !jobs[j].sc || !jobs[j].dst || jobs[j].m <= 0)
      return set_error("%s: job %d has a null pointer or no rows", what, j);
    J.w[j] = (const int8_t *)jobs[j].w;
    J.ws[j] = jobs[j].sc;
    J.y[j] = jobs[j].dst;
    rows += jobs[j].m;
    J.row_end[j] = rows;
  }
  J.njobs = njobs;
  return 0;
}

GCU_EXPORT int gcu_dev_geglu_quantize_gemv_multi(const gcu_gemv_job *jobs, int njobs, int8_t *q, float *s,
                                                 const float *gate, const float *up, int k, void *stream) {
  GemvJobs J;
  if (gemv_jobs_of(jobs, njobs, J, "geglu_quantize_gemv")) return 1;
  return launch_geglu_gemv(J, gate, up, q, s, k, as_stream(stream));
}

GCU_EXPORT int gcu_dev_residual_norm_quantize_gemv_multi(const gcu_gemv_job *jobs, int njobs, float *x, int8_t *q,
                                                         float *s, const float *y, const float *resid,
                                                         const float *w_post, const float *w_next, float eps,
                                                         int dim, void *stream) {
  GemvJobs J;
  if (gemv_jobs_of(jobs, njobs, J, "residual_norm_quantize_gemv")) return 1;
  return launch_resnorm_gemv(J, y, resid, w_post, w_next, eps, x, q, s, dim, as_stream(stream));
}

// Tuning hook (not in gcu.h): the multi-job GEMM with a forced tile shape
// ((128*mb) x bn) and K split.  Used by the benchmark's sweeps.
GCU_EXPORT int gcu_dev_gemm_int8_multi_tuned(const gcu_gemv_job *jobs, int njobs, const int8_t *src,
                                             int sstr, const float *ssc, int m, int k, int bn,
                                             int split, int mb, void *stream) {
  if (m <= 0 || njobs <= 0) return 0;
  if (sstr == 0) sstr = k;
  if (njobs > 4) return set_error("gemm_int8_multi: at most 4 jobs on the tensor-core path");
  GemmArgs a[4];
  for (int j = 0; j < njobs; ++j)
    a[j] = GemmArgs{jobs[j].dst, jobs[j].m, (const int8_t *)jobs[j].w, k, jobs[j].sc,
                    src, sstr, ssc, m, jobs[j].m, k};
  return launch_gemm_tc_jobs(src, sstr, ssc, m, k, a, njobs, as_stream(stream), bn, split, nullptr,
                             mb);
}

// Tuning hook (not in gcu.h): force the tensor-core kernel's tile shape
// ((128*mb) x bn) and K split for one call.  Used by the benchmark's sweeps.
GCU_EXPORT int gcu_dev_gemm_int8_tuned(float *dst, int dstr, const int8_t *mat, int mstr,
                                       const float *matsc, const int8_t *src, int sstr,
                                       const float *ssc, int m, int n, int k, int bn, int split,
                                       int mb, void *stream) {
  if (dstr == 0) dstr = n;
  if (mstr == 0) mstr = k;
  if (sstr == 0) sstr = k;
  GemmArgs a{dst, dstr, mat, mstr, matsc, src, sstr, ssc, m, n, k};
  return launch_gemm_tc(a, as_stream(stream), bn, split, mb);
}
