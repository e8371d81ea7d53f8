// gcu_noalloc.cu -- gemm_int8 on device data without any device allocation.
//
// gcu_dev_gemm_int8 splits K across CTAs when a GEMM has few output tiles
// and a long reduction (the prefill down projection, for instance), and the
// int32 partial sums of the splits need scratch memory.  Normally the
// library cudaMalloc's that scratch on first use and grows it as shapes
// grow.  Some callers cannot let a library allocate device memory at call
// time: a serving process that sizes every device buffer once at start-up
// and treats any later allocation as a failure, a caller whose stream must
// never be implicitly synchronised (cudaMalloc / cudaFree can synchronise
// the device), or a host program linked against a custom allocator that
// owns all device memory.  gcu_dev_gemm_int8_noalloc serves them: the
// split-K scratch lives in a fixed array in the library's device image, so
// a call allocates nothing.
//
// The array is a file-scope __device__ variable, so every GPU that loads
// libgcu.so holds it (kMaxScratchBytes plus kMaxCounters ints) until the
// process exits.  Host code must not use the array's name as a pointer: it
// names a host-side stand-in.  Its device address is looked up once per
// device with cudaGetSymbolAddress, the first time this entry point runs on
// that device (so make that first call before any stream capture).  All
// calls share the array: calls that overlap on the GPU (two streams, or two
// threads on different streams) race on it and must be serialised by the
// caller.  Each call zeroes the arrival counters it uses before its launch;
// the partial sums need no clearing because every split writes its own
// slot before it is read.
#include "gcu_internal.cuh"

#include <mutex>

#define GCU_EXPORT extern "C" __attribute__((visibility("default")))

namespace gcu {
namespace {

// 8 MiB of int32 partial sums: enough for, e.g., M=256 x N=1152 x K=6912
// split six ways (6.75 MiB); plans that need more are rejected.
constexpr size_t kMaxScratchBytes = (size_t)8 << 20;
constexpr int kMaxCounters = 4096;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kMaxScratchBytes +
                                                                 kMaxCounters * sizeof(int)];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_addr[kMaxDevices] = {};  // device address of the array, per device

// The array's address on the device this thread launches on: the same device
// (calling_device(), fixed by gcu_init or the first call) whose error word,
// SM count and tensor-map encoder the launch uses.  cudaGetSymbolAddress
// answers for the CUDA runtime's current device, so the two must agree.
int scratch_address(void **out) {
  const int dev = calling_device();
  int cur = 0;
  GCU_CUDA(cudaGetDevice(&cur));
  if (cur != dev)
    return set_error("noalloc: the current CUDA device (%d) is not this thread's device (%d); "
                     "call gcu_init(%d) after switching devices", cur, dev, cur);
  if (dev < 0 || dev >= kMaxDevices) return set_error("noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return check_cuda(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return 0;
}

}  // namespace
}  // namespace gcu

using namespace gcu;

namespace {

int noalloc_gemm(float *dst, int dstr, const int8_t *mat, int mstr, const float *matsc,
                 const int8_t *src, int sstr, const float *ssc, int m, int n, int k, void *stream,
                 int force_bn, int force_split, int force_mb) {
  if (m <= 0 || n <= 0) return 0;
  if (k <= 0) return set_error("gemm_int8_noalloc: k must be positive (got %d)", k);
  if (dstr == 0) dstr = n;
  if (mstr == 0) mstr = k;
  if (sstr == 0) sstr = k;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (m <= 8) {
    // the streaming GEMV kernel needs no scratch
    if (mstr != k)
      return set_error("gemm_int8_noalloc: m <= 8 needs dense weight rows (mstr %d, k %d)", mstr, k);
    GemvJobs J{};
    J.w[0] = mat;
    J.ws[0] = matsc;
    J.y[0] = dst;
    J.row_end[0] = n;
    J.njobs = 1;
    return launch_gemv(J, src, sstr, ssc, m, dstr, k, st);
  }
  void *base = nullptr;
  if (scratch_address(&base)) return 1;
  ExtWorkspace ext{base, kMaxScratchBytes,
                   reinterpret_cast<int *>(static_cast<unsigned char *>(base) + kMaxScratchBytes),
                   kMaxCounters};
  GemmArgs a{dst, dstr, mat, mstr, matsc, src, sstr, ssc, m, n, k};
  return launch_gemm_tc_jobs(src, sstr, ssc, m, k, &a, 1, st, force_bn, force_split, &ext,
                             force_mb);
}

}  // namespace

GCU_EXPORT int gcu_dev_gemm_int8_noalloc(float *dst, int dstr, const int8_t *mat, int mstr,
                                         const float *matsc, const int8_t *src, int sstr,
                                         const float *ssc, int m, int n, int k, void *stream) {
  return noalloc_gemm(dst, dstr, mat, mstr, matsc, src, sstr, ssc, m, n, k, stream, 0, 0, 0);
}

// Same with a forced tile shape ((128*mb) x bn) and K split, for tests that
// need a given amount of scratch whatever the planner would pick (not part
// of the public header).
GCU_EXPORT int gcu_dev_gemm_int8_noalloc_tuned(float *dst, int dstr, const int8_t *mat, int mstr,
                                               const float *matsc, const int8_t *src, int sstr,
                                               const float *ssc, int m, int n, int k, int bn,
                                               int split, int mb, void *stream) {
  return noalloc_gemm(dst, dstr, mat, mstr, matsc, src, sstr, ssc, m, n, k, stream, bn, split, mb);
}
