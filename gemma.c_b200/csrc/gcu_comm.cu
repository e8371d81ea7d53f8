// gcu_comm.cu -- row-sharded W8A8 matmul across the GPUs of one node.
//
// The reference is single-process (README.md:614); this is the one place the
// library adds communication.  Every output row of gemm_int8 / gemv_int8 is
// independent, so rank r computes rows [r*n/world, (r+1)*n/world) of the
// output from its slice of the weight and an NCCL all-gather over NVLink
// assembles the full output on every rank.  NCCL is opened with dlopen on
// first use so the single-GPU entry points never depend on it.
#include "gcu_internal.cuh"

#include <dlfcn.h>
#include <nccl.h>

#include <mutex>

#define GCU_EXPORT extern "C" __attribute__((visibility("default")))

namespace gcu {
namespace {

struct Nccl {
  void *lib = nullptr;
  ncclResult_t (*getUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*commInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*allGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
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
    g_nccl.commDestroy = (decltype(g_nccl.commDestroy))dlsym(g_nccl.lib, "ncclCommDestroy");
    g_nccl.getErrorString = (decltype(g_nccl.getErrorString))dlsym(g_nccl.lib, "ncclGetErrorString");
  });
  if (!g_nccl.lib || !g_nccl.getUniqueId || !g_nccl.commInitRank || !g_nccl.allGather ||
      !g_nccl.commDestroy)
    return set_error("NCCL (libnccl.so.2) could not be loaded");
  return 0;
}

int nccl_err(ncclResult_t r, const char *what) {
  return set_error("%s: %s", what, g_nccl.getErrorString ? g_nccl.getErrorString(r) : "nccl error");
}

struct Comm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
};
Comm g_comm;
std::mutex g_comm_mu;

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
  return 0;
}

GCU_EXPORT int gcu_comm_destroy(void) {
  std::lock_guard<std::mutex> lk(g_comm_mu);
  if (!g_comm.comm) return 0;
  ncclResult_t r = g_nccl.commDestroy(g_comm.comm);
  g_comm.comm = nullptr;
  if (r != ncclSuccess) return nccl_err(r, "ncclCommDestroy");
  return 0;
}

GCU_EXPORT int gcu_dev_gemm_int8_rowshard(float *dst, float *work, const int8_t *mat_local,
                                          const float *matsc_local, const int8_t *src,
                                          const float *ssc, int m, int n, int k, void *stream) {
  if (!g_comm.comm) return set_error("gcu_dev_gemm_int8_rowshard: gcu_comm_init first");
  const int world = g_comm.world, rank = g_comm.rank;
  if (n % world) return set_error("rowshard: n %d not divisible by world %d", n, world);
  if (m <= 0) return 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nl = n / world;
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
