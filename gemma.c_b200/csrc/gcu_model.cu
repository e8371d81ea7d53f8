// gcu_model.cu -- gemma.c's `-q` model image -> one device allocation.
//
// gemma.c either reads every tensor into its own malloc'd buffer
// (read_gemma_model, gemma.c:2045-2110) or maps the whole file
// (mmap_gemma_model, gemma.c:1946-2043; tensors are then pointers into the
// mapping, mmap_qtensor gemma.c:1156-1171).  Registering its matmul weights
// one by one costs a cudaMalloc and two pageable copies per QTensor (337 of
// them for the 12B text decoder).  Here they are found in the image by the
// file's own layout and uploaded as ONE arena:
//
//   - the parser follows check_head (gemma.c:1915-1940), read_text_config
//     (770-865: big-endian fields, the sliding-window bit field, the flag
//     byte), read_vision_config (723-738), read_tokenizer (905-990: pascal
//     strings, skipped), then the tensor order of mmap_text_decoder
//     (1470-1560) and mmap_vision_encoder (1765-1875);
//   - the arena holds each QTensor's int8 rows and its scales at 256-byte
//     aligned offsets (TMA wants 16-byte aligned bases; the file packs them
//     back to back after variable-length strings);
//   - T host threads each own two pinned 8 MB slots: a thread packs the next
//     arena window of its own into a free slot (memcpy from the image, which
//     also pages a mapped file in) and queues the window's host->device copy
//     on its stream, so packing and the copy engine overlap.
#include "gcu_internal.cuh"

#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#define GCU_EXPORT extern "C" __attribute__((visibility("default")))

namespace gcu {
namespace {

// ---------------------------------------------------------------------------
// parser
// ---------------------------------------------------------------------------
struct Cursor {
  const uint8_t *p;
  size_t size, off = 0;
  bool ok = true;
  bool need(size_t n) {
    if (!ok || n > size - off) ok = false;
    return ok;
  }
  uint32_t u8() { return need(1) ? p[off++] : 0; }
  uint32_t u16() {  // gemma.c:634-640: big-endian
    if (!need(2)) return 0;
    const uint32_t v = ((uint32_t)p[off] << 8) | p[off + 1];
    off += 2;
    return v;
  }
  uint32_t u32() {  // gemma.c:642-649
    if (!need(4)) return 0;
    const uint32_t v = ((uint32_t)p[off] << 24) | ((uint32_t)p[off + 1] << 16) |
                       ((uint32_t)p[off + 2] << 8) | p[off + 3];
    off += 4;
    return v;
  }
  void skip(size_t n) {
    if (need(n)) off += n;
  }
  void strings(uint64_t count) {  // pascal strings, gemma.c:672-684
    for (uint64_t i = 0; i < count && ok; ++i) skip(u8());
  }
};

struct TextCfg {
  uint32_t nl, n_heads, nkv, hdim, dim, mlp_dim, nvocab;
  bool has_mm, qk_norm, mlp_pre, mlp_pst;
};
struct VisionCfg {
  uint32_t nl, mlp_dim, dim, img_px, psize;
};

struct Walk {
  const uint8_t *base;
  size_t off;
  std::vector<gcu_qtensor> out;
  void floats(size_t n) { off += n * sizeof(float); }
  // mmap_qtensor (gemma.c:1156-1171): int8 [rows][k], then fp32 [rows]
  void qtensor(uint64_t rows, uint64_t k, int kind, int layer, bool keep) {
    if (keep) {
      gcu_qtensor t;
      t.q = reinterpret_cast<const int8_t *>(base + off);
      t.scales = reinterpret_cast<const float *>(base + off + rows * k);
      t.rows = (int)rows;
      t.k = (int)k;
      t.kind = kind;
      t.layer = layer;
      out.push_back(t);
    }
    off += rows * k + rows * sizeof(float);
  }
};

int parse(const void *image, size_t size, int allow_mm, std::vector<gcu_qtensor> &out) {
  if (!image) return set_error("bin_qtensors: null image");
  Cursor c{static_cast<const uint8_t *>(image), size};
  if (!c.need(8)) return set_error("bin_qtensors: image of %zu bytes has no header", size);
  const uint8_t *h = c.p;
  if (memcmp(h, "GEMA", 4) != 0) return set_error("bin_qtensors: not a gemma model file (magic)");
  if (memcmp(h + 4, "f32", 3) != 0)
    return set_error("bin_qtensors: dtype '%c%c%c' (only f32 builds use this library)", h[4], h[5], h[6]);
  if (h[7] == 'U') return set_error("bin_qtensors: not a W8A8 (-q) model file");
  if (h[7] != 'Q') return set_error("bin_qtensors: not a gemma model file (flag)");
  c.off = 8;

  TextCfg tc{};
  tc.nl = c.u8();
  tc.n_heads = c.u8();
  tc.nkv = c.u8();
  tc.hdim = c.u16();
  tc.dim = c.u16();
  tc.mlp_dim = c.u16();
  c.u16();  // q_scale
  c.u16();  // slide
  c.u16();  // img_tok
  c.u32();  // max_seq
  tc.nvocab = c.u32();
  c.skip(5 * 4);  // theta_l, theta_g, eps, sc_att, sc_log
  const uint32_t swa_bytes = c.u8();
  if (c.ok && swa_bytes * 8 < tc.nl) return set_error("bin_qtensors: insufficient att_layers bytes");
  c.skip(swa_bytes);
  const uint32_t flags = c.u8();
  tc.has_mm = flags & 8;
  tc.qk_norm = flags & 4;
  tc.mlp_pre = flags & 2;
  tc.mlp_pst = flags & 1;

  VisionCfg vc{};
  if (tc.has_mm) {  // read even when it is not used, like gemma.c:1977-1983
    vc.nl = c.u8();
    c.u8();  // n_heads
    vc.mlp_dim = c.u16();
    vc.dim = c.u16();
    vc.img_px = c.u16();
    vc.psize = c.u16();
    c.skip(4);  // eps
  }
  c.strings((uint64_t)tc.nvocab + (tc.has_mm ? 1 : 0));  // vocab (+ <image_soft_token>)
  const uint32_t nmerge = c.u32();
  c.strings(2ull * nmerge);
  if (!c.ok) return set_error("bin_qtensors: image truncated inside the configs or tokenizer");
  if (tc.nvocab > 0x7fffffffu) return set_error("bin_qtensors: vocabulary of %u rows", tc.nvocab);
  const bool use_mm = tc.has_mm && allow_mm;
  if (use_mm && (vc.psize == 0 || vc.img_px < vc.psize))
    return set_error("bin_qtensors: vision patch size %u for %u px", vc.psize, vc.img_px);

  Walk w{c.p, c.off, {}};
  const uint64_t dim = tc.dim, mlp = tc.mlp_dim, q_sz = (uint64_t)tc.n_heads * tc.hdim,
                 kv_sz = (uint64_t)tc.nkv * tc.hdim;
  // mmap_text_decoder, gemma.c:1470-1560
  w.qtensor(tc.nvocab, dim, GCU_QT_LM_HEAD, -1, true);
  for (int l = 0; l < (int)tc.nl; ++l) {
    w.qtensor(q_sz, dim, GCU_QT_WQ, l, true);
    w.qtensor(kv_sz, dim, GCU_QT_WK, l, true);
    w.qtensor(kv_sz, dim, GCU_QT_WV, l, true);
    w.qtensor(dim, q_sz, GCU_QT_WO, l, true);
    if (tc.qk_norm) w.floats(2 * (uint64_t)tc.hdim);  // nq, nk
    w.qtensor(mlp, dim, GCU_QT_W1, l, true);
    w.qtensor(mlp, dim, GCU_QT_W2, l, true);
    w.qtensor(dim, mlp, GCU_QT_W3, l, true);
    w.floats(2 * dim);  // n1, n2
    if (tc.mlp_pre) w.floats(dim);
    if (tc.mlp_pst) w.floats(dim);
  }
  w.floats(dim);  // fnorm
  if (use_mm) {
    // mmap_vision_encoder, gemma.c:1765-1875
    const uint64_t vd = vc.dim, vm = vc.mlp_dim, P = vc.psize, side = vc.img_px / vc.psize;
    w.floats(vd * 3 * P * P + vd);                  // pe, pe_b
    w.qtensor(side * side, vd, -1, -1, false);      // pos_emb: a lookup table, not a matmul
    for (int l = 0; l < (int)vc.nl; ++l) {
      w.floats(2 * vd);  // n1, n1_b
      w.qtensor(vd, vd, GCU_QT_VWQ, l, true);
      w.qtensor(vd, vd, GCU_QT_VWK, l, true);
      w.qtensor(vd, vd, GCU_QT_VWV, l, true);
      w.qtensor(vd, vd, GCU_QT_VWO, l, true);
      w.floats(4 * vd + 2 * vd);  // bq, bk, bv, bo, n2, n2_b
      w.qtensor(vm, vd, GCU_QT_VW1, l, true);
      w.qtensor(vd, vm, GCU_QT_VW2, l, true);
      w.floats(vm + vd);  // b1, b2
    }
    w.floats(3 * vd);  // post_n, post_nb, norm
    w.qtensor(dim, vd, GCU_QT_VPROJ, -1, true);
  }
  if (w.off > size)
    return set_error("bin_qtensors: image of %zu bytes ends before its tensors (%zu)", size, w.off);
  for (const gcu_qtensor &t : w.out)
    if (t.rows <= 0 || t.k <= 0) return set_error("bin_qtensors: empty weight (kind %d)", t.kind);
  out.swap(w.out);
  return 0;
}

// ---------------------------------------------------------------------------
// bulk upload
// ---------------------------------------------------------------------------
constexpr size_t kAlign = 256;
constexpr size_t kSlotBytes = 8u << 20;
constexpr int kMaxThreads = 16;

// packing threads: three quarters of the host's hardware threads, at most
// kMaxThreads (packing is bound by host DRAM bandwidth well before that);
// GCU_UPLOAD_THREADS overrides (1..kMaxThreads)
int upload_threads() {
  if (const char *e = getenv("GCU_UPLOAD_THREADS")) {
    const int v = atoi(e);
    if (v >= 1) return std::min(v, kMaxThreads);
  }
  const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
  return (int)std::min<unsigned>(kMaxThreads, std::max(1u, hw * 3 / 4));
}

// Copy into a pinned slot with non-temporal 32-byte stores: the slot is only
// read again by the copy engine, so its lines need not be fetched into the
// cache first (a plain copy reads every destination line before writing
// it).  dst must be 32-byte aligned; the caller fences before the DMA.
__attribute__((target("avx2"))) void stream_copy_avx2(uint8_t *dst, const uint8_t *src, size_t n) {
  size_t i = 0;
  for (; i + 128 <= n; i += 128) {
    const __m256i a = _mm256_loadu_si256(reinterpret_cast<const __m256i *>(src + i));
    const __m256i b = _mm256_loadu_si256(reinterpret_cast<const __m256i *>(src + i + 32));
    const __m256i c = _mm256_loadu_si256(reinterpret_cast<const __m256i *>(src + i + 64));
    const __m256i d = _mm256_loadu_si256(reinterpret_cast<const __m256i *>(src + i + 96));
    _mm256_stream_si256(reinterpret_cast<__m256i *>(dst + i), a);
    _mm256_stream_si256(reinterpret_cast<__m256i *>(dst + i + 32), b);
    _mm256_stream_si256(reinterpret_cast<__m256i *>(dst + i + 64), c);
    _mm256_stream_si256(reinterpret_cast<__m256i *>(dst + i + 96), d);
  }
  if (i < n) memcpy(dst + i, src + i, n - i);
}

bool use_stream_copy() {
  static const bool ok = [] {
    if (const char *e = getenv("GCU_UPLOAD_NT")) return atoi(e) != 0;
    return (bool)__builtin_cpu_supports("avx2");
  }();
  return ok;
}

void pack_copy(uint8_t *dst, const uint8_t *src, size_t n) {
  if (n >= 4096 && ((uintptr_t)dst & 31) == 0 && use_stream_copy())
    stream_copy_avx2(dst, src, n);
  else
    memcpy(dst, src, n);
}

struct Piece {
  const uint8_t *src;
  size_t off, len;
};

// pinned slots, two per packing thread, kept for later uploads
std::mutex g_stage_mu;
std::vector<void *> g_slots;

int staging(int nslots) {
  while ((int)g_slots.size() < nslots) {
    void *p = nullptr;
    GCU_CUDA(cudaHostAlloc(&p, kSlotBytes, cudaHostAllocDefault));
    g_slots.push_back(p);
  }
  return 0;
}

void pack_windows(int t, int nthreads, int device, uint8_t *dbase, size_t total,
                  const std::vector<Piece> &pieces, std::atomic<int> &failed, std::string &msg,
                  std::mutex &msg_mu) {
  auto fail = [&](cudaError_t e, const char *what) {
    std::lock_guard<std::mutex> lk(msg_mu);
    if (!failed.exchange(1)) msg = std::string(what) + ": " + cudaGetErrorString(e);
  };
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return fail(e, "cudaSetDevice");
  cudaStream_t st;
  if ((e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking)) != cudaSuccess)
    return fail(e, "cudaStreamCreate");
  cudaEvent_t ev[2] = {nullptr, nullptr};
  bool used[2] = {false, false};
  for (int i = 0; i < 2 && e == cudaSuccess; ++i) e = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming);
  const size_t nwin = (total + kSlotBytes - 1) / kSlotBytes;
  size_t first = 0;  // first piece that may meet the current window
  for (size_t win = t, i = 0; e == cudaSuccess && win < nwin && !failed.load(); win += nthreads, ++i) {
    const int slot = (int)(i & 1);
    if (used[slot] && (e = cudaEventSynchronize(ev[slot])) != cudaSuccess) break;
    uint8_t *buf = static_cast<uint8_t *>(g_slots[2 * t + slot]);
    const size_t w0 = win * kSlotBytes, w1 = std::min(total, w0 + kSlotBytes);
    while (first < pieces.size() && pieces[first].off + pieces[first].len <= w0) ++first;
    for (size_t p = first; p < pieces.size() && pieces[p].off < w1; ++p) {
      const size_t a = std::max(w0, pieces[p].off), b = std::min(w1, pieces[p].off + pieces[p].len);
      if (a < b) pack_copy(buf + (a - w0), pieces[p].src + (a - pieces[p].off), b - a);
    }
    _mm_sfence();  // the streaming stores are globally visible before the copy reads the slot
    if ((e = cudaMemcpyAsync(dbase + w0, buf, w1 - w0, cudaMemcpyHostToDevice, st)) != cudaSuccess) break;
    if ((e = cudaEventRecord(ev[slot], st)) != cudaSuccess) break;
    used[slot] = true;
  }
  const cudaError_t drained = cudaStreamSynchronize(st);  // no copy may outlive its slot
  if (e == cudaSuccess) e = drained;
  if (e != cudaSuccess) fail(e, "model upload");
  for (int i = 0; i < 2; ++i)
    if (ev[i]) cudaEventDestroy(ev[i]);
  cudaStreamDestroy(st);
}

int upload(const gcu_qtensor *list, int n, int *arena) {
  if (n <= 0 || !list) return set_error("register_qtensors: no tensors");
  std::vector<RegRec> recs((size_t)n);
  std::vector<Piece> pieces;
  pieces.reserve(2 * (size_t)n);
  size_t total = 0;
  for (int i = 0; i < n; ++i) {
    const gcu_qtensor &t = list[i];
    if (!t.q || !t.scales || t.rows <= 0 || t.k <= 0)
      return set_error("register_qtensors: tensor %d: bad arguments", i);
    const size_t qb = (size_t)t.rows * t.k, sb = (size_t)t.rows * sizeof(float);
    RegRec &r = recs[i];
    r.q = (uintptr_t)t.q;
    r.s = (uintptr_t)t.scales;
    r.rows = t.rows;
    r.k = t.k;
    r.dq_off = total;
    pieces.push_back({reinterpret_cast<const uint8_t *>(t.q), total, qb});
    total = (total + qb + kAlign - 1) / kAlign * kAlign;
    r.ds_off = total;
    pieces.push_back({reinterpret_cast<const uint8_t *>(t.scales), total, sb});
    total = (total + sb + kAlign - 1) / kAlign * kAlign;
  }
  const int d = calling_device();
  GCU_CUDA(cudaSetDevice(d));
  void *base = nullptr;
  GCU_CUDA(cudaMalloc(&base, total));
  const size_t nwin = (total + kSlotBytes - 1) / kSlotBytes;
  const int nthreads = (int)std::min<size_t>(nwin, (size_t)upload_threads());
  std::atomic<int> failed{0};
  std::string msg;
  {
    std::lock_guard<std::mutex> lk(g_stage_mu);  // the slots serve one upload at a time
    if (staging(2 * nthreads)) {
      cudaFree(base);
      return 1;
    }
    std::mutex msg_mu;
    std::vector<std::thread> th;
    for (int t = 1; t < nthreads; ++t)
      th.emplace_back(pack_windows, t, nthreads, d, static_cast<uint8_t *>(base), total, std::cref(pieces),
                      std::ref(failed), std::ref(msg), std::ref(msg_mu));
    pack_windows(0, nthreads, d, static_cast<uint8_t *>(base), total, pieces, failed, msg, msg_mu);
    for (auto &x : th) x.join();
  }
  if (failed.load()) {
    cudaFree(base);
    return set_error("register_qtensors: %s", msg.c_str());
  }
  if (registry_add_arena(recs.data(), n, base, total, arena)) {
    cudaFree(base);
    return 1;
  }
  return 0;
}

}  // namespace

void release_staging() {
  std::lock_guard<std::mutex> lk(g_stage_mu);
  for (void *p : g_slots) cudaFreeHost(p);
  g_slots.clear();
}

}  // namespace gcu

using namespace gcu;

GCU_EXPORT int gcu_bin_qtensors(const void *image, size_t size, int allow_mm, gcu_qtensor *out, int cap) {
  std::vector<gcu_qtensor> v;
  if (parse(image, size, allow_mm, v)) return -1;
  if (out)
    for (int i = 0; i < cap && i < (int)v.size(); ++i) out[i] = v[i];
  return (int)v.size();
}

GCU_EXPORT int gcu_register_qtensors(const gcu_qtensor *list, int n, int *arena) {
  return upload(list, n, arena);
}

GCU_EXPORT int gcu_register_model(const void *image, size_t size, int allow_mm, int *arena) {
  std::vector<gcu_qtensor> v;
  if (parse(image, size, allow_mm, v)) return 1;
  return upload(v.data(), (int)v.size(), arena);
}
