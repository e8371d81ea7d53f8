/*
 * gcu.h -- C ABI of libgcu.so, the B200 (sm_100a) W8A8 matmul hot path of
 * Gemma.c.
 *
 * The reference keeps the path in five `static` functions of gemma.c; this
 * library exports one entry point per function with the same argument
 * meaning, plus device-pointer variants for callers whose activations already
 * live in GPU memory.  Everything is plain C: pointers, ints, floats.
 *
 * Conventions shared by every entry point:
 *   - return 0 on success and 1 on error (gemma.c's gemm_int8 convention,
 *     gemma.c:3977-3982); gcu_last_error() then holds a message.  The
 *     message is thread local, like gemma.c's g_err (gemma.c:577).
 *   - "host" entry points take HOST pointers exactly as gemma.c passes them
 *     and return when the result is in host memory.  Weights should be
 *     registered once (gcu_register_weight) so calls find their device copy;
 *     an unregistered weight is uploaded for that call only.
 *   - "dev" entry points take DEVICE pointers and a cudaStream_t (as void*,
 *     NULL = the legacy default stream) and only enqueue work.
 *   - every entry point may be called concurrently from several host threads
 *     (gemma.c calls gemm_int8 from inside OpenMP regions, gemma.c:5045-5091);
 *     each thread gets its own stream and staging buffers.
 *   - weight layout is gemma.c's QTensor (gemma.c:1102-1131): int8 values
 *     row-major [rows][k] followed by one fp32 scale per row.
 */
#ifndef GCU_H
#define GCU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GCU_MAX_JOBS 8

/* ---- lifecycle ---------------------------------------------------------- */

/* Select the CUDA device the calling thread uses (default 0). Idempotent. */
int gcu_init(int device);
/* Free every registered weight, stream and buffer of this process. */
int gcu_shutdown(void);
/* Thread-local message of the last failed call ("" if none). */
const char *gcu_last_error(void);
/* Wait for the device and return 1 if a kernel recorded a device-side error
 * (a bounded wait that gave up), clearing it; 0 otherwise. */
int gcu_check_device(void);
/* Library version string. */
const char *gcu_version(void);

/* ---- weight registry ------------------------------------------------------
 * Replaces nothing in gemma.c: it is the hook a maintainer adds after the
 * weights are read or mapped (read_qtensor / mmap_qtensor, gemma.c:1134-1171;
 * setup_gemma_model, gemma.c:6867).  q points at rows*k int8 values, scales
 * at rows floats.  Any pointer INSIDE a registered range (gemma.c passes
 * w->i8.q + hd*hdim*dim, gemma.c:5080-5086) resolves to the device copy. */
int gcu_register_weight(const int8_t *q, const float *scales, int rows, int k);
int gcu_unregister_weight(const int8_t *q);
/* Bytes of device memory held by registered weights. */
size_t gcu_registered_bytes(void);

/* ---- model images: every matmul weight of a `-q` .bin at once -------------
 * A W8A8 model file (export.py -q; header "GEMA" "f32" 'Q', gemma.c:1915-1940)
 * holds, after its configs (gemma.c:723-865) and tokenizer (gemma.c:905-990),
 * every QTensor back to back in mmap_text_decoder's / mmap_vision_encoder's
 * order (gemma.c:1470-1560, 1765-1875).  These entry points find the
 * QTensors the matmul path uses in such an image (the mmap gemma.c made,
 * GemmaModel.mm_data / mm_sz, gemma.c:2005-2018, or the file read into memory)
 * and upload them as ONE device allocation: host threads pack pinned staging
 * slots in the device layout while the copy engine drains earlier slots. */
typedef enum {
  GCU_QT_LM_HEAD = 0, /* text embedding, tied lm_head (gemma.c:1398-1406) */
  GCU_QT_WQ, GCU_QT_WK, GCU_QT_WV, GCU_QT_WO, /* text attention, per layer */
  GCU_QT_W1, GCU_QT_W2, GCU_QT_W3,            /* text FFN up, gate, down */
  GCU_QT_VWQ, GCU_QT_VWK, GCU_QT_VWV, GCU_QT_VWO, /* SigLIP attention */
  GCU_QT_VW1, GCU_QT_VW2,                         /* SigLIP fc1, fc2 */
  GCU_QT_VPROJ                                    /* multimodal projection */
} gcu_qt_kind;

typedef struct {
  const int8_t *q;      /* int8 [rows][k] */
  const float *scales;  /* fp32 [rows] */
  int rows, k;
  int kind;             /* gcu_qt_kind */
  int layer;            /* layer index, -1 for LM_HEAD and VPROJ */
} gcu_qtensor;

/* List the matmul QTensors of a model image of `size` bytes: the text
 * decoder's, plus the vision encoder's when the file is multimodal and
 * allow_mm is set (gemma.c's allow_mm, 1970-1983).  Fills up to cap records
 * (out may be NULL) and returns how many there are, or -1 with a message for
 * an image that is not a well-formed f32 W8A8 model or is truncated.  Host
 * only: needs no GPU. */
int gcu_bin_qtensors(const void *image, size_t size, int allow_mm, gcu_qtensor *out, int cap);
/* Register n QTensors (any host memory) as one device allocation; *arena
 * (may be NULL) receives its handle.  Each tensor then resolves like a
 * gcu_register_weight one.  Tensors already registered are an error. */
int gcu_register_qtensors(const gcu_qtensor *list, int n, int *arena);
/* gcu_bin_qtensors + gcu_register_qtensors on a model image. */
int gcu_register_model(const void *image, size_t size, int allow_mm, int *arena);
/* Drop an arena's tensors from the registry and free its device memory. */
int gcu_unregister_arena(int arena);

/* ---- host-pointer entry points (gemma.c signatures) ----------------------- */

/* gemma.c:2590 quantize_act: per-vector symmetric int8 of vec[0..dim);
 * returns the scale (the reference returns floatx).  On error returns NaN. */
float gcu_quantize_act(int8_t *dst, const float *vec, int dim);

/* gemma.c:2656 quantize_acts: m rows of src (row stride sstr floats, 0 = n)
 * to dense int8 dst (m, n) and scales dsc (m). */
int gcu_quantize_acts(int8_t *dst, float *dsc, const float *src, int sstr,
                      int m, int n);

/* gemma.c:2770 gemv_int8: dst[i] = dequant(dot(mat row i, vec)), i < m,
 * reduction length n (note: m = rows, n = k, as in the reference). */
int gcu_gemv_int8(float *dst, const int8_t *mat, const float *matsc,
                  const int8_t *vec, float vsc, int m, int n);

/* gemma.c:2795 GemvJob (floatx = float). */
typedef struct {
  const void *w;
  const float *sc;
  float *dst;
  int m;
} gcu_gemv_job;

/* gemma.c:2818 gemv_int8_multi: up to GCU_MAX_JOBS GEMVs sharing vec. */
int gcu_gemv_int8_multi(const gcu_gemv_job *jobs, int njobs, const int8_t *vec,
                        float vsc, int n);

/* gemma.c:3943 gemm_int8: NT GEMM
 *   dst[i*dstr + j] = (float)sum_l src[i*sstr+l]*mat[j*mstr+l] * (ssc[i]*matsc[j])
 * for i < m (tokens), j < n (weight rows), l < k; strides 0 = dense. */
int gcu_gemm_int8(float *dst, int dstr, const int8_t *mat, int mstr,
                  const float *matsc, const int8_t *src, int sstr,
                  const float *ssc, int m, int n, int k);

/* ---- device-pointer entry points ------------------------------------------
 * Same arithmetic as the host entry points; all pointers are device
 * pointers; work is enqueued on `stream` and not waited for. */

/* quantize_acts on device data. */
int gcu_dev_quantize_acts(int8_t *dst, float *dsc, const float *src, int sstr,
                          int m, int n, void *stream);

/* gemv_int8 on device data; vsc points at the one device-resident scale
 * written by gcu_dev_quantize_acts. */
int gcu_dev_gemv_int8(float *dst, const int8_t *mat, const float *matsc,
                      const int8_t *vec, const float *vsc, int m, int n,
                      void *stream);

/* gemv_int8_multi on device data (jobs hold device pointers; the job array
 * itself is host memory). */
int gcu_dev_gemv_int8_multi(const gcu_gemv_job *jobs, int njobs,
                            const int8_t *vec, const float *vsc, int n,
                            void *stream);

/* gemm_int8 on device data. m <= 8 runs the streaming GEMV kernel, larger m
 * the tcgen05 tensor-core kernel; both give the same bits. */
int gcu_dev_gemm_int8(float *dst, int dstr, const int8_t *mat, int mstr,
                      const float *matsc, const int8_t *src, int sstr,
                      const float *ssc, int m, int n, int k, void *stream);

/* gemm_int8 on device data that allocates no device memory.  This entry
 * point has no counterpart in the reference.  For callers that may not allocate once they are
 * running -- processes that size all GPU memory at start-up, or that cannot
 * afford the device synchronisation cudaMalloc/cudaFree may cause -- the
 * split-K scratch comes from a fixed 8 MiB array inside libgcu.so (held on
 * every GPU that loads the library).  Same arguments and bits as
 * gcu_dev_gemm_int8; returns 1 with a message when the split-K plan needs
 * more than that array.  The first call on a device looks the array's
 * address up (make it before any stream capture).  Calls share the array:
 * calls that overlap on the GPU race and must be serialised by the caller. */
int gcu_dev_gemm_int8_noalloc(float *dst, int dstr, const int8_t *mat,
                              int mstr, const float *matsc, const int8_t *src,
                              int sstr, const float *ssc, int m, int n, int k,
                              void *stream);

/* One A operand against several weights in one launch, e.g. the prefill
 * Q/K/V projections (gemma.c:5045-5091) or up/gate (gemma.c:5367-5372):
 * job j writes dst_j (m, rows_j) dense.  Weights must be dense [rows_j][k]. */
int gcu_dev_gemm_int8_multi(const gcu_gemv_job *jobs, int njobs,
                            const int8_t *src, int sstr, const float *ssc,
                            int m, int k, void *stream);

/* quantize_acts followed by gemm_int8 / gemv_int8_multi on its result, in one
 * launch: gemma.c always calls them as a pair on the same activations
 * (gemma.c:4768-4773, 4911-4915, 5034-5091, 5365-5372, 5389-5391).  x holds
 * m fp32 rows (row stride xstr floats, 0 = k); the int8 codes go to q (dense
 * [m][k]) and the scales to s, exactly as gcu_dev_quantize_acts writes them,
 * and job j's output to its dst (m, rows_j) dense.  m <= 8: one launch, the
 * streaming GEMV kernel quantizes x while staging it; m > 8 (k % 16 == 0):
 * the quantize kernel and the tensor-core GEMM back to back (the GEMM's
 * prologue overlaps the quantize kernel).  Same bits as separate calls. */
int gcu_dev_quantize_gemm_int8_multi(const gcu_gemv_job *jobs, int njobs,
                                     int8_t *q, float *s, const float *x,
                                     int xstr, int m, int k, void *stream);

/* ---- chains of quantize_acts -> gemm_int8 steps, one launch -----------------
 * gemma.c's prefill is a sequence of such pairs (gemma.c:5034-5091 Q/K/V,
 * 5302-5304 O, 5365-5372 up/gate, 5389-5391 down; the vision tower at
 * 4497-4633).  A chain runs a list of them in order in ONE persistent
 * launch: step i quantizes x_i (m_i fp32 rows, row stride xstr floats, 0 =
 * k) into q_i (dense [m][k]) and s_i, then computes every job's gemm_int8
 * on them into its dst (dense [m][rows]).  Each step sees everything the
 * earlier steps wrote (x_i may be an earlier step's dst); weights and their
 * scales must not be written by the chain.  The bits are those of
 * gcu_dev_quantize_acts + gcu_dev_gemm_int8_multi called step by step.
 * Device pointers; m >= 1; k % 16 == 0, k <= 16384; 16-byte aligned x rows,
 * q and weights; 1..4 jobs per step.
 * create: plans every step's tiles and encodes its descriptors once (device
 * memory owned by the handle); the pointers are fixed from then on.
 * force: NULL, or per step {bn, mb, splits} to pin the tile shape
 * ((128*mb) x bn, mb 1 with bn 64/128/256 or mb 2 with bn 128/192/256) and
 * K split (0 = planner's).  run: enqueues cooperative launches on `stream`
 * (one CTA per SM, all resident at once).  plan: the chosen {bn, mb,
 * splits} per step.  No single counterpart in the reference. */
typedef struct {
  const float *x;
  int xstr;
  int8_t *q;
  float *s;
  int m, k;
  int njobs;
  gcu_gemv_job jobs[4];
} gcu_qgemm_step;
int gcu_gemm_chain_create(const gcu_qgemm_step *steps, int nsteps,
                          const int *force, int *handle);
int gcu_gemm_chain_run(int handle, void *stream);
int gcu_gemm_chain_plan(int handle, int *plan, int nsteps);
int gcu_gemm_chain_destroy(int handle);

/* ---- producers fused with quantize_acts -------------------------------------
 * gemma.c quantizes each block input right after its RMSNorm (rmsnorm,
 * gemma.c:2509-2524, at 4754 / 5026, then quantize_act(s) at 4768 / 5034) and
 * the down projection's input right after the GeGLU gate (gelu with `mul`,
 * gemma.c:4139-4170, at 4921 / 5379, then 4927 / 5389).  These compute the
 * producer and quantize its result in one pass over device memory: codes to
 * q (dense [m][dim]) and scales to s as gcu_dev_quantize_acts writes them,
 * and the fp32 result to `out` unless it is NULL.  dim % 4 == 0, dim <= 16384,
 * 16-byte aligned rows.  The quantize step is bit-exact on the computed
 * values; those values agree with gemma.c's to ~1e-6 relative (a different
 * summation order for the sum of squares, CUDA's tanhf), so a code can
 * differ by one where a value sits that close to a rounding boundary.
 * No single counterpart in the reference (each fuses two of its calls). */

/* out = (x * rms) * (weight + 1), rms = 1 / sqrtf(mean(x^2) + eps); x rows at
 * stride xstr floats (0 = dim), weight [dim]. */
int gcu_dev_rmsnorm_quantize(int8_t *q, float *s, float *out, const float *x, int xstr,
                             const float *weight, float eps, int m, int dim, void *stream);
/* out = gelu_tanh(gate) * up, gate and up dense [m][dim]. */
int gcu_dev_geglu_quantize(int8_t *q, float *s, float *out, const float *gate, const float *up,
                           int m, int dim, void *stream);

/* gemma.c:4862-4881, 4950-4962: the residual update after a block, m rows
 * of dim: x = clamp(resid + rmsnorm(y, weight)) (weight NULL: no post-norm,
 * x = clamp(resid + y)); clamp to the float range as clamp_fpx does.  x may
 * be resid.  dim a multiple of 4, at most 4096. */
int gcu_dev_rmsnorm_residual(float *x, const float *y, const float *resid, const float *weight,
                             float eps, int m, int dim, void *stream);
/* The residual update fused with the next block's norm + quantize: x =
 * clamp(resid + rmsnorm(y, w_post)) as gcu_dev_rmsnorm_residual, then the
 * codes q (dense [m][dim]) and scales s of rmsnorm(x, w_next) as
 * gcu_dev_rmsnorm_quantize -- one launch.  gemma.c runs the pair after the
 * attention block (n2, then n3: gemma.c:4862-4910) and across a layer
 * boundary (n4, then the next layer's n1: 4950-4962, 4754-4768). */
int gcu_dev_residual_norm_quantize(float *x, int8_t *q, float *s, const float *y, const float *resid,
                                   const float *w_post, const float *w_next, float eps, int m, int dim,
                                   void *stream);

/* One token (m = 1): a producer and the decode projection that consumes it in
 * one launch, every CTA of the GEMV computing the producer row itself.  The
 * codes, scale and outputs are bit for bit those of the producer call above
 * followed by gcu_dev_gemv_int8_multi on the same jobs; q and s receive the
 * codes and scale as the producer call writes them.
 *   geglu:    h = gelu_tanh(gate) * up over k (gemma.c:4921-4927 then the down
 *             projection 4929); k % 16 == 0, k <= 16384.
 *   residual: x = clamp(resid + rmsnorm(y, w_post)), then rmsnorm(x, w_next)
 *             quantized and multiplied (gemma.c:4862-4915 / 4950-4962 with
 *             4754-4773); dim % 16 == 0, dim <= 4096.  x must not overlap
 *             resid or y: every CTA reads those while one CTA writes x.
 * 16-byte aligned rows and codes.  No single counterpart in the reference. */
int gcu_dev_geglu_quantize_gemv_multi(const gcu_gemv_job *jobs, int njobs, int8_t *q, float *s,
                                      const float *gate, const float *up, int k, void *stream);
int gcu_dev_residual_norm_quantize_gemv_multi(const gcu_gemv_job *jobs, int njobs, float *x, int8_t *q,
                                              float *s, const float *y, const float *resid,
                                              const float *w_post, const float *w_next, float eps, int dim,
                                              void *stream);
/* gemma.c:4971-4976: x[i] = tanh(x[i] / cap) * cap (the final logit softcap). */
int gcu_dev_softcap(float *x, long n, float cap, void *stream);

/* ---- attention (fp32) between the Q/K/V and O matmuls ----------------------
 * gemma.c's KV cache layout (gemma.c:4806-4808): kv head hk's position t at
 * cache + hk*kv_stride + t*hdim (kv_stride = clen*hdim), K and V separate;
 * each cache holds nkv*kv_stride floats.  hdim 64, 128 or 256, at most 8
 * query heads per kv head, 16-byte aligned buffers.  fp32 arithmetic with
 * gemma.c's fast_expf softmax; results agree with the reference to fp32
 * reassociation (the reference's dot products are vectorized). */

/* gemma.c:4775-4818 (decode, ntok = 1) and 5095-5145 (prefill): the steps
 * between the Q/K/V matmuls and attention.  Per-head RMSNorm of the query and
 * key rows (weights nq / nk; NULL = the model has no qk_norm), RoPE with
 * freqs, the position's (cos, sin) table [ntok][hdim] exactly as gemma.c's
 * rope_freqs builds it for the layer kind, queries also scaled by q_scale (1
 * at decode, the attention scale at prefill), then the chunk's rotated keys
 * and its values written to the cache at [spos, spos+ntok).  xq
 * [n_heads][ntok][hdim] is rotated in place; xk, xv [nkv][ntok][hdim] are
 * only read.  8-byte aligned buffers. */
int gcu_dev_qk_norm_rope_cache(float *xq, const float *xk, const float *xv, float *k_cache,
                               float *v_cache, long kv_stride, const float *nq, const float *nk,
                               float eps, const float *freqs, float q_scale, int n_heads, int nkv,
                               int hdim, int spos, int ntok, void *stream);
/* The same step on the fused projection of a prefill chunk: row t of qkv
 * (row stride ld floats) holds the token's query heads, then its key heads,
 * then its value heads (one GEMM over wq|wk|wv gives exactly the values of
 * gemma.c's per-head GEMMs, gemma.c:5045-5091); the rotated queries go to xq
 * [n_heads][ntok][hdim], the rotated keys and the values to the cache. */
int gcu_dev_qkv_norm_rope_cache(float *xq, const float *qkv, long ld, float *k_cache, float *v_cache,
                                long kv_stride, const float *nq, const float *nk, float eps,
                                const float *freqs, float q_scale, int n_heads, int nkv, int hdim,
                                int spos, int ntok, void *stream);
/* gemma.c:4836-4848 (att_scores_gqa, att_finalize, att_values_gqa): one
 * decode step of one layer.  xq [n_heads][hdim] (normed and rotated), the
 * window [spos, spos+attlen) of the cache, scores scaled by asc
 * (1/sqrt(q_scale)) then soft-capped by sc_att (0 = off).  xo [n_heads][hdim]. */
int gcu_dev_attention_decode(float *xo, const float *xq, const float *k_cache, const float *v_cache,
                             long kv_stride, int n_heads, int nkv, int hdim, int spos, int attlen,
                             float asc, float sc_att, void *stream);
/* gcu_dev_qk_norm_rope_cache for one token at position pos = spos+attlen-1
 * (q_scale 1) followed by gcu_dev_attention_decode, in one launch: xq, xk, xv
 * are the Q/K/V projections as the GEMVs wrote them ([n_heads][hdim],
 * [nkv][hdim], [nkv][hdim]); each CTA normalises (nq / nk, NULL = no qk_norm)
 * and rotates its query heads with freqs (the position's table, hdim floats),
 * and the last CTA over each kv head's window writes the rotated key and the
 * value to cache row pos before reading it.  xo, and the cache rows, are bit
 * for bit those of the two calls; xq is left as it is (the two-call form
 * rotates it in place).  gemma.c:4775-4848. */
int gcu_dev_attention_decode_rope(float *xo, const float *xq, const float *xk, const float *xv,
                                  float *k_cache, float *v_cache, long kv_stride, const float *nq,
                                  const float *nk, float eps, const float *freqs, int n_heads, int nkv,
                                  int hdim, int spos, int attlen, float asc, float sc_att, void *stream);
/* gemma.c:5160-5295: a prefill chunk of ntok tokens at positions
 * [spos, spos+ntok) whose keys and values are already in the cache.  xq
 * [n_heads][ntok][hdim], rotated and scaled by the attention scale
 * (gemma.c:5121-5133).  mask = 1: causal, and a sliding window of `slide`
 * positions when slide > 0 (gemma.c's tc->swa[l] layers); mask = 0: every
 * token sees [0, spos+ntok).  Token i of head h goes to xo + i*xostr + h*hdim
 * (xostr 0 = n_heads*hdim, gemma.c's xo rows). */
int gcu_dev_attention_prefill(float *xo, int xostr, const float *xq, const float *k_cache,
                              const float *v_cache, long kv_stride, int n_heads, int nkv, int hdim,
                              int spos, int ntok, int slide, float sc_att, int mask, void *stream);

/* ---- SigLIP head (fp32) around the vision tower's matmuls ------------------
 * gemma.c:4411-4466: the patch embedding, Conv2d(3, dim, kernel = stride =
 * psize, bias) of the (img_px, img_px, 3) image img, then the int8 position
 * embedding (pos_q rows of dim, scales pos_s; the -q model's QTensor) added
 * dequantized; each step clamped to the float range.  pe [dim][3][psize][psize],
 * pe_b [dim]; x [(img_px/psize)^2][dim].  psize <= 16. */
int gcu_dev_patch_embed(float *x, const float *img, const float *pe, const float *pe_b,
                        const int8_t *pos_q, const float *pos_s, int img_px, int psize, int dim,
                        void *stream);
/* gemma.c:4660-4705 + the quantize_acts of 4714: LayerNorm (post_n, post_nb)
 * of every patch row of x [ppi*ppi][dim], the average of each
 * (ppi/side) x (ppi/side) block, gemma-style RMSNorm (norm), then the int8
 * codes q [side*side][dim] and scales s of the pooled rows -- the input of the
 * projection gcu_dev_gemm_int8.  out (may be NULL) receives the fp32 rows.
 * dim a multiple of 4, at most 4096. */
int gcu_dev_vision_pool_quantize(int8_t *q, float *s, float *out, const float *x, const float *post_n,
                                 const float *post_nb, const float *norm, float eps, int ppi, int side,
                                 int dim, void *stream);

/* ---- row-sharded entry points (NCCL over NVLink) ---------------------------
 * No counterpart in the reference, which is single-process (README.md:614).
 * Rank r of `world` owns weight rows [r*n/world, (r+1)*n/world) of an n-row
 * matrix (n divisible by world) and computes that slice; the slices are
 * all-gathered so every rank ends with the full output. */

/* 128-byte NCCL unique id, created on one rank and given to all. */
int gcu_comm_unique_id(unsigned char id[128]);
int gcu_comm_init(int rank, int world, const unsigned char id[128]);
int gcu_comm_destroy(void);
/* 1 if gcu_dev_gemm_int8_rowshard fuses its all-gather into the GEMV as
 * NVLink loads from the peers' buffers (m <= 8, every rank mapped every
 * peer's buffer through CUDA IPC at gcu_comm_init); 0 if it uses an NCCL
 * all-gather. */
int gcu_comm_fused_allgather(void);

/* dst (m, n) dense = sharded gemm_int8 with this rank's rows mat_local
 * (n/world rows) and scales matsc_local.  `work` is device scratch of
 * m*n floats used as the NCCL all-gather buffer.  m <= 8 uses the GEMV
 * kernel, with the all-gather fused into it when gcu_comm_fused_allgather()
 * is 1.  Every rank must make the same sequence of calls; calls of one rank
 * are ordered by its stream. */
int gcu_dev_gemm_int8_rowshard(float *dst, float *work,
                               const int8_t *mat_local,
                               const float *matsc_local, const int8_t *src,
                               const float *ssc, int m, int n, int k,
                               void *stream);

/* quantize_acts on x (m <= 8 fp32 rows, row stride xstr floats, 0 = k) and
 * the row-sharded gemm_int8 of every job on the result, e.g. a layer's
 * up/gate pair (gemma.c:4911-4915) with its FFN rows split over the ranks.
 * Job j: w / sc hold this rank's rows_j/world rows of weight j and their
 * scales, dst its full (m, rows_j) output, and the job's `m` field is the
 * FULL row count rows_j (a multiple of world).  q / s receive the codes and
 * scales as gcu_dev_quantize_acts writes them.  With the peers mapped
 * (gcu_comm_fused_allgather() == 1), m <= 8, k % 16 == 0, every slice a
 * multiple of 4 rows, 16-byte aligned dst and m * sum(rows_j) floats within
 * 8 MiB, this is ONE launch: the GEMV quantizes x while staging it, and one
 * cross-rank signal followed by NVLink loads completes the all-gather of all
 * jobs.  Otherwise it runs gcu_dev_quantize_acts and then
 * gcu_dev_gemm_int8_rowshard per job, using `work` (m * max rows_j floats)
 * as that call's scratch.  No counterpart in the reference. */
int gcu_dev_quantize_gemm_int8_rowshard_multi(const gcu_gemv_job *jobs, int njobs,
                                              int8_t *q, float *s, const float *x,
                                              int xstr, int m, int k, float *work,
                                              void *stream);

/* Gemma's feed-forward block for m > 8 tokens (gemma.c:5365-5391 with the
 * GeGLU of 4139-4170 between), the hidden dimension `ffn` split over the
 * ranks of gcu_comm_init (fl = ffn/world, a multiple of 16; dim % 16 == 0):
 *   up   = gemm_int8(w_up, xq, xs), gate = gemm_int8(w_gate, xq, xs)   rows [r*fl, (r+1)*fl) of w1 / w2
 *   h    = gelu(gate) * up;  (hq, hs) = quantize_acts(h)
 *   out  = gemm_int8(w_down, hq, hs)           w_down: columns [r*fl, (r+1)*fl) of w3, [dim][fl],
 *                                               row stride w_down_stride bytes (0 = fl)
 * s_down holds all dim scales of w3.  Each rank quantizes its slice of h with
 * the maxima of the full rows (an all-reduce of m floats) and sums its int32
 * partial products of down with the other ranks' (an all-reduce of m*dim
 * int32, exact), so `out` [m][dim] is the same on every rank and bit for
 * bit the unsharded block's.  Without gcu_comm_init it runs unsharded (the
 * same bits as gcu_dev_gemm_int8_multi + gcu_dev_geglu_quantize +
 * gcu_dev_gemm_int8).  No single counterpart in the reference (it is the
 * sharded form of three of its calls). */
int gcu_dev_ffn_rowshard(float *out, const int8_t *xq, const float *xs, int m, int dim, int ffn,
                         const int8_t *w_up, const float *s_up, const int8_t *w_gate,
                         const float *s_gate, const int8_t *w_down, int w_down_stride,
                         const float *s_down, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* GCU_H */
