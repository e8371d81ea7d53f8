/*
 * ref_harness.c -- exposes the reference's own hot-path functions.
 *
 * TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together
 * with the reference's gemma.c, included from where it lies (path given as
 * GEMMA_REF_SOURCE), with the reference Makefile's flags
 * (-O3 -ffast-math -march=... -fopenmp, DTYPE unset = FP32).  The result,
 * oracle/_ref/libgemma_ref_*.so, is used to pin the C restatement in
 * gemma_oracle.c and as the timed CPU baseline ("kind": "reference").
 *
 * gemma.c's functions are `static`, so they are wrapped here in the same
 * translation unit.  `main` is renamed before the include, and the one-letter
 * macros that the embedded stb blob leaks (gemma.c:7494 onwards) are
 * #undef'd by the generated header undef_blob.h before any code of ours.
 */
#define main gemma_ref_main
#include GEMMA_REF_SOURCE
#undef main
#include "undef_blob.h"

/* gemma.c:2590 */
float ref_quantize_act(int8_t *dst, const float *vec, int dim) {
  return quantize_act(dst, vec, dim, NULL);
}

/* gemma.c:2656; threads > 1 takes the OpenMP branch like the call sites
 * (gemma.c:4497, 5034) do with omp = true. */
void ref_quantize_acts(int8_t *dst, float *dsc, const float *src, int sstr,
                       int m, int n, int threads) {
  quantize_acts(dst, dsc, src, sstr, m, n, threads > 1, threads, NULL);
}

/* gemma.c:2770 */
void ref_gemv_int8(float *dst, const int8_t *mat, const float *matsc,
                   const int8_t *vec, float vsc, int m, int n, int threads) {
  gemv_int8(dst, mat, matsc, vec, vsc, m, n, threads > 1, threads, NULL);
}

/* gemma.c:2818; `jobs` points at GemvJob records (gemma.c:2795). */
void ref_gemv_int8_multi(const void *jobs, int njobs, const int8_t *vec,
                         float vsc, int n, int threads) {
  gemv_int8_multi((const GemvJob *)jobs, njobs, vec, vsc, n, threads, NULL);
}

/* gemma.c:3943 */
int ref_gemm_int8(float *dst, int dstr, const int8_t *mat, int mstr,
                  const float *matsc, const int8_t *src, int sstr,
                  const float *ssc, int m, int n, int k, int threads) {
  return gemm_int8(dst, dstr, mat, mstr, matsc, src, sstr, ssc, m, n, k,
                   threads > 1, threads, NULL);
}

/* The prefill Q/K/V projections as forward_text_chunk issues them
 * (gemma.c:5037-5091): one task per (tensor head, 128-token block), tasks
 * spread over `threads` OpenMP threads with a dynamic schedule, each task a
 * single-threaded gemm_int8 (omp = false) of its token block against one
 * head's hdim weight rows, written head-major into xq / xk / xv
 * ([head][ntok][hdim]).  Returns 1 if any task failed. */
int ref_qkv_head_tasks(float *xq, float *xk, float *xv, const int8_t *wq, const float *sq,
                       const int8_t *wk, const float *sk, const int8_t *wv, const float *sv,
                       const int8_t *x, const float *xsc, int ntok, int dim, int n_heads,
                       int nkv, int hdim, int threads) {
  const int rblock = 128;
  const int n_rb = (ntok + rblock - 1) / rblock;
  const int n_task = (n_heads + 2 * nkv) * n_rb;
  int quit = 0;
#pragma omp parallel for reduction(|| : quit) schedule(dynamic) num_threads(threads)
  for (int idx = 0; idx < n_task; idx++) {
    const int h = idx / n_rb;
    const int8_t *w;
    const float *sc;
    float *dst;
    int hd;
    if (h < n_heads) {
      w = wq, sc = sq, dst = xq, hd = h;
    } else if (h < n_heads + nkv) {
      w = wk, sc = sk, dst = xk, hd = h - n_heads;
    } else {
      w = wv, sc = sv, dst = xv, hd = h - n_heads - nkv;
    }
    const int t0 = (idx % n_rb) * rblock;
    const int tn = min(rblock, ntok - t0);
    float *dst_b = dst + ((size_t)hd * ntok + t0) * hdim;
    const size_t woff = (size_t)hd * hdim * dim;
    if (gemm_int8(dst_b, hdim, w + woff, 0, sc + hd * hdim, x + (size_t)t0 * dim, 0, xsc + t0,
                  tn, hdim, dim, false, threads, NULL) == 1)
      quit = 1;
  }
  return quit;
}

/* gemma.c:2509: gemma-style RMSNorm of one row (dst may equal src). */
void ref_rmsnorm(float *dst, const float *src, const float *weight, int dim, float eps) {
  rmsnorm(dst, src, weight, dim, eps, NULL);
}

/* gemma.c:4150: dst[i] = gelu_tanh(src[i] + bias) * mul[i] over rows x dim,
 * here without bias and with `mul` (the GeGLU gate * up of 4921, 5379). */
void ref_gelu_mul(float *dst, const float *src, const float *mul, int rows, int dim) {
  gelu(dst, src, rows, dim, NULL, mul, false, 1, NULL);
}

/* gemma.c:484: GEMM_MC / GEMM_NC / GEMM_KC tile sizes from the environment. */
void ref_setup(void) { setup_runtime_config(); }

/* gemma.c:4056: frees the calling thread's GEMM scratch. */
void ref_free_thread_scratch(void) { gemm_free_thread_scratch(); }

/* sizeof(GemvJob), so callers can check their record layout. */
int ref_gemv_job_size(void) { return (int)sizeof(GemvJob); }

/* which int8 micro-kernel this build selected (gemma.c:537-545). */
const char *ref_isa(void) {
#if defined(GEMMA_GEMM_VNNI8)
  return "avx-vnni-int8";
#elif defined(GEMMA_GEMM_AVX2)
  return "avx2";
#else
  return "portable";
#endif
}

/* gemma.c:1946 mmap_gemma_model, walked like its users do: every QTensor of
 * the matmul path as six numbers (kind, layer, int8 offset, scales offset,
 * rows, k), offsets from the mapping's base, in the order mmap_text_decoder
 * (gemma.c:1470) and mmap_vision_encoder (gemma.c:1765) lay them out.  The
 * kind numbers are gcu.h's gcu_qt_kind.  Returns the count, or -1 when the
 * reference refuses the file. */
int ref_bin_layout(const char *path, int allow_mm, long long *rec, int cap) {
  GemmaModel *m = mmap_gemma_model(path, allow_mm != 0);
  if (m == NULL || !m->quant) {
    if (m) munmap_gemma_model(m);
    return -1;
  }
  const uint8_t *base = (const uint8_t *)m->mm_data;
  int n = 0;
#define REF_PUT(KIND, LAYER, QT, ROWS, K)                            \
  do {                                                               \
    if (n < cap) {                                                   \
      long long *r = rec + 6 * n;                                    \
      r[0] = (KIND);                                                 \
      r[1] = (LAYER);                                                \
      r[2] = (long long)((const uint8_t *)(QT)->i8.q - base);        \
      r[3] = (long long)((const uint8_t *)(QT)->i8.scales - base);   \
      r[4] = (ROWS);                                                 \
      r[5] = (K);                                                    \
    }                                                                \
    n++;                                                             \
  } while (0)
  const TextDecoder *dec = m->decoder;
  const TextConfig *tc = dec->config;
  const int q_sz = tc->n_heads * tc->hdim, kv_sz = tc->nkv * tc->hdim;
  REF_PUT(0, -1, dec->emb, tc->nvocab, tc->dim);
  for (int l = 0; l < tc->nl; l++) {
    const TextDecoderLayer *L = dec->layers[l];
    REF_PUT(1, l, L->wq, q_sz, tc->dim);
    REF_PUT(2, l, L->wk, kv_sz, tc->dim);
    REF_PUT(3, l, L->wv, kv_sz, tc->dim);
    REF_PUT(4, l, L->wo, tc->dim, q_sz);
    REF_PUT(5, l, L->w1, tc->mlp_dim, tc->dim);
    REF_PUT(6, l, L->w2, tc->mlp_dim, tc->dim);
    REF_PUT(7, l, L->w3, tc->dim, tc->mlp_dim);
  }
  if (m->encoder) {
    const VisionEncoder *enc = m->encoder;
    const VisionConfig *vc = enc->config;
    for (int l = 0; l < vc->nl; l++) {
      const VisionEncoderLayer *L = enc->layers[l];
      REF_PUT(8, l, L->wq, vc->dim, vc->dim);
      REF_PUT(9, l, L->wk, vc->dim, vc->dim);
      REF_PUT(10, l, L->wv, vc->dim, vc->dim);
      REF_PUT(11, l, L->wo, vc->dim, vc->dim);
      REF_PUT(12, l, L->w1, vc->mlp_dim, vc->dim);
      REF_PUT(13, l, L->w2, vc->dim, vc->mlp_dim);
    }
    REF_PUT(14, -1, enc->proj, tc->dim, vc->dim);
  }
#undef REF_PUT
  munmap_gemma_model(m);
  return n;
}

/* gemma.c:2045 read_gemma_model: the reference's own load of a model file
 * into host memory (every tensor fread into its own buffer).  Returns the
 * seconds it took (CLOCK_MONOTONIC, the free afterwards not counted), or -1
 * when the reference refuses the file. */
double ref_read_model_seconds(const char *path, int allow_mm) {
  struct timespec t0, t1;
  clock_gettime(CLOCK_MONOTONIC, &t0);
  GemmaModel *m = read_gemma_model(path, allow_mm != 0);
  clock_gettime(CLOCK_MONOTONIC, &t1);
  if (m == NULL) return -1.0;
  free_gemma_model(m);
  return (double)(t1.tv_sec - t0.tv_sec) + 1e-9 * (double)(t1.tv_nsec - t0.tv_nsec);
}

/* gemma.c:4836-4848: one decode step's attention, through the reference's
 * own att_scores_gqa, att_finalize and att_values_gqa, with its buffer
 * layout (att row h starts at att + spos + h*attlen; the cache rows of kv
 * head hk at kc/vc + hk*kv_stride).  att: spos + n_heads*attlen floats. */
void ref_attention_decode(float *xo, const float *xq, const float *kc, const float *vc,
                          long kv_stride, int n_heads, int nkv, int hdim, int spos, int attlen,
                          float asc, float sc_att, float *att, int threads) {
  att_scores_gqa(att + spos, attlen, xq, kc + (size_t)spos * hdim, (int)kv_stride, nkv, n_heads,
                 attlen, hdim, threads, NULL);
  for (int h = 0; h < n_heads; h++)
    att_finalize(att + (size_t)h * attlen + spos, attlen, asc, sc_att, NULL);
  att_values_gqa(xo, att + spos, attlen, vc + (size_t)spos * hdim, (int)kv_stride, nkv, n_heads,
                 attlen, hdim, threads, NULL);
}

/* gemma.c:5160-5295: a prefill chunk's attention, the per (head, query
 * block) loop of forward_text_chunk restated around the reference's own
 * gemm_fpx, softmax and gemm_fpx_nn.  xq [n_heads][ntok][hdim] (rotated and
 * scaled); slide > 0 marks a sliding-window layer (tc->swa[l], tc->slide);
 * xo row i of head h at xo + i*xostr + h*hdim.  att: n_heads*ntok*(spos+ntok)
 * floats.  `threads` OpenMP threads over the (head, query block) tasks, as
 * the reference runs them; each task calls the GEMMs single-threaded. */
int ref_attention_prefill(float *xo, int xostr, const float *xq, const float *kc, const float *vc,
                          long kv_stride, int n_heads, int nkv, int hdim, int spos, int ntok,
                          int slide, float sc_att, int mask, float *att, int threads) {
  const bool sliding = slide > 0;
  const int epos = spos + ntok - 1, max_k = epos + 1;
  const int qk = g_rt.qk_blk;
  const int n_qb = mask ? (ntok + qk - 1) / qk : 1;
  bool quit = false;
  int qidx;
#pragma omp parallel for private(qidx) schedule(dynamic) reduction(|| : quit) num_threads(threads)
  for (qidx = 0; qidx < n_heads * n_qb; qidx++) {
    const int h = qidx / n_qb, qbi = qidx % n_qb;
    const int h_kv = h * nkv / n_heads;
    float *att_h = att + (size_t)h * ntok * max_k;
    const float *xv_head = vc + (size_t)h_kv * kv_stride;
    float *xo_head = xo + (size_t)h * hdim;
    if (mask) {
      const int q_start = qbi * qk;
      const float *qb = xq + (size_t)h * ntok * hdim + (size_t)q_start * hdim;
      const int q_end = min(q_start + qk, ntok);
      const int qabs_e = spos + q_end;
      int qabs_s = spos + q_start;
      if (sliding && qabs_s >= slide)
        qabs_s = qabs_s + 1 - slide;
      else
        qabs_s = 0;
      const int spos_b = qabs_s / qk * qk;
      for (int k_start = spos_b; k_start < qabs_e; k_start += qk) {
        const float *kb = kc + (size_t)h_kv * kv_stride + (size_t)k_start * hdim;
        const int k_end = min(k_start + qk, max_k);
        float *att_b = att_h + (size_t)q_start * max_k + k_start;
        if (gemm_fpx(att_b, max_k, kb, 0, qb, 0, q_end - q_start, k_end - k_start, hdim, false, 1, NULL))
          quit = true;
        for (int qi = q_start; qi < q_end; qi++) {
          const int pos_i = spos + qi;
          const int spos_i = (sliding && pos_i >= slide) ? (pos_i + 1 - slide) : 0;
          for (int ki = k_start; ki < k_end; ki++)
            if (ki > pos_i || ki < spos_i) att_h[(size_t)qi * max_k + ki] = 0.0f;
        }
      }
      for (int qi = q_start; qi < q_end; qi++) {
        float *att_row = att_h + (size_t)qi * max_k;
        const int pos_i = spos + qi;
        const int spos_i = (sliding && pos_i >= slide) ? (pos_i + 1 - slide) : 0;
        if (sc_att != 0.0f)
          for (int t = spos_i; t <= pos_i; t++) att_row[t] = tanhf(att_row[t] / sc_att) * sc_att;
        softmax(att_row + spos_i, att_row + spos_i, pos_i - spos_i + 1, NULL);
      }
      gemm_fpx_nn(xo_head + (size_t)q_start * xostr, xostr, xv_head + (size_t)spos_b * hdim, 0,
                  att_h + (size_t)q_start * max_k + spos_b, max_k, q_end - q_start, hdim, qabs_e - spos_b,
                  false, 1, NULL);
    } else {
      const float *xq_head = xq + (size_t)h * ntok * hdim;
      const float *xk_head = kc + (size_t)h_kv * kv_stride;
      if (gemm_fpx(att_h, max_k, xk_head, 0, xq_head, 0, ntok, max_k, hdim, false, 1, NULL)) quit = true;
      for (int qi = 0; qi < ntok; qi++) {
        float *att_row = att_h + (size_t)qi * max_k;
        if (sc_att != 0.0f)
          for (int t = 0; t < max_k; t++) att_row[t] = tanhf(att_row[t] / sc_att) * sc_att;
        softmax(att_row, att_row, max_k, NULL);
      }
      gemm_fpx_nn(xo_head, xostr, xv_head, 0, att_h, max_k, ntok, hdim, max_k, false, 1, NULL);
    }
  }
  return quit ? 1 : 0;
}

/* gemma.c:4391 forward_vision on an encoder with no layers: the patch
 * embedding and position embedding (gemma.c:4411-4466), the post LayerNorm,
 * average pooling and RMSNorm (gemma.c:4660-4705), then quantize_acts and the
 * int8 projection (gemma.c:4714-4716) -- the reference's own code end to end.
 * img [img_px][img_px][3]; pe [dim][3][psize][psize]; pos_q/pos_s the
 * position embedding QTensor (npatch rows of dim); proj_q/proj_s the
 * projection QTensor (tdim rows of dim).  Outputs: out [img_tok][tdim] (the
 * projection), and when non-null the pooled RMSNorm'd rows pooled
 * [img_tok][dim] with their codes q and scales s. */
int ref_vision_head(float *out, float *pooled, int8_t *q, float *s, const float *img, int img_px,
                    int psize, int dim, int img_tok, int tdim, float eps, const float *pe,
                    const float *pe_b, const int8_t *pos_q, const float *pos_s, const float *post_n,
                    const float *post_nb, const float *norm, const int8_t *proj_q,
                    const float *proj_s, int threads) {
  const int ppi = img_px / psize, npatch = ppi * ppi;
  VisionConfig vc;
  memset(&vc, 0, sizeof(vc));
  vc.nl = 0;
  vc.n_heads = 1;
  vc.img_px = (uint16_t)img_px;
  vc.psize = (uint16_t)psize;
  vc.dim = (uint16_t)dim;
  vc.mlp_dim = (uint16_t)dim;
  vc.eps = eps;
  TextConfig tc;
  memset(&tc, 0, sizeof(tc));
  tc.img_tok = (uint16_t)img_tok;
  tc.dim = (uint16_t)tdim;
  QTensor pos, proj;
  memset(&pos, 0, sizeof(pos));
  memset(&proj, 0, sizeof(proj));
  pos.quant = true;
  pos.i8.q = (int8_t *)pos_q;
  pos.i8.scales = (floatx *)pos_s;
  proj.quant = true;
  proj.i8.q = (int8_t *)proj_q;
  proj.i8.scales = (floatx *)proj_s;
  VisionEncoder enc;
  memset(&enc, 0, sizeof(enc));
  enc.config = &vc;
  enc.pe = (floatx *)pe;
  enc.pe_b = (floatx *)pe_b;
  enc.pos_emb = &pos;
  enc.layers = NULL;
  enc.post_n = (floatx *)post_n;
  enc.post_nb = (floatx *)post_nb;
  enc.norm = (floatx *)norm;
  enc.proj = &proj;
  VisionBuffer vb;
  memset(&vb, 0, sizeof(vb));
  vb.x = malloc((size_t)npatch * dim * sizeof(floatx));
  vb.x_i8 = malloc((size_t)npatch * dim);
  vb.xsc = malloc((size_t)npatch * sizeof(floatx));
  TextBuffer tb;
  memset(&tb, 0, sizeof(tb));
  tb.x = out;
  int rc = 1;
  if (vb.x && vb.x_i8 && vb.xsc) {
    rc = forward_vision(&enc, &tc, &tb, &vb, img, true, threads, NULL);
    if (pooled) memcpy(pooled, vb.x, (size_t)img_tok * dim * sizeof(floatx));
    if (q) memcpy(q, vb.x_i8, (size_t)img_tok * dim);
    if (s) memcpy(s, vb.xsc, (size_t)img_tok * sizeof(floatx));
  }
  free(vb.x);
  free(vb.x_i8);
  free(vb.xsc);
  return rc;
}

/* gemma.c:4198-4216 rope_freqs: the cos/sin tables (hdim floats per
 * position, `stride` apart) for n positions from pos, sliding and full. */
void ref_rope_freqs(float *slid, float *full, int hdim, int stride, float theta_l, float theta_g, int pos, int n) {
  rope_freqs(slid, full, hdim, stride, theta_l, theta_g, pos, n, 1, NULL);
}

/* The steps between the Q/K/V matmuls and attention, as the call sites run
 * them: per-head QK RMSNorm (gemma.c:4778-4790 decode, 5095-5113 prefill;
 * skipped when nq / nk are NULL), rope_apply on q (scaled by q_scale: 1 at
 * decode, the attention scale at prefill, gemma.c:4796-4797, 5121-5133) and
 * on k, then the K/V cache writes (gemma.c:4806-4818, 5136-5145).  xq
 * [n_heads][ntok][hdim] and xk [nkv][ntok][hdim] are changed in place, as in
 * gemma.c; freqs is one table block per position (stride hdim). */
void ref_qk_norm_rope_cache(float *xq, float *xk, const float *xv, float *kc, float *vc, long kv_stride,
                            const float *nq, const float *nk, float eps, const float *freqs, float q_scale,
                            int n_heads, int nkv, int hdim, int spos, int ntok) {
  if (nq)
    for (int h = 0; h < n_heads; h++)
      for (int t = 0; t < ntok; t++) {
        float *row = xq + ((size_t)h * ntok + t) * hdim;
        rmsnorm(row, row, nq, hdim, eps, NULL);
      }
  if (nk)
    for (int h = 0; h < nkv; h++)
      for (int t = 0; t < ntok; t++) {
        float *row = xk + ((size_t)h * ntok + t) * hdim;
        rmsnorm(row, row, nk, hdim, eps, NULL);
      }
  for (int h = 0; h < n_heads; h++) rope_apply(xq + (size_t)h * ntok * hdim, ntok, hdim, freqs, hdim, q_scale, NULL);
  for (int h = 0; h < nkv; h++) rope_apply(xk + (size_t)h * ntok * hdim, ntok, hdim, freqs, hdim, 1.0f, NULL);
  for (int h = 0; h < nkv; h++) {
    memcpy(kc + (size_t)h * kv_stride + (size_t)spos * hdim, xk + (size_t)h * ntok * hdim,
           (size_t)ntok * hdim * sizeof(float));
    memcpy(vc + (size_t)h * kv_stride + (size_t)spos * hdim, xv + (size_t)h * ntok * hdim,
           (size_t)ntok * hdim * sizeof(float));
  }
}

/* A W8A8 text decoder (gemma.c:1174-1301) around caller-owned tensors, and
 * a TextBuffer (gemma.c:2241-2273) for chunks of up to ntok tokens. */
typedef struct {
  TextConfig tc;
  bool *flags;
  QTensor *qts;
  TextDecoderLayer *lay;
  TextDecoderLayer **lp;
  TextDecoder dec;
} RefDecoder;

static void ref_free_decoder(RefDecoder *m) {
  free(m->flags);
  free(m->qts);
  free(m->lay);
  free(m->lp);
}

/* qt: 14 pointers per layer (wq, wk, wv, wo, w1 = up, w2 = gate, w3 = down;
 * int8 values then fp32 scales each); nrm: 6 per layer (n1, n2, n3, n4, nq,
 * nk); swa: the sliding-window flag per layer. */
static int ref_build_decoder(RefDecoder *m, int nl, int n_heads, int nkv, int hdim, int dim, int mlp_dim,
                             int nvocab, int q_scale, int slide, int max_seq, const int *swa, int qk_norm,
                             int mlp_pre, int mlp_pst, float theta_l, float theta_g, float eps, float sc_att,
                             float sc_log, void *const *qt, float *const *nrm, const int8_t *emb_q,
                             const float *emb_s, const float *fnorm) {
  memset(m, 0, sizeof(*m));
  TextConfig *tc = &m->tc;
  tc->nl = (uint8_t)nl;
  tc->n_heads = (uint8_t)n_heads;
  tc->nkv = (uint8_t)nkv;
  tc->hdim = (uint16_t)hdim;
  tc->dim = (uint16_t)dim;
  tc->mlp_dim = (uint16_t)mlp_dim;
  tc->q_scale = (uint16_t)q_scale;
  tc->slide = (uint16_t)slide;
  tc->max_seq = (uint32_t)max_seq;
  tc->nvocab = (uint32_t)nvocab;
  tc->theta_l = theta_l;
  tc->theta_g = theta_g;
  tc->eps = eps;
  tc->sc_att = sc_att;
  tc->sc_log = sc_log;
  tc->qk_norm = qk_norm != 0;
  tc->mlp_pre = mlp_pre != 0;
  tc->mlp_pst = mlp_pst != 0;
  m->flags = calloc((size_t)nl, sizeof(bool));
  m->qts = calloc((size_t)nl * 7 + 1, sizeof(QTensor));
  m->lay = calloc((size_t)nl, sizeof(TextDecoderLayer));
  m->lp = calloc((size_t)nl, sizeof(TextDecoderLayer *));
  if (!m->flags || !m->qts || !m->lay || !m->lp) return 1;
  for (int l = 0; l < nl; l++) {
    m->flags[l] = swa[l] != 0;
    QTensor *t = m->qts + (size_t)l * 7;
    for (int j = 0; j < 7; j++) {
      t[j].quant = true;
      t[j].i8.q = (int8_t *)qt[(size_t)l * 14 + 2 * j];
      t[j].i8.scales = (floatx *)qt[(size_t)l * 14 + 2 * j + 1];
    }
    TextDecoderLayer *L = m->lay + l;
    L->wq = t + 0;
    L->wk = t + 1;
    L->wv = t + 2;
    L->wo = t + 3;
    L->w1 = t + 4;
    L->w2 = t + 5;
    L->w3 = t + 6;
    L->n1 = nrm[(size_t)l * 6 + 0];
    L->n2 = nrm[(size_t)l * 6 + 1];
    L->n3 = nrm[(size_t)l * 6 + 2];
    L->n4 = nrm[(size_t)l * 6 + 3];
    L->nq = nrm[(size_t)l * 6 + 4];
    L->nk = nrm[(size_t)l * 6 + 5];
    m->lp[l] = L;
  }
  tc->swa = m->flags;
  QTensor *emb = m->qts + (size_t)nl * 7;
  emb->quant = true;
  emb->i8.q = (int8_t *)emb_q;
  emb->i8.scales = (floatx *)emb_s;
  m->dec.config = tc;
  m->dec.emb = emb;
  m->dec.layers = m->lp;
  m->dec.fnorm = (floatx *)fnorm;
  return 0;
}

static void ref_free_tb(TextBuffer *tb) {
  free(tb->x_i8);
  free(tb->xsc);
  free(tb->xo_i8);
  free(tb->xosc);
  free(tb->xg_i8);
  free(tb->xgsc);
  free(tb->cs_slid);
  free(tb->cs_full);
  free(tb->x);
  free(tb->resid);
  free(tb->xq);
  free(tb->xk);
  free(tb->xv);
  free(tb->xo);
  free(tb->att);
  free(tb->kvc);
  free(tb->xg);
  free(tb->xu);
  free(tb->logits);
}

static int ref_alloc_tb(TextBuffer *tb, const TextConfig *tc, int ntok, int clen) {
  memset(tb, 0, sizeof(*tb));
  const size_t dim = tc->dim, mlp = tc->mlp_dim, q_sz = (size_t)tc->n_heads * tc->hdim,
               kv_sz = (size_t)tc->nkv * tc->hdim, n = (size_t)ntok;
  tb->clen = clen;
  tb->x_i8 = malloc(n * (dim > q_sz ? dim : q_sz));
  tb->xsc = malloc(n * sizeof(float));
  tb->xo_i8 = malloc(n * q_sz);
  tb->xosc = malloc(n * sizeof(float));
  tb->xg_i8 = malloc(n * mlp);
  tb->xgsc = malloc(n * sizeof(float));
  tb->cs_slid = malloc(n * tc->hdim * sizeof(float));
  tb->cs_full = malloc(n * tc->hdim * sizeof(float));
  tb->x = malloc(n * dim * sizeof(float));
  tb->resid = malloc(n * dim * sizeof(float));
  tb->xq = malloc(n * q_sz * sizeof(float));
  tb->xk = malloc(n * kv_sz * sizeof(float));
  tb->xv = malloc(n * kv_sz * sizeof(float));
  tb->xo = malloc(n * q_sz * sizeof(float));
  tb->att = malloc((size_t)tc->n_heads * n * clen * sizeof(float));
  tb->kvc = calloc((size_t)tc->nl * 2 * clen * kv_sz, sizeof(float));
  tb->xg = malloc(n * mlp * sizeof(float));
  tb->xu = malloc(n * mlp * sizeof(float));
  tb->logits = malloc((size_t)tc->nvocab * sizeof(float));
  return !(tb->x_i8 && tb->xsc && tb->xo_i8 && tb->xosc && tb->xg_i8 && tb->xgsc && tb->cs_slid && tb->cs_full &&
           tb->x && tb->resid && tb->xq && tb->xk && tb->xv && tb->xo && tb->att && tb->kvc && tb->xg && tb->xu &&
           tb->logits);
}

/* gemma.c:4727-4978 forward_text_decode, the reference's whole decode step,
 * on a decoder built from the given tensors: npos steps at positions
 * 0 .. npos-1, step p's input embedding x0[p] placed in tb->x as its caller
 * does (gemma.c:5470-5490).  Outputs per step: the logits (after the
 * optional softcap) and the final hidden state (after the final RMSNorm). */
int ref_decode_steps(float *logits, float *hid, const float *x0, int npos, int nl, int n_heads, int nkv,
                     int hdim, int dim, int mlp_dim, int nvocab, int q_scale, int slide, const int *swa,
                     int qk_norm, int mlp_pre, int mlp_pst, float theta_l, float theta_g, float eps, float sc_att,
                     float sc_log, void *const *qt, float *const *nrm, const int8_t *emb_q, const float *emb_s,
                     const float *fnorm, int threads) {
  RefDecoder m;
  TextBuffer tb;
  int rc = ref_build_decoder(&m, nl, n_heads, nkv, hdim, dim, mlp_dim, nvocab, q_scale, slide, npos, swa, qk_norm,
                             mlp_pre, mlp_pst, theta_l, theta_g, eps, sc_att, sc_log, qt, nrm, emb_q, emb_s, fnorm);
  rc = rc || ref_alloc_tb(&tb, &m.tc, 1, npos);
  for (int p = 0; p < npos && rc == 0; p++) {
    memcpy(tb.x, x0 + (size_t)p * dim, (size_t)dim * sizeof(float));
    rc = forward_text_decode(&m.dec, &tb, p, true, true, threads, NULL);
    memcpy(logits + (size_t)p * nvocab, tb.logits, (size_t)nvocab * sizeof(float));
    memcpy(hid + (size_t)p * dim, tb.x, (size_t)dim * sizeof(float));
  }
  ref_free_tb(&tb);
  ref_free_decoder(&m);
  return rc;
}

/* gemma.c:4985-5455 forward_text_chunk, the reference's prefill of a chunk,
 * on the same kind of decoder: chunks[c] tokens at a time from position 0
 * (causal mask, as prompt processing calls it), chunk c's input embeddings
 * the next chunks[c] rows of x0.  Outputs: each chunk's last-token logits,
 * and every token's final hidden state (after the final RMSNorm). */
int ref_prefill_chunks(float *logits, float *hid, const float *x0, const int *chunks, int nchunks, int nl,
                       int n_heads, int nkv, int hdim, int dim, int mlp_dim, int nvocab, int q_scale, int slide,
                       const int *swa, int qk_norm, int mlp_pre, int mlp_pst, float theta_l, float theta_g,
                       float eps, float sc_att, float sc_log, void *const *qt, float *const *nrm,
                       const int8_t *emb_q, const float *emb_s, const float *fnorm, int threads) {
  int total = 0, maxc = 1;
  for (int c = 0; c < nchunks; c++) {
    total += chunks[c];
    maxc = chunks[c] > maxc ? chunks[c] : maxc;
  }
  RefDecoder m;
  TextBuffer tb;
  int rc = ref_build_decoder(&m, nl, n_heads, nkv, hdim, dim, mlp_dim, nvocab, q_scale, slide, total, swa,
                             qk_norm, mlp_pre, mlp_pst, theta_l, theta_g, eps, sc_att, sc_log, qt, nrm, emb_q,
                             emb_s, fnorm);
  rc = rc || ref_alloc_tb(&tb, &m.tc, maxc, total);
  for (int c = 0, spos = 0; c < nchunks && rc == 0; spos += chunks[c], c++) {
    memcpy(tb.x, x0 + (size_t)spos * dim, (size_t)chunks[c] * dim * sizeof(float));
    rc = forward_text_chunk(&m.dec, &tb, spos, chunks[c], true, true, true, threads, NULL);
    memcpy(logits + (size_t)c * nvocab, tb.logits, (size_t)nvocab * sizeof(float));
    memcpy(hid + (size_t)spos * dim, tb.x, (size_t)chunks[c] * dim * sizeof(float));
  }
  ref_free_tb(&tb);
  ref_free_decoder(&m);
  return rc;
}

/* 1 when this build routes the hot path through the CUDA drop-in
 * (gemma_gcu.h, built with -DGEMMA_CUDA), 0 for the reference's own code. */
int ref_dropin(void) {
#if defined(GEMMA_CUDA)
  return 1;
#else
  return 0;
#endif
}

/* gemma.c's own model path, end to end: setup_gemma_model (gemma.c:6867,
 * read_gemma_model or mmap_gemma_model, plus the registration hook in a
 * GEMMA_CUDA build), then optionally forward_gemma_image (gemma.c:5561: the
 * SigLIP tower, its projection and the image tokens' prefill), then
 * forward_gemma_prefill (gemma.c:5497) of nprompt tokens in chunks of `chunk`
 * with logits, then ndecode forward_gemma_decode steps (gemma.c:5456), and
 * cleanup_gemma_model (gemma.c:6909).  logits receives (1 + ndecode) rows of
 * nvocab: the prompt's last logits, then each decode step's.  Returns 0, or
 * 1 when any stage fails (the message is in gemma.c's g_err). */
int ref_model_run(const char *path, int mmap_on, int allow_mm, int seqlen, int chunk, const float *image,
                  const int *tokens, int nprompt, int ndecode, float *logits, int nvocab, int threads) {
  GemmaModel *model = NULL;
  TextBuffer *tb = NULL;
  VisionBuffer *vb = NULL;
  int rc = setup_gemma_model(path, mmap_on != 0, allow_mm != 0, seqlen, chunk, &model, &tb, &vb);
  int pos = 0;
  if (rc == 0 && (int)model->decoder->config->nvocab != nvocab) rc = 1;
  if (rc == 0 && image != NULL)
    rc = forward_gemma_image(model, tb, vb, image, &pos, false, threads, NULL);
  if (rc == 0) {
    rc = forward_gemma_prefill(model, tb, (int *)tokens, nprompt, &pos, chunk, NULL, true, threads, NULL);
    if (rc == 0) memcpy(logits, tb->logits, (size_t)nvocab * sizeof(float));
  }
  for (int i = 0; i < ndecode && rc == 0; i++, pos++) {
    rc = forward_gemma_decode(model, tb, tokens[nprompt + i], pos, threads, NULL);
    if (rc == 0) memcpy(logits + (size_t)(1 + i) * nvocab, tb->logits, (size_t)nvocab * sizeof(float));
  }
  if (model != NULL) cleanup_gemma_model(model, tb, vb, mmap_on != 0);
  return rc;
}

/* Device bytes the registration hook holds while the model is set up
 * (GEMMA_CUDA builds; -1 elsewhere): setup_gemma_model, gcu_registered_bytes,
 * cleanup_gemma_model. */
long long ref_model_registered_bytes(const char *path, int mmap_on, int allow_mm, int seqlen, int chunk) {
#if defined(GEMMA_CUDA)
  GemmaModel *model = NULL;
  TextBuffer *tb = NULL;
  VisionBuffer *vb = NULL;
  long long held = -1;
  if (setup_gemma_model(path, mmap_on != 0, allow_mm != 0, seqlen, chunk, &model, &tb, &vb) == 0)
    held = (long long)gcu_registered_bytes();
  if (model != NULL) cleanup_gemma_model(model, tb, vb, mmap_on != 0);
  return held;
#else
  (void)path, (void)mmap_on, (void)allow_mm, (void)seqlen, (void)chunk;
  return -1;
#endif
}
