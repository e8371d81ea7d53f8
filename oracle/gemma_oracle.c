/*
 * gemma_oracle.c -- CPU restatement of Gemma.c's W8A8 matmul hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the CUDA library is
 * compared against; nothing in the product links it.  Only tests/, the
 * smoke() entry point and bench.py's cpu_baseline leg load it.
 *
 * Parity pinning: the reference ships no tests or golden vectors, so this
 * restatement is pinned against the reference's own functions compiled from
 * gemma.c by oracle/Makefile (target `ref`, output in oracle/_ref/), through
 * the committed fixtures in tests/golden/ and a randomized cross-check.
 *
 * Arithmetic follows the reference built the way its Makefile builds it
 * (-O3 -ffast-math -march=native).  Under -ffast-math gcc rewrites three
 * expressions of the source, and this file states the rewritten forms:
 *   scale = amax * (1/127)      for `amax / 127.0f`        (gemma.c:2615)
 *   inv   = 127 / amax          for `1.0f / scale`         (gemma.c:2616)
 *   y     = (float)acc * (xs*ws) for `acc * xs * ws`       (gemma.c:2762, 3862)
 * This file must itself be compiled WITHOUT fast-math and without FMA
 * contraction (-O3 -ffp-contract=off), so the C text is the arithmetic.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* Per-vector symmetric int8 quantization, gemma.c:2586-2650 (quantize_act).
 * Round half away from zero by truncating v +/- 0.5 (gemma.c:2628-2631 and
 * 2642-2645), clamp to [-127, 127].  amax == 0 gives scale 1, inv 1. */
float orc_quantize_act(int8_t *dst, const float *vec, int dim) {
  float amax = 0.0f;
  for (int d = 0; d < dim; d++) {
    float a = fabsf(vec[d]);
    amax = a > amax ? a : amax;
  }
  float scale = amax > 0.0f ? amax * (1.0f / 127.0f) : 1.0f;
  float inv = amax > 0.0f ? 127.0f / amax : 1.0f;
  for (int d = 0; d < dim; d++) {
    float v = vec[d] * inv;
    float t = v + (signbit(v) ? -0.5f : 0.5f);
    int q = (int)t; /* C conversion truncates toward zero */
    dst[d] = (int8_t)(q > 127 ? 127 : (q < -127 ? -127 : q));
  }
  return scale;
}

/* Row loop of quantize_acts, gemma.c:2652-2674: sstr == 0 means dense rows
 * of n; dst is always dense (m, n). */
void orc_quantize_acts(int8_t *dst, float *dsc, const float *src, int sstr,
                       int m, int n) {
  if (sstr == 0)
    sstr = n;
  for (int i = 0; i < m; i++)
    dsc[i] = orc_quantize_act(dst + (size_t)i * n, src + (size_t)i * sstr, n);
}

/* int32 accumulators of the NT product acc[i][j] = sum_l src[i,l]*mat[j,l]
 * (the quantity gemm_int8_kernel_dot/_widen/_accum and gemv_int8_row sum,
 * gemma.c:2758-2761, 3617-3661, 3675-3845).  Integer addition is exact and
 * order independent, so any summation order gives the same bits. */
void orc_acc_int8(int32_t *acc, const int8_t *mat, int mstr,
                  const int8_t *src, int sstr, int m, int n, int k) {
  if (mstr == 0)
    mstr = k;
  if (sstr == 0)
    sstr = k;
  for (int i = 0; i < m; i++) {
    const int8_t *a = src + (size_t)i * sstr;
    for (int j = 0; j < n; j++) {
      const int8_t *b = mat + (size_t)j * mstr;
      int32_t s = 0;
      for (int l = 0; l < k; l++)
        s += (int32_t)a[l] * (int32_t)b[l];
      acc[(size_t)i * n + j] = s;
    }
  }
}

/* Dequant epilogue: (float)acc * (xs * ws), gemma.c:2762 / 3859-3862 in the
 * form the -ffast-math build evaluates. */
static inline float orc_dequant(int32_t acc, float xs, float ws) {
  return (float)acc * (xs * ws);
}

/* gemv_int8, gemma.c:2765-2788: dst[i] = dot(mat row i, vec) dequantized.
 * m = rows of mat (outputs), n = reduction length. */
void orc_gemv_int8(float *dst, const int8_t *mat, const float *matsc,
                   const int8_t *vec, float vsc, int m, int n) {
  for (int i = 0; i < m; i++) {
    const int8_t *w = mat + (size_t)i * n;
    int32_t s = 0;
    for (int l = 0; l < n; l++)
      s += (int32_t)w[l] * (int32_t)vec[l];
    dst[i] = orc_dequant(s, vsc, matsc[i]);
  }
}

/* GemvJob, gemma.c:2795-2800 (floatx = float). */
typedef struct {
  const void *w;
  const float *sc;
  float *dst;
  int m;
} OrcGemvJob;

/* gemv_int8_multi, gemma.c:2814-2837: every job shares vec, vsc and n. */
void orc_gemv_int8_multi(const OrcGemvJob *jobs, int njobs,
                         const int8_t *vec, float vsc, int n) {
  for (int j = 0; j < njobs; j++)
    orc_gemv_int8(jobs[j].dst, (const int8_t *)jobs[j].w, jobs[j].sc, vec,
                  vsc, jobs[j].m, n);
}

/* gemm_int8, gemma.c:3937-4054: NT GEMM with per-row (ssc) and per-column
 * (matsc) scales.  Strides of 0 mean dense (dstr = n, mstr = sstr = k).
 * Returns 0 like the reference on success. */
int orc_gemm_int8(float *dst, int dstr, const int8_t *mat, int mstr,
                  const float *matsc, const int8_t *src, int sstr,
                  const float *ssc, int m, int n, int k) {
  if (dstr == 0)
    dstr = n;
  if (mstr == 0)
    mstr = k;
  if (sstr == 0)
    sstr = k;
  for (int i = 0; i < m; i++) {
    const int8_t *a = src + (size_t)i * sstr;
    for (int j = 0; j < n; j++) {
      const int8_t *b = mat + (size_t)j * mstr;
      int32_t s = 0;
      for (int l = 0; l < k; l++)
        s += (int32_t)a[l] * (int32_t)b[l];
      dst[(size_t)i * dstr + j] = orc_dequant(s, ssc[i], matsc[j]);
    }
  }
  return 0;
}

/* Per-output-row weight quantizer of the exporter, model.py:151-161
 * (Linear.quantize, called by export.py:430-457 on the transposed weight, so
 * each gemma.c row n gets one scale) and model.py:97-107 (Embedding.quantize,
 * lm_head).  fp32 throughout: s = max(amax, 1e-8) / 127 (IEEE division),
 * q = round-half-to-even(w / s) (torch.round), clamp to [-127, 127]. */
void orc_quantize_weight_rows(int8_t *q, float *scales, const float *w, int n,
                              int k) {
  for (int j = 0; j < n; j++) {
    const float *row = w + (size_t)j * k;
    float amax = 0.0f;
    for (int l = 0; l < k; l++) {
      float a = fabsf(row[l]);
      amax = a > amax ? a : amax;
    }
    if (amax < 1e-8f)
      amax = 1e-8f;
    float s = amax / 127.0f;
    scales[j] = s;
    for (int l = 0; l < k; l++) {
      float r = nearbyintf(row[l] / s); /* default mode: half to even */
      if (r > 127.0f)
        r = 127.0f;
      if (r < -127.0f)
        r = -127.0f;
      q[(size_t)j * k + l] = (int8_t)r;
    }
  }
}

/* gemma-style RMSNorm of each row followed by quantize_act, the pair gemma.c
 * runs on every block input: rmsnorm (gemma.c:2509-2524) at 4754 / 5026,
 * then quantize_act / quantize_acts at 4768 / 5034.  Sequential fp32 sum of
 * squares (the reference's -ffast-math build vectorizes it, so its last bits
 * may differ), rms = 1 / sqrtf(sum / dim + eps), xn = (x * rms) * (w + 1).
 * xn (optional) receives the normalized rows, q / s the codes and scales. */
void orc_rmsnorm_quantize(int8_t *q, float *s, float *xn, const float *x, const float *w,
                          float eps, int m, int dim) {
  for (int i = 0; i < m; i++) {
    const float *row = x + (size_t)i * dim;
    float sq = 0.0f;
    for (int d = 0; d < dim; d++)
      sq += row[d] * row[d];
    const float rms = 1.0f / sqrtf(sq / (float)dim + eps);
    float tmp[16384];
    for (int d = 0; d < dim; d++)
      tmp[d] = row[d] * rms * (w[d] + 1.0f);
    if (xn)
      memcpy(xn + (size_t)i * dim, tmp, (size_t)dim * sizeof(float));
    s[i] = orc_quantize_act(q + (size_t)i * dim, tmp, dim);
  }
}

/* GeGLU gate followed by quantize_act: h = gelu_tanh(gate) * up
 * (gemma.c:4139-4170, gelu with `mul`, called at 4921 / 5379), then
 * quantize_act / quantize_acts on h (the down projection's input).
 * gelu_tanh(x) = 0.5 x (1 + tanhf(sqrt(2/pi) (x + 0.044715 x^3))) in the
 * reference's operation order; tanhf is this C library's. */
void orc_geglu_quantize(int8_t *q, float *s, float *h, const float *gate, const float *up,
                        int m, int dim) {
  const float c = 0.79788456080287f;
  for (int i = 0; i < m; i++) {
    float tmp[16384];
    for (int d = 0; d < dim; d++) {
      const float x = gate[(size_t)i * dim + d];
      const float g = 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x * x * x)));
      tmp[d] = g * up[(size_t)i * dim + d];
    }
    if (h)
      memcpy(h + (size_t)i * dim, tmp, (size_t)dim * sizeof(float));
    s[i] = orc_quantize_act(q + (size_t)i * dim, tmp, dim);
  }
}

/* ---- attention (fp32), the layer around the matmuls ------------------------
 * gemma.c keeps attention in fp32 ("typically people don't quantize this",
 * gemma.c:5221).  These restate its two forms with plain loops; the reference
 * vectorizes its dot products under -ffast-math, so agreement is to within
 * fp32 reassociation, not bit for bit. */

/* gemma.c:4066-4089 fast_expf: cephes-style exp, 0 below -87.33654. */
static float orc_fast_expf(float x) {
  float xl = x < -87.33654f ? -87.33654f : x;
  xl = xl > 88.0f ? 88.0f : xl;
  float fx = floorf(xl * 1.44269504088896341f + 0.5f);
  float r = xl - fx * 0.693359375f;
  r -= fx * -2.12194440e-4f;
  float z = r * r;
  float y = 1.9875691500e-4f;
  y = y * r + 1.3981999507e-3f;
  y = y * r + 8.3334519073e-3f;
  y = y * r + 4.1665795894e-2f;
  y = y * r + 1.6666665459e-1f;
  y = y * r + 5.0000001201e-1f;
  y = y * z + r + 1.0f;
  union {
    int i;
    float f;
  } u;
  u.i = ((int)fx + 127) << 23;
  y *= u.f;
  return x < -87.33654f ? 0.0f : y;
}

/* gemma.c:4091-4112 softmax of one row in place. */
static void orc_softmax(float *row, int n) {
  float max = -3.402823466e38f;
  for (int i = 0; i < n; i++) max = row[i] > max ? row[i] : max;
  float sum = 0.0f;
  for (int i = 0; i < n; i++) {
    row[i] = orc_fast_expf(row[i] - max);
    sum += row[i];
  }
  for (int i = 0; i < n; i++) row[i] = row[i] / sum;
}

/* the optional tanh softcap, gemma.c:4124-4129 / 5245-5250 */
static void orc_softcap(float *row, int n, float sc) {
  if (sc == 0.0f) return;
  for (int i = 0; i < n; i++) row[i] = tanhf(row[i] / sc) * sc;
}

static float orc_dot(const float *a, const float *b, int n) {
  float s = 0.0f;
  for (int i = 0; i < n; i++) s += a[i] * b[i];
  return s;
}

/* One decode step's attention for one layer, gemma.c:4836-4848:
 * att_scores_gqa (2868-2896), att_finalize per head (4117-4133),
 * att_values_gqa (2902-2985).  Query head h reads kv head hk when
 * gqa_head_of(hk) <= h < gqa_head_of(hk+1), gqa_head_of(hk) =
 * (hk*n_heads + nkv - 1) / nkv (gemma.c:2861-2863).  Head hk's cache row t
 * is at cache + hk*kv_stride + t*hdim; the window is [spos, spos+attlen).
 * att: scratch of n_heads*attlen floats. */
void orc_attention_decode(float *xo, const float *xq, const float *kc, const float *vc,
                          long kv_stride, int n_heads, int nkv, int hdim, int spos, int attlen,
                          float asc, float sc_att, float *att) {
  for (int hk = 0; hk < nkv; hk++) {
    const int h0 = (hk * n_heads + nkv - 1) / nkv;
    const int h1 = ((hk + 1) * n_heads + nkv - 1) / nkv;
    const float *kh = kc + (size_t)hk * kv_stride + (size_t)spos * hdim;
    const float *vh = vc + (size_t)hk * kv_stride + (size_t)spos * hdim;
    for (int h = h0; h < h1; h++) {
      float *a = att + (size_t)h * attlen;
      for (int t = 0; t < attlen; t++) a[t] = orc_dot(kh + (size_t)t * hdim, xq + (size_t)h * hdim, hdim);
      for (int t = 0; t < attlen; t++) a[t] *= asc;
      orc_softcap(a, attlen, sc_att);
      orc_softmax(a, attlen);
      for (int d = 0; d < hdim; d++) {
        float acc = 0.0f;
        for (int t = 0; t < attlen; t++) acc += a[t] * vh[(size_t)t * hdim + d];
        xo[(size_t)h * hdim + d] = acc;
      }
    }
  }
}

/* A prefill chunk's attention for one layer, gemma.c:5160-5295.  xq
 * [n_heads][ntok][hdim] is already rotated and scaled by the attention
 * scale (gemma.c:5121-5133); this chunk's keys and values are in the cache at
 * [spos, spos+ntok).  Query head h reads kv head h*nkv/n_heads (gemma.c:5172).
 * mask != 0 (the blockwise-causal path): token i (position spos+i) attends to
 * [spos_i, spos+i], spos_i = spos+i+1-slide when the layer slides (slide > 0)
 * and spos+i >= slide, else 0.  mask == 0 (the dense path): every token
 * attends to [0, spos+ntok).  The softcap is applied to the scores that enter
 * the softmax.  Token i's output row is xo + i*xostr + h*hdim.  att: scratch
 * of spos+ntok floats. */
void orc_attention_prefill(float *xo, int xostr, const float *xq, const float *kc, const float *vc,
                           long kv_stride, int n_heads, int nkv, int hdim, int spos, int ntok,
                           int slide, float sc_att, int mask, float *att) {
  for (int h = 0; h < n_heads; h++) {
    const int hk = h * nkv / n_heads;
    const float *kh = kc + (size_t)hk * kv_stride;
    const float *vh = vc + (size_t)hk * kv_stride;
    for (int i = 0; i < ntok; i++) {
      const int pos = spos + i;
      int t0 = 0, t1 = spos + ntok - 1;
      if (mask) {
        t0 = (slide > 0 && pos >= slide) ? pos + 1 - slide : 0;
        t1 = pos;
      }
      const int n = t1 - t0 + 1;
      const float *q = xq + ((size_t)h * ntok + i) * hdim;
      for (int t = 0; t < n; t++) att[t] = orc_dot(q, kh + (size_t)(t0 + t) * hdim, hdim);
      orc_softcap(att, n, sc_att);
      orc_softmax(att, n);
      float *o = xo + (size_t)i * xostr + (size_t)h * hdim;
      for (int d = 0; d < hdim; d++) {
        float acc = 0.0f;
        for (int t = 0; t < n; t++) acc += att[t] * vh[(size_t)(t0 + t) * hdim + d];
        o[d] = acc;
      }
    }
  }
}

/* ---- SigLIP head: patch embedding, pooling --------------------------------- */

static float orc_clamp(float v) { /* clamp_fpx for floatx = float, gemma.c:2504-2506 */
  const float m = 3.402823466e38f;
  return v > m ? m : (v < -m ? -m : v);
}

/* gemma.c:4411-4466: Conv2d(3, dim, kernel = stride = psize, bias) over the
 * (img_px, img_px, 3) image, one row of x per patch (row-major patches), then
 * the dequantized int8 position embedding added per element.
 *   x[p][oc] = clamp(sum_{py,px,c} pe[oc][c][py][px] * img[oy*P+py][ox*P+px][c] + pe_b[oc])
 *   x[p][oc] = clamp(x[p][oc] + (float)pos_q[p][oc] * pos_s[p]) */
void orc_patch_embed(float *x, const float *img, const float *pe, const float *pe_b, const int8_t *pos_q,
                     const float *pos_s, int img_px, int psize, int dim) {
  const int ppi = img_px / psize, idim = 3 * psize * psize;
  for (int pi = 0; pi < ppi * ppi; pi++) {
    const int oy = pi / ppi, ox = pi - oy * ppi;
    for (int oc = 0; oc < dim; oc++) {
      float sum = 0.0f;
      for (int py = 0; py < psize; py++)
        for (int px = 0; px < psize; px++)
          for (int c = 0; c < 3; c++)
            sum += pe[(size_t)oc * idim + c * psize * psize + py * psize + px] *
                   img[((size_t)(oy * psize + py) * img_px + (ox * psize + px)) * 3 + c];
      float v = orc_clamp(sum + pe_b[oc]);
      v = orc_clamp(v + (float)pos_q[(size_t)pi * dim + oc] * pos_s[pi]);
      x[(size_t)pi * dim + oc] = v;
    }
  }
}

/* gemma.c:4660-4705, 4714: LayerNorm of every patch row (weight post_n, bias
 * post_nb, gemma.c:2526-2551), average pooling of ksize x ksize patches
 * (ksize = ppi / side) in (ky, kx) order, gemma-style RMSNorm (norm,
 * gemma.c:2509-2523), then quantize_acts of the pooled rows.  out (optional)
 * [side*side][dim]; q [side*side][dim], s [side*side]. */
void orc_vision_pool(int8_t *q, float *s, float *out, const float *x, const float *post_n,
                     const float *post_nb, const float *norm, float eps, int ppi, int side, int dim,
                     float *scratch /* dim floats */) {
  const int ks = ppi / side;
  for (int oy = 0; oy < side; oy++) {
    for (int ox = 0; ox < side; ox++) {
      float *acc = scratch;
      for (int d = 0; d < dim; d++) acc[d] = 0.0f;
      for (int ky = 0; ky < ks; ky++) {
        for (int kx = 0; kx < ks; kx++) {
          const float *row = x + ((size_t)(oy * ks + ky) * ppi + (ox * ks + kx)) * dim;
          float mean = 0.0f;
          for (int d = 0; d < dim; d++) mean += row[d];
          mean /= (float)dim;
          float var = 0.0f;
          for (int d = 0; d < dim; d++) {
            const float df = row[d] - mean;
            var += df * df;
          }
          var /= (float)dim;
          const float inv_std = 1.0f / sqrtf(var + eps);
          for (int d = 0; d < dim; d++) acc[d] += (row[d] - mean) * inv_std * post_n[d] + post_nb[d];
        }
      }
      const int o = oy * side + ox;
      float sq = 0.0f;
      for (int d = 0; d < dim; d++) {
        acc[d] = acc[d] / (float)(ks * ks);
        sq += acc[d] * acc[d];
      }
      const float rms = 1.0f / sqrtf(sq / (float)dim + eps);
      for (int d = 0; d < dim; d++) acc[d] = acc[d] * rms * (norm[d] + 1.0f);
      if (out) memcpy(out + (size_t)o * dim, acc, (size_t)dim * sizeof(float));
      s[o] = orc_quantize_act(q + (size_t)o * dim, acc, dim);
    }
  }
}

/* ---- between the Q/K/V matmuls and attention ------------------------------- */

/* gemma.c:2509-2523 rmsnorm of one row in place: x * rms * (w + 1). */
static void orc_rmsnorm_row(float *x, const float *w, int n, float eps) {
  float sq = 0.0f;
  for (int i = 0; i < n; i++) sq += x[i] * x[i];
  const float rms = 1.0f / sqrtf(sq / (float)n + eps);
  for (int i = 0; i < n; i++) x[i] = x[i] * rms * (w[i] + 1.0f);
}

/* gemma.c:4223-4245 rope_apply on one vector: pairs (d, d + hdim/2) rotated
 * by the table's (cos, sin) for d, times scale. */
static void orc_rope_row(float *x, const float *fr, int hdim, float scale) {
  for (int d = 0; d < hdim / 2; d++) {
    const float c = fr[2 * d], s = fr[2 * d + 1];
    const float a = x[d], b = x[d + hdim / 2];
    x[d] = (a * c - b * s) * scale;
    x[d + hdim / 2] = (a * s + b * c) * scale;
  }
}

/* QK RMSNorm (when nq / nk are given), RoPE (q scaled by q_scale) and the
 * K/V cache writes of a chunk of ntok tokens at [spos, spos+ntok), as
 * gemma.c:4775-4818 (decode) and 5095-5145 (prefill) run them.  xq
 * [n_heads][ntok][hdim] rotated in place; xk [nkv][ntok][hdim] normed and
 * rotated in place (then copied to the cache); freqs [ntok][hdim]. */
void orc_qk_norm_rope_cache(float *xq, float *xk, const float *xv, float *kc, float *vc, long kv_stride,
                            const float *nq, const float *nk, float eps, const float *freqs, float q_scale,
                            int n_heads, int nkv, int hdim, int spos, int ntok) {
  for (int h = 0; h < n_heads; h++)
    for (int t = 0; t < ntok; t++) {
      float *row = xq + ((size_t)h * ntok + t) * hdim;
      if (nq) orc_rmsnorm_row(row, nq, hdim, eps);
      orc_rope_row(row, freqs + (size_t)t * hdim, hdim, q_scale);
    }
  for (int h = 0; h < nkv; h++)
    for (int t = 0; t < ntok; t++) {
      float *row = xk + ((size_t)h * ntok + t) * hdim;
      if (nk) orc_rmsnorm_row(row, nk, hdim, eps);
      orc_rope_row(row, freqs + (size_t)t * hdim, hdim, 1.0f);
      memcpy(kc + (size_t)h * kv_stride + (size_t)(spos + t) * hdim, row, (size_t)hdim * sizeof(float));
      memcpy(vc + (size_t)h * kv_stride + (size_t)(spos + t) * hdim, xv + ((size_t)h * ntok + t) * hdim,
             (size_t)hdim * sizeof(float));
    }
}
