/*
 * gemma_gcu_model.h -- the model hooks of the CUDA drop-in for gemma.c.
 *
 * Included by gemma.c (under GEMMA_CUDA) right after the GemmaModel type
 * (gemma.c:1882-1890), so it sees QTensor (gemma.c:1102), TextConfig
 * (gemma.c:740-761), VisionConfig (gemma.c:713-721), TextDecoderLayer
 * (gemma.c:1174-1195), VisionEncoderLayer (gemma.c:1234-1256), TextDecoder
 * (gemma.c:1295-1300), VisionEncoder (gemma.c:1572-1585) and log_error
 * (gemma.c:579).  Two hooks:
 *
 *   gcu_setup_gemma_model    called by setup_gemma_model (gemma.c:6867) once
 *                            the model is read or mapped: every matmul
 *                            QTensor goes to the GPU as ONE device arena
 *                            (gcu_register_model on the mmap of the -m path,
 *                            gcu_register_qtensors on the per-tensor buffers
 *                            read_gemma_model made)
 *   gcu_release_gemma_model  called by cleanup_gemma_model (gemma.c:6909)
 *                            before the host copies go away
 *
 * Registration is a performance step: an unregistered weight is uploaded for
 * each call that uses it.  Both hooks return 0 / 1 and report through
 * log_error, like the loader they sit in.
 */
#ifndef GEMMA_GCU_MODEL_H
#define GEMMA_GCU_MODEL_H

#include "gcu.h"

static int g_gcu_arena = -1; /* the registered model's arena, -1 for none */

static int gcu_put_qtensor(gcu_qtensor *list, int n, const QTensor *t, int rows, int k, int kind,
                           int layer) {
  list[n].q = t->i8.q;
  list[n].scales = (const float *)t->i8.scales;
  list[n].rows = rows;
  list[n].k = k;
  list[n].kind = kind;
  list[n].layer = layer;
  return n + 1;
}

/* The matmul QTensors of a model whose tensors read_gemma_model placed in
 * their own buffers, in file order (gemma.c:1470-1560, 1765-1875). */
static int gcu_list_model_qtensors(const GemmaModel *model, gcu_qtensor **out) {
  const TextDecoder *dec = model->decoder;
  const TextConfig *tc = dec->config;
  const VisionEncoder *enc = model->encoder;
  const int q_sz = tc->n_heads * tc->hdim, kv_sz = tc->nkv * tc->hdim;
  int cap = 1 + 7 * tc->nl;
  if (enc != NULL) cap += 6 * enc->config->nl + 1;
  gcu_qtensor *list = (gcu_qtensor *)malloc((size_t)cap * sizeof(gcu_qtensor));
  if (list == NULL) return -1;
  int n = gcu_put_qtensor(list, 0, dec->emb, (int)tc->nvocab, tc->dim, GCU_QT_LM_HEAD, -1);
  for (int l = 0; l < tc->nl; l++) {
    const TextDecoderLayer *L = dec->layers[l];
    n = gcu_put_qtensor(list, n, L->wq, q_sz, tc->dim, GCU_QT_WQ, l);
    n = gcu_put_qtensor(list, n, L->wk, kv_sz, tc->dim, GCU_QT_WK, l);
    n = gcu_put_qtensor(list, n, L->wv, kv_sz, tc->dim, GCU_QT_WV, l);
    n = gcu_put_qtensor(list, n, L->wo, tc->dim, q_sz, GCU_QT_WO, l);
    n = gcu_put_qtensor(list, n, L->w1, tc->mlp_dim, tc->dim, GCU_QT_W1, l);
    n = gcu_put_qtensor(list, n, L->w2, tc->mlp_dim, tc->dim, GCU_QT_W2, l);
    n = gcu_put_qtensor(list, n, L->w3, tc->dim, tc->mlp_dim, GCU_QT_W3, l);
  }
  if (enc != NULL) {
    const VisionConfig *vc = enc->config;
    for (int l = 0; l < vc->nl; l++) {
      const VisionEncoderLayer *L = enc->layers[l];
      n = gcu_put_qtensor(list, n, L->wq, vc->dim, vc->dim, GCU_QT_VWQ, l);
      n = gcu_put_qtensor(list, n, L->wk, vc->dim, vc->dim, GCU_QT_VWK, l);
      n = gcu_put_qtensor(list, n, L->wv, vc->dim, vc->dim, GCU_QT_VWV, l);
      n = gcu_put_qtensor(list, n, L->wo, vc->dim, vc->dim, GCU_QT_VWO, l);
      n = gcu_put_qtensor(list, n, L->w1, vc->mlp_dim, vc->dim, GCU_QT_VW1, l);
      n = gcu_put_qtensor(list, n, L->w2, vc->dim, vc->mlp_dim, GCU_QT_VW2, l);
    }
    n = gcu_put_qtensor(list, n, enc->proj, tc->dim, vc->dim, GCU_QT_VPROJ, -1);
  }
  *out = list;
  return n;
}

/* setup_gemma_model hook (gemma.c:6867), after the read or mmap succeeded. */
static int gcu_setup_gemma_model(const GemmaModel *model, bool allow_mm) {
  if (!model->quant) return 0; /* only the W8A8 path runs on the GPU */
  int rc;
  if (model->mm_data != NULL) {
    rc = gcu_register_model(model->mm_data, model->mm_sz, allow_mm, &g_gcu_arena);
  } else {
    gcu_qtensor *list = NULL;
    const int n = gcu_list_model_qtensors(model, &list);
    if (n < 0) {
      log_error("cuda register: out of host memory");
      return 1;
    }
    rc = gcu_register_qtensors(list, n, &g_gcu_arena);
    free(list);
  }
  if (rc) {
    log_error("cuda register: %s", gcu_last_error());
    g_gcu_arena = -1;
  }
  return rc;
}

/* cleanup_gemma_model hook (gemma.c:6909): drop the arena before the host
 * tensors it mirrors are freed or unmapped. */
static void gcu_release_gemma_model(void) {
  if (g_gcu_arena >= 0 && gcu_unregister_arena(g_gcu_arena))
    log_error("cuda unregister: %s", gcu_last_error());
  g_gcu_arena = -1;
}

#endif /* GEMMA_GCU_MODEL_H */
