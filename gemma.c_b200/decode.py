"""decode.py -- device-resident W8A8 decode steps and prefill chunks through libgcu.so.

`Decoder.step` runs gemma.c's forward_text_decode (gemma.c:4727-4978) for one
token with every activation, weight and the KV cache in GPU memory, one C-ABI
call per step of the reference:

    per layer (gemma.c:4750-4962)
      rmsnorm(x, n1) + quantize_act            gcu_dev_rmsnorm_quantize (first layer)
      q, k, v = gemv_int8_multi                gcu_dev_gemv_int8_multi
      QK norm, RoPE, KV-cache write            gcu_dev_qk_norm_rope_cache
      attention (scores, softmax, values)      gcu_dev_attention_decode
      quantize_act(xo) + gemv_int8(wo)         gcu_dev_quantize_gemm_int8_multi
      x = clamp(resid + rmsnorm(o, n2)),
        rmsnorm(x, n3) + quantize_act          gcu_dev_residual_norm_quantize
      gate, up = gemv_int8_multi               gcu_dev_gemv_int8_multi
      gelu(gate) * up + quantize_act           gcu_dev_geglu_quantize
      down = gemv_int8(w3)                     gcu_dev_gemv_int8
      x = clamp(resid + rmsnorm(down, n4)),
        next layer's rmsnorm(x, n1) + quantize gcu_dev_residual_norm_quantize
                                               (last layer: gcu_dev_rmsnorm_residual)
    final rmsnorm + quantize_act, lm_head gemv_int8, logit softcap

`Decoder.prefill` runs gemma.c's forward_text_chunk (gemma.c:4985-5455) for
a chunk of tokens the same way, with one GEMM over wq|wk|wv (the values of
gemma.c's per-head GEMMs), the tensor-core GEMMs for the projections, and
the causal attention kernel.

Weights follow gemma.c's TextDecoder (gemma.c:1174-1301); torch only holds
the device memory and the stream.  The RoPE tables are computed on the host
per position as rope_freqs does (gemma.c:4178-4216) unless the caller passes
its own.
"""
from __future__ import annotations

import numpy as np

import gcu


def rope_tables(hdim: int, theta_l: float, theta_g: float, pos: int):
    """gemma.c:4178-4193 in float32: (cos, sin) interleaved per frequency, for
    sliding-window and full-attention layers."""
    d = np.arange(hdim // 2, dtype=np.float32)
    e = (np.float32(-2.0) * d) / np.float32(hdim)
    out = []
    for theta in (theta_l, theta_g):
        freq = np.power(np.float32(theta), e, dtype=np.float32)
        ang = (freq * np.float32(pos)).astype(np.float32)
        t = np.empty(hdim, np.float32)
        t[0::2] = np.cos(ang)
        t[1::2] = np.sin(ang)
        out.append(t)
    return out[0], out[1]


class Decoder:
    """A W8A8 Gemma text decoder resident on one GPU.

    cfg: nl, n_heads, nkv, hdim, dim, mlp_dim, nvocab, q_scale, slide, swa
    (per-layer sliding flags), qk_norm, mlp_pre, mlp_pst, theta_l, theta_g,
    eps, sc_att, sc_log.  layers: per layer a dict of (q, scales) numpy pairs
    wq, wk, wv, wo, w1 (up), w2 (gate), w3 (down) and norm vectors n1..n4, nq,
    nk.  emb: the tied embedding (q, scales) used as lm_head; fnorm: the final
    norm.  clen: KV-cache positions."""

    def __init__(self, cfg: dict, layers: list, emb, fnorm, clen: int, device="cuda"):
        import torch
        self.torch = torch
        self.cfg = cfg
        self.dev = device
        self.clen = clen
        c = cfg
        t = lambda a: a.to(device).contiguous() if torch.is_tensor(a) else torch.from_numpy(np.ascontiguousarray(a)).to(device)
        self.L = []
        for lay in layers:
            d = {k: (t(lay[k][0]), t(lay[k][1])) for k in ("wq", "wk", "wv", "wo", "w1", "w2", "w3")}
            for k in ("n1", "n2", "n3", "n4", "nq", "nk"):
                d[k] = t(lay[k]) if lay.get(k) is not None else None
            self.L.append(d)
        self.emb = (t(emb[0]), t(emb[1]))
        self.fnorm = t(fnorm)
        q_sz = c["n_heads"] * c["hdim"]
        f32 = dict(dtype=torch.float32, device=device)
        i8 = dict(dtype=torch.int8, device=device)
        self.kv = torch.zeros((c["nl"], 2, c["nkv"], clen, c["hdim"]), **f32)
        self.x = torch.empty((1, c["dim"]), **f32)
        self.x2 = torch.empty((1, c["dim"]), **f32)  # the residual stream alternates between x and x2
        self.out = torch.empty((1, c["dim"]), **f32)
        self.xq = torch.empty((c["n_heads"], 1, c["hdim"]), **f32)
        self.xk = torch.empty((c["nkv"], 1, c["hdim"]), **f32)
        self.xv = torch.empty((c["nkv"], 1, c["hdim"]), **f32)
        self.xo = torch.empty((1, q_sz), **f32)
        self.xg = torch.empty((1, c["mlp_dim"]), **f32)
        self.xu = torch.empty((1, c["mlp_dim"]), **f32)
        self.q = torch.empty((1, max(c["dim"], q_sz, c["mlp_dim"])), **i8)
        self.s = torch.empty(1, **f32)
        self.logits = torch.empty((1, c["nvocab"]), **f32)
        self.freqs = torch.empty((2, c["hdim"]), **f32)  # sliding, full

    def set_freqs(self, slid, full, stream=None):
        """Upload the RoPE tables of the position about to be decoded."""
        torch = self.torch
        host = torch.from_numpy(np.stack([np.asarray(slid, np.float32), np.asarray(full, np.float32)]))
        with torch.cuda.stream(stream) if stream is not None else _null():
            self.freqs.copy_(host, non_blocking=False)

    def step(self, pos: int, stream=None):
        """Decode position `pos` from the embedding already in self.x (dim,);
        leaves the logits in self.logits and the final hidden state in self.x.
        The RoPE tables for `pos` must be set (set_freqs) beforehand."""
        c = self.cfg
        dim, mlp, hdim = c["dim"], c["mlp_dim"], c["hdim"]
        nh, nkv = c["n_heads"], c["nkv"]
        q_sz = nh * hdim
        asc = float(np.float32(1.0) / np.sqrt(np.float32(c["q_scale"])))
        eps = c["eps"]
        q = self.q
        nl = len(self.L)
        # gemma.c:4750-4768: the first layer's rmsnorm(x, n1) -> quantize_act
        # (every later layer's runs in front of its Q/K/V projection, in the
        # launch that also adds the previous layer's FFN output to the residual)
        gcu.dev_rmsnorm_quantize(q, self.s, self.x, self.L[0]["n1"], eps, 1, dim, stream=stream)
        # The residual stream alternates between x and x2: a launch whose CTAs
        # all read the residual writes the updated one to the other buffer.
        xa, xb = self.x, self.x2
        qkv = lambda w: [(w["wq"][0], w["wq"][1], self.xq), (w["wk"][0], w["wk"][1], self.xk),
                         (w["wv"][0], w["wv"][1], self.xv)]
        gcu.dev_gemv_int8_multi(qkv(self.L[0]), q, self.s, dim, stream=stream)  # gemma.c:4769-4773
        for l, w in enumerate(self.L):
            # gemma.c:4775-4848: QK norm, RoPE and the cache write of position
            # pos, then attention over [spos, pos] -- one launch
            kc, vc = self.kv[l, 0], self.kv[l, 1]
            sliding = bool(c["swa"][l])
            spos = pos + 1 - c["slide"] if sliding and pos >= c["slide"] else 0
            gcu.dev_attention_decode_rope(self.xo.view(nh, hdim), self.xq.view(nh, hdim), self.xk.view(nkv, hdim),
                                          self.xv.view(nkv, hdim), kc, vc, self.freqs[0 if sliding else 1], spos,
                                          pos + 1 - spos, asc, c["sc_att"],
                                          nq=w["nq"] if c["qk_norm"] else None,
                                          nk=w["nk"] if c["qk_norm"] else None, eps=eps, stream=stream)
            # gemma.c:4855-4860: O projection (quantize_act of the attention
            # output in the same launch)
            gcu.dev_quantize_gemm_int8_multi([(w["wo"][0], w["wo"][1], self.out)], q, self.s, self.xo, 1, q_sz,
                                             stream=stream)
            # gemma.c:4862-4915: post-attention norm + residual, pre-FFN norm +
            # quantize, and the gate/up projections -- one launch
            gcu.dev_residual_norm_quantize_gemv_multi(
                [(w["w2"][0], w["w2"][1], self.xg), (w["w1"][0], w["w1"][1], self.xu)], xb, q, self.s, self.out, xa,
                w["n2"] if c["mlp_pre"] else None, w["n3"] if c["mlp_pre"] else w["n2"], eps, dim, stream=stream)
            xa, xb = xb, xa
            # gemma.c:4921-4930: GeGLU + quantize and the down projection -- one launch
            gcu.dev_geglu_quantize_gemv_multi([(w["w3"][0], w["w3"][1], self.out)], q, self.s, self.xg, self.xu,
                                              mlp, stream=stream)
            # gemma.c:4934-4962: post-FFN norm + residual, with the next layer's
            # rmsnorm(x, n1) + quantize_act and its Q/K/V projections (4754-4773)
            post = w["n4"] if c["mlp_pst"] else None
            if l + 1 < nl:
                gcu.dev_residual_norm_quantize_gemv_multi(qkv(self.L[l + 1]), xb, q, self.s, self.out, xa, post,
                                                          self.L[l + 1]["n1"], eps, dim, stream=stream)
            else:
                gcu.dev_rmsnorm_residual(xb, self.out, xa, post, eps, 1, dim, stream=stream)
            xa, xb = xb, xa
        # gemma.c:4965-4976: final norm (into x), tied lm_head, logit softcap
        gcu.dev_rmsnorm_quantize(q, self.s, xa, self.fnorm, eps, 1, dim, out=self.x, stream=stream)
        gcu.dev_gemv_int8(self.logits, self.emb[0], self.emb[1], q, self.s, c["nvocab"], dim, stream=stream)
        if c["sc_log"]:
            gcu.dev_softcap(self.logits, c["sc_log"], stream=stream)

    # ---- prefill ---------------------------------------------------------------
    def _prefill_buffers(self, nmax: int):
        torch = self.torch
        c = self.cfg
        if getattr(self, "_pmax", 0) >= nmax:
            return
        self._pmax = nmax
        dim, mlp, hd = c["dim"], c["mlp_dim"], c["hdim"]
        q_sz, kv_sz = c["n_heads"] * hd, c["nkv"] * hd
        f32 = dict(dtype=torch.float32, device=self.dev)
        i8 = dict(dtype=torch.int8, device=self.dev)
        self.px = torch.empty((nmax, dim), **f32)           # residual stream, one row per token
        self.pqkv = torch.empty((nmax, q_sz + 2 * kv_sz), **f32)
        self.pxq = torch.empty(c["n_heads"] * nmax * hd, **f32)
        self.pxo = torch.empty((nmax, q_sz), **f32)
        self.pout = torch.empty((nmax, dim), **f32)
        self.pxg = torch.empty((nmax, mlp), **f32)
        self.pxu = torch.empty((nmax, mlp), **f32)
        self.pq_dim = torch.empty((nmax, dim), **i8)
        self.pq_qsz = torch.empty((nmax, q_sz), **i8)
        self.pq_mlp = torch.empty((nmax, mlp), **i8)
        self.ps = torch.empty(nmax, **f32)
        self.pfreq = torch.empty((2, nmax, hd), **f32)        # sliding, full
        if not hasattr(self, "wqkv"):
            # one GEMM over wq|wk|wv: the same values as gemma.c's per-head GEMMs
            self.wqkv = [(torch.cat([w["wq"][0], w["wk"][0], w["wv"][0]]).contiguous(),
                          torch.cat([w["wq"][1], w["wk"][1], w["wv"][1]]).contiguous()) for w in self.L]

    def set_prefill_freqs(self, slid, full):
        """Upload the RoPE tables (ntok, hdim) of the chunk about to be prefilled."""
        torch = self.torch
        n = len(slid)
        self._prefill_buffers(n)
        self.pfreq[0, :n].copy_(torch.from_numpy(np.ascontiguousarray(slid, np.float32)))
        self.pfreq[1, :n].copy_(torch.from_numpy(np.ascontiguousarray(full, np.float32)))

    def prefill(self, spos: int, ntok: int, stream=None):
        """gemma.c's forward_text_chunk (gemma.c:4985-5455) for the ntok input
        embeddings in self.px[:ntok] at positions spos .. spos+ntok-1 (causal):
        every layer, the final norm of every row (left in self.px) and the
        last token's logits (self.logits).  set_prefill_freqs first."""
        c = self.cfg
        if not 0 < ntok <= getattr(self, "_pmax", 0):
            # the chunk's embeddings and RoPE tables live in buffers that
            # set_prefill_freqs sized; growing them here would drop both
            raise ValueError(f"prefill of {ntok} tokens: call set_prefill_freqs with the chunk's "
                             f"{ntok} rows of tables first")
        if spos < 0 or spos + ntok > self.clen:
            raise ValueError(f"prefill of positions [{spos}, {spos + ntok}) outside a cache of {self.clen}")
        dim, mlp, hd = c["dim"], c["mlp_dim"], c["hdim"]
        nh, nkv = c["n_heads"], c["nkv"]
        q_sz, kv_sz = nh * hd, nkv * hd
        asc = float(np.float32(1.0) / np.sqrt(np.float32(c["q_scale"])))
        eps = c["eps"]
        n = ntok
        px, ps, pout = self.px[:n], self.ps[:n], self.pout[:n]
        q_dim, q_qsz, q_mlp = self.pq_dim[:n], self.pq_qsz[:n], self.pq_mlp[:n]
        xq = self.pxq[:nh * n * hd].view(nh, n, hd)
        nl = len(self.L)
        # gemma.c:5019-5034: the first layer's rmsnorm(x, n1) -> quantize_acts
        gcu.dev_rmsnorm_quantize(q_dim, ps, px, self.L[0]["n1"], eps, n, dim, stream=stream)
        for l, w in enumerate(self.L):
            # gemma.c:5036-5091: q, k, v of every token (one fused GEMM)
            gcu.dev_gemm_int8(self.pqkv[:n], self.wqkv[l][0], self.wqkv[l][1], q_dim, ps, n, q_sz + 2 * kv_sz, dim,
                              stream=stream)
            # gemma.c:5095-5145: QK norm, RoPE (queries scaled), cache write
            kc, vc = self.kv[l, 0], self.kv[l, 1]
            sliding = bool(c["swa"][l])
            gcu.dev_qkv_norm_rope_cache(xq, self.pqkv[:n], kc, vc, self.pfreq[0 if sliding else 1, :n], spos, nh,
                                        asc, w["nq"] if c["qk_norm"] else None, w["nk"] if c["qk_norm"] else None,
                                        eps, stream=stream)
            # gemma.c:5160-5295: causal attention, sliding window on local layers
            gcu.dev_attention_prefill(self.pxo[:n], xq, kc, vc, spos, c["slide"] if sliding else 0, c["sc_att"],
                                      True, stream=stream)
            # gemma.c:5296-5340: O projection, post-attention norm + residual,
            # pre-FFN norm + quantize
            gcu.dev_quantize_gemm_int8_multi([(w["wo"][0], w["wo"][1], pout)], q_qsz, ps, self.pxo[:n], n, q_sz,
                                             stream=stream)
            gcu.dev_residual_norm_quantize(px, q_dim, ps, pout, px, w["n2"] if c["mlp_pre"] else None,
                                           w["n3"] if c["mlp_pre"] else w["n2"], eps, n, dim, stream=stream)
            # gemma.c:5357-5392: gate/up, GeGLU + quantize, down
            gcu.dev_gemm_int8_multi([(w["w2"][0], w["w2"][1], self.pxg[:n]), (w["w1"][0], w["w1"][1], self.pxu[:n])],
                                    q_dim, ps, n, dim, stream=stream)
            gcu.dev_geglu_quantize(q_mlp, ps, self.pxg[:n], self.pxu[:n], n, mlp, stream=stream)
            gcu.dev_gemm_int8(pout, w["w3"][0], w["w3"][1], q_mlp, ps, n, dim, mlp, stream=stream)
            # gemma.c:5399-5418: post-FFN norm + residual (+ the next layer's input norm)
            post = w["n4"] if c["mlp_pst"] else None
            if l + 1 < nl:
                gcu.dev_residual_norm_quantize(px, q_dim, ps, pout, px, post, self.L[l + 1]["n1"], eps, n, dim,
                                               stream=stream)
            else:
                gcu.dev_rmsnorm_residual(px, pout, px, post, eps, n, dim, stream=stream)
        # gemma.c:5420-5450: final norm of every row, the last token's logits
        gcu.dev_rmsnorm_quantize(q_dim, ps, px, self.fnorm, eps, n, dim, out=px, stream=stream)
        gcu.dev_gemv_int8(self.logits, self.emb[0], self.emb[1], q_dim[n - 1:n], ps[n - 1:n], c["nvocab"], dim,
                          stream=stream)
        if c["sc_log"]:
            gcu.dev_softcap(self.logits, c["sc_log"], stream=stream)

    def launches_per_step(self, prefill: bool = False) -> int:
        """Kernel launches of one decode step (5 per layer: the residual
        updates, norms, GeGLU and quantize steps run in front of the GEMVs
        that consume them, QK norm and RoPE inside the attention kernel, plus
        the first layer's norm and Q/K/V) or one prefill chunk (11 per layer:
        the chunk merge of the attention and the separate quantize of the O
        projection's input at m > 8); an attention window split over CTAs adds
        its merge launch to the decode count."""
        if prefill:
            return 11 * self.cfg["nl"] + 3 + (1 if self.cfg["sc_log"] else 0)
        return 5 * self.cfg["nl"] + 4 + (1 if self.cfg["sc_log"] else 0)


class _null:
    def __enter__(self):
        return None

    def __exit__(self, *a):
        return False
