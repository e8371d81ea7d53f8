"""Seeded synthetic inputs and the workload shapes of the benchmark configs.

No model files or datasets exist for this path, so inputs are synthetic with
the shapes and value distributions of the Gemma-3 configs:

* weights  fp32 N(0, 0.02), quantized per output row the way the exporter
  does it (model.py:151-161 Linear.quantize via export.py:430-457):
  s = max(amax, 1e-8) / 127, q = round-half-even(w / s), clamp +-127;
* activations fp32 N(0, 1), optionally with 1% outlier channels x20.

Small tensors come from a counter-based splitmix64 -> Box-Muller generator
(seed 0x5EED0000 + tensor id), identical on every machine up to the last
float64 ulp of libm's log/cos; large benchmark tensors are drawn on the GPU
with torch's seeded generator.
"""
from __future__ import annotations

import math

import numpy as np

SEED_BASE = 0x5EED0000
_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(seed: int, count: int) -> np.ndarray:
    """The first `count` outputs of splitmix64 started at state `seed`."""
    with np.errstate(over="ignore"):
        i = np.arange(1, count + 1, dtype=np.uint64)
        z = np.uint64(seed) + i * _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def normal(tensor_id: int, shape, std: float = 1.0) -> np.ndarray:
    """fp32 N(0, std^2) of the given shape from seed SEED_BASE + tensor_id."""
    n = int(np.prod(shape))
    pairs = (n + 1) // 2
    u = splitmix64(SEED_BASE + tensor_id, 2 * pairs)
    u1 = ((u[0::2] >> np.uint64(11)).astype(np.float64) + 1.0) * (1.0 / 9007199254740992.0)
    u2 = (u[1::2] >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
    r = np.sqrt(-2.0 * np.log(u1))
    z = np.empty(2 * pairs, np.float64)
    z[0::2] = r * np.cos(2.0 * math.pi * u2)
    z[1::2] = r * np.sin(2.0 * math.pi * u2)
    return (z[:n] * std).astype(np.float32).reshape(shape)


def outlier_columns(tensor_id: int, k: int, frac: float = 0.01) -> np.ndarray:
    """ceil(frac*k) distinct seeded column indices."""
    c = int(math.ceil(frac * k))
    h = splitmix64(SEED_BASE + 0x10000 + tensor_id, k)
    return np.sort(np.argsort(h, kind="stable")[:c])


def activations(tensor_id: int, m: int, k: int, outliers: bool = False) -> np.ndarray:
    x = normal(tensor_id, (m, k), 1.0)
    if outliers:
        x[:, outlier_columns(tensor_id, k)] *= 20.0
    return x


def attention_inputs(tensor_id: int, n_heads: int, nkv: int, hdim: int, clen: int, ntok: int = 0):
    """Seeded attention operands: K and V caches (nkv, clen, hdim) of N(0, 1)
    and the queries, (n_heads, hdim) N(0, 1) for a decode step (the kernel
    applies the attention scale) or (n_heads, ntok, hdim) N(0, 1/hdim) for a
    prefill chunk (queries arrive already scaled, gemma.c:5121-5133)."""
    kc = normal(tensor_id, (nkv, clen, hdim))
    vc = normal(tensor_id + 1, (nkv, clen, hdim))
    if ntok:
        xq = normal(tensor_id + 2, (n_heads, ntok, hdim), 1.0 / math.sqrt(hdim))
    else:
        xq = normal(tensor_id + 2, (n_heads, hdim))
    return xq, kc, vc


def rope_inputs(tensor_id: int, n_heads: int, nkv: int, hdim: int, clen: int, ntok: int, qk_norm: bool):
    """Seeded operands of the QK-norm / RoPE / KV-cache step: head rows xq
    (n_heads, ntok, hdim), xk and xv (nkv, ntok, hdim) of N(0, 1), caches
    (nkv, clen, hdim), and when qk_norm the norm weights N(0, 0.1^2)."""
    xq = normal(tensor_id, (n_heads, ntok, hdim))
    xk = normal(tensor_id + 1, (nkv, ntok, hdim))
    xv = normal(tensor_id + 2, (nkv, ntok, hdim))
    kc = normal(tensor_id + 3, (nkv, clen, hdim))
    vc = normal(tensor_id + 4, (nkv, clen, hdim))
    nq = normal(tensor_id + 5, (hdim,), 0.1) if qk_norm else None
    nk = normal(tensor_id + 6, (hdim,), 0.1) if qk_norm else None
    return xq, xk, xv, kc, vc, nq, nk


def decoder_model(tensor_id: int, cfg: dict):
    """Seeded W8A8 text decoder for decode-step tests: per layer the QTensors
    wq, wk, wv, wo, w1 (up), w2 (gate), w3 (down) quantized per row like the
    exporter, norm weights N(0, 0.1^2) (n1..n4, and nq, nk of head size);
    the tied embedding (nvocab rows of dim) and the final norm."""
    dim, mlp, hd = cfg["dim"], cfg["mlp_dim"], cfg["hdim"]
    q_sz, kv_sz = cfg["n_heads"] * hd, cfg["nkv"] * hd
    layers = []
    for l in range(cfg["nl"]):
        b = tensor_id + 100 * l
        lay = {"wq": weight(b + 1, q_sz, dim), "wk": weight(b + 2, kv_sz, dim), "wv": weight(b + 3, kv_sz, dim),
               "wo": weight(b + 4, dim, q_sz), "w1": weight(b + 5, mlp, dim), "w2": weight(b + 6, mlp, dim),
               "w3": weight(b + 7, dim, mlp)}
        for i, k in enumerate(("n1", "n2", "n3", "n4")):
            lay[k] = normal(b + 10 + i, (dim,), 0.1)
        lay["nq"] = normal(b + 20, (hd,), 0.1)
        lay["nk"] = normal(b + 21, (hd,), 0.1)
        layers.append(lay)
    emb = weight(tensor_id + 90, cfg["nvocab"], dim)
    fnorm = normal(tensor_id + 91, (dim,), 0.1)
    return layers, emb, fnorm


def vision_head_inputs(tensor_id: int, img_px: int, psize: int, dim: int, img_tok: int, tdim: int):
    """Seeded operands of the SigLIP head (gemma.c:4411-4716): an
    (img_px, img_px, 3) image of N(0, 0.5^2) pixels, patch-embedding weights
    pe (dim, 3, psize, psize) and bias of N(0, 0.02^2), the int8 position
    embedding (npatch rows of dim) and projection (tdim rows of dim)
    quantized per row as the exporter does, LayerNorm weight 1 + N(0, 0.1^2)
    and bias N(0, 0.1^2), RMSNorm weight N(0, 0.1^2)."""
    ppi = img_px // psize
    pos_q, pos_s = weight(tensor_id + 3, ppi * ppi, dim)
    proj_q, proj_s = weight(tensor_id + 4, tdim, dim)
    return {"img_px": img_px, "psize": psize, "dim": dim, "img_tok": img_tok, "tdim": tdim, "eps": 1e-6,
            "img": normal(tensor_id, (img_px, img_px, 3), 0.5),
            "pe": normal(tensor_id + 1, (dim, 3, psize, psize), 0.02),
            "pe_b": normal(tensor_id + 2, (dim,), 0.02),
            "pos_q": pos_q, "pos_s": pos_s, "proj_q": proj_q, "proj_s": proj_s,
            "post_n": 1.0 + normal(tensor_id + 5, (dim,), 0.1),
            "post_nb": normal(tensor_id + 6, (dim,), 0.1),
            "norm": normal(tensor_id + 7, (dim,), 0.1)}


def quantize_weight_rows(w: np.ndarray):
    """Exporter quantizer (model.py:151-161) in numpy fp32 arithmetic."""
    w = np.asarray(w, np.float32)
    amax = np.maximum(np.abs(w).max(axis=1), np.float32(1e-8)).astype(np.float32)
    s = (amax / np.float32(127.0)).astype(np.float32)
    q = np.clip(np.rint(w / s[:, None]), -127, 127).astype(np.int8)
    return q, s


def weight(tensor_id: int, rows: int, k: int, std: float = 0.02):
    """Seeded N(0, std) weight quantized per row -> (int8 [rows][k], fp32 [rows])."""
    return quantize_weight_rows(normal(tensor_id, (rows, k), std))


# --------------------------------------------------------------------------
# GPU generation for the large benchmark tensors (torch is the allocator)
# --------------------------------------------------------------------------

def weight_torch(rows: int, k: int, gen, device, std: float = 0.02, chunk_rows: int = 16384):
    """Same quantizer on the GPU, row chunk by row chunk (bounded temporaries)."""
    import torch
    q = torch.empty((rows, k), dtype=torch.int8, device=device)
    s = torch.empty((rows,), dtype=torch.float32, device=device)
    for r0 in range(0, rows, chunk_rows):
        r1 = min(rows, r0 + chunk_rows)
        w = torch.randn((r1 - r0, k), generator=gen, device=device, dtype=torch.float32) * std
        amax = w.abs().amax(1, keepdim=True).clamp_min(1e-8)
        sc = amax / 127.0
        q[r0:r1] = torch.round(w / sc).clamp(-127, 127).to(torch.int8)
        s[r0:r1] = sc.squeeze(1)
        del w
    return q, s


def activations_torch(m: int, k: int, gen, device, outliers: bool = False, cols=None):
    import torch
    x = torch.randn((m, k), generator=gen, device=device, dtype=torch.float32)
    if outliers:
        if cols is None:
            c = int(math.ceil(0.01 * k))
            cols = torch.randperm(k, generator=gen, device=device)[:c]
        x[:, cols] *= 20.0
    return x


# --------------------------------------------------------------------------
# the Gemma-3 shapes of the benchmark configs
# --------------------------------------------------------------------------
# per layer: (name, rows n, reduction k); "qkv"/"gu" groups share one input
CONFIGS = {
    "270m": dict(layers=18, dim=640, q=1024, kv=256, ffn=2048, vocab=262144),
    "1b": dict(layers=26, dim=1152, q=1024, kv=256, ffn=6912, vocab=262144),
    "4b": dict(layers=34, dim=2560, q=2048, kv=1024, ffn=10240, vocab=262144),
    "12b": dict(layers=48, dim=3840, q=4096, kv=2048, ffn=15360, vocab=262144),
    "siglip": dict(layers=27, dim=1152, q=1152, kv=1152, ffn=4304, vocab=0),
}


def layer_groups(cfg: dict):
    """The W8A8 calls of one layer, in gemma.c's order (gemma.c:4768-4930 /
    5034-5391): each group is (input width k, [(name, rows)...]) sharing one
    quantized input."""
    d, q, kv, f = cfg["dim"], cfg["q"], cfg["kv"], cfg["ffn"]
    return [
        (d, [("wq", q), ("wk", kv), ("wv", kv)]),
        (q, [("wo", d)]),
        (d, [("w1_up", f), ("w2_gate", f)]),
        (f, [("w3_down", d)]),
    ]


def vision_layer_groups(cfg: dict):
    """The W8A8 calls of one SigLIP encoder layer (gemma.c:4497-4633): Q/K/V
    share one quantized input, then O, fc1 and fc2 (an ungated MLP)."""
    d, f = cfg["dim"], cfg["ffn"]
    return [
        (d, [("wq", d), ("wk", d), ("wv", d)]),
        (d, [("wo", d)]),
        (d, [("w1_fc1", f)]),
        (f, [("w2_fc2", d)]),
    ]


def projector_groups(vision: dict, text: dict):
    """The image-token projection into the text stream (gemma.c:4714-4716)."""
    return [(vision["dim"], [("proj", text["dim"])])]


def groups_ops(groups, m: int) -> int:
    return sum(2 * m * n * k for k, jobs in groups for _, n in jobs)


def layer_ops(cfg: dict, m: int) -> int:
    return groups_ops(layer_groups(cfg), m)


def layer_weight_bytes(cfg: dict) -> int:
    return sum(n * k + 4 * n for k, jobs in layer_groups(cfg) for _, n in jobs)
