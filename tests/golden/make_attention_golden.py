"""Generate tests/golden/attention.npz from the reference's own attention.

gemma.c's decode attention (att_scores_gqa, att_finalize, att_values_gqa,
gemma.c:4836-4848) and its prefill attention loop (gemm_fpx, softmax,
gemm_fpx_nn around the blockwise causal mask, gemma.c:5160-5295), and the
QK-norm / RoPE / KV-cache step before them (rmsnorm, rope_apply and the cache
copies of gemma.c:4775-4818 and 5095-5145, with rope_freqs' own tables), compiled
by ``make -C oracle ref`` with the reference Makefile's flags, run on the
seeded inputs of synth.attention_inputs.  The fixture stores each case's
parameters and the reference's output; the tests regenerate the inputs.
Needs the reference sources (run where they are mounted):

    python tests/golden/make_attention_golden.py
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "gemma.c_b200"))

import oracle  # noqa: E402
import synth  # noqa: E402

# (tensor id, n_heads, nkv, hdim, clen, spos, attlen, softcap)
DECODE = [
    (100, 4, 1, 256, 400, 0, 400, 0.0),      # Gemma-3-1B / 270m heads, full window
    (110, 8, 4, 256, 1200, 177, 1000, 50.0),  # 4B heads, sliding-window start, softcap
    (120, 2, 1, 64, 40, 3, 37, 0.0),
    (130, 16, 8, 128, 2100, 0, 2100, 0.0),    # many splits of the window
    (140, 4, 1, 256, 9, 0, 1, 0.0),           # first token: one position
]
# (tensor id, n_heads, nkv, hdim, spos, ntok, slide, softcap, mask)
PREFILL = [
    (200, 4, 1, 256, 0, 40, 0, 0.0, 1),
    (210, 4, 1, 128, 20, 70, 32, 50.0, 1),   # sliding window, softcap, second chunk
    (220, 2, 2, 64, 5, 33, 0, 0.0, 0),       # dense path
    (230, 8, 4, 64, 100, 64, 48, 0.0, 1),
    (240, 3, 1, 128, 0, 1, 0, 0.0, 1),       # one token
]


# (tensor id, n_heads, nkv, hdim, clen, spos, ntok, q_scale, qk_norm, theta_l, theta_g)
ROPE = [
    (300, 4, 1, 256, 600, 511, 1, 1.0, 1, 10000.0, 1000000.0),     # a decode step (1B heads)
    (310, 8, 4, 256, 300, 100, 40, 0.0625, 1, 10000.0, 1000000.0),  # a prefill chunk, scaled queries
    (320, 2, 1, 64, 40, 0, 24, 0.125, 0, 10000.0, 10000.0),         # no qk_norm
]


def main() -> None:
    if not oracle.build_ref():
        raise SystemExit("reference sources not found; cannot generate fixtures")
    R = oracle.Ref("native", threads=4)
    out = {}
    meta = {"decode": DECODE, "prefill": PREFILL, "isa": R.isa}
    for tid, nh, nkv, hd, clen, spos, attlen, sc in DECODE:
        xq, kc, vc = synth.attention_inputs(tid, nh, nkv, hd, clen)
        out[f"decode_{tid}"] = R.attention_decode(xq, kc, vc, spos, attlen, np.float32(1.0 / np.sqrt(hd)), sc)
    for tid, nh, nkv, hd, spos, ntok, slide, sc, mask in PREFILL:
        xq, kc, vc = synth.attention_inputs(tid, nh, nkv, hd, spos + ntok + 3, ntok)
        out[f"prefill_{tid}"] = R.attention_prefill(xq, kc, vc, spos, slide, sc, bool(mask))
    meta["rope"] = ROPE
    for tid, nh, nkv, hd, clen, spos, ntok, qs, norm, tl, tg in ROPE:
        slid, full = R.rope_freqs(hd, tl, tg, spos, ntok)
        xq, xk, xv, kc, vc, nq, nk = synth.rope_inputs(tid, nh, nkv, hd, clen, ntok, norm)
        rq, rk, _ = R.qk_norm_rope_cache(xq, xk, xv, kc, vc, slid, spos, qs, nq, nk)
        out.update({f"rope_{tid}_freqs": slid, f"rope_{tid}_xq": rq, f"rope_{tid}_k": rk[:, spos:spos + ntok]})
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(os.path.join(HERE, "attention.npz"), **out)
    print(f"{len(DECODE)} decode, {len(PREFILL)} prefill cases")


if __name__ == "__main__":
    main()
