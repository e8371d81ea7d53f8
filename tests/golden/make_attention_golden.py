"""Generate tests/golden/attention.npz from the reference's own attention.

gemma.c's decode attention (att_scores_gqa, att_finalize, att_values_gqa,
gemma.c:4836-4848) and its prefill attention loop (gemm_fpx, softmax,
gemm_fpx_nn around the blockwise causal mask, gemma.c:5160-5295), compiled
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
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(os.path.join(HERE, "attention.npz"), **out)
    print(f"{len(DECODE)} decode, {len(PREFILL)} prefill cases")


if __name__ == "__main__":
    main()
