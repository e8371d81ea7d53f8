"""Generate tests/golden/vision.npz from the reference's own forward_vision.

gemma.c's forward_vision (gemma.c:4391-4720) runs, through
oracle/ref_harness.c's ref_vision_head, on a SigLIP encoder with no layers:
the patch and position embedding (4411-4466), the post LayerNorm, average
pooling and RMSNorm (4660-4705), quantize_acts and the int8 projection
(4714-4716).  Inputs are synth.vision_head_inputs (seeded); the fixture keeps
the pooled rows, their codes and scales, and the projection output.  Needs
the reference sources (run where they are mounted):

    python tests/golden/make_vision_golden.py
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

# (tensor id, img_px, psize, dim, img_tok, text dim)
CASES = [
    (600, 112, 14, 96, 16, 64),    # 8 x 8 patches pooled 2 x 2
    (610, 224, 14, 192, 64, 128),  # 16 x 16 patches pooled 2 x 2
    (620, 96, 8, 72, 9, 40),       # 12 x 12 patches pooled 4 x 4, odd sizes
    (630, 56, 14, 64, 16, 32),     # no pooling (1 x 1)
]


def main() -> None:
    if not oracle.build_ref():
        raise SystemExit("reference sources not found; cannot generate fixtures")
    R = oracle.Ref("native", threads=4)
    out = {"meta": np.array(json.dumps({"cases": CASES, "isa": R.isa}))}
    for case in CASES:
        tid = case[0]
        v = synth.vision_head_inputs(*case)
        y, pooled, q, s = R.vision_head(v)
        out.update({f"proj_{tid}": y, f"pooled_{tid}": pooled, f"q_{tid}": q, f"s_{tid}": s})
    np.savez_compressed(os.path.join(HERE, "vision.npz"), **out)
    print(f"{len(CASES)} cases")


if __name__ == "__main__":
    main()
