"""Generate tests/golden/bin_layout.json from the reference's own model loader.

gemma.c's mmap_gemma_model (gemma.c:1946-2043) is run, through
oracle/ref_harness.c's ref_bin_layout, on synthetic `-q` model files written
by gemma.c_b200/binfmt.py from the configs below (text-only and multimodal,
every combination of the qk_norm / pre / post-FFN norm flags, odd vocabulary
sizes so tensors start at unaligned offsets).  For each file and allow_mm
setting the fixture records where the reference finds every matmul QTensor.
The images themselves are regenerated from (config, seed) by the tests.
Needs the reference sources (run where they are mounted):

    python tests/golden/make_bin_layout.py
"""
from __future__ import annotations

import json
import os
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "gemma.c_b200"))

import binfmt  # noqa: E402
import oracle  # noqa: E402

CASES = [
    # name, text config, vision config, seed
    ("text_plain", dict(nl=3, n_heads=3, nkv=1, hdim=16, dim=48, mlp_dim=64, nvocab=123), None, 1),
    ("text_qk", dict(nl=2, n_heads=2, nkv=2, hdim=24, dim=40, mlp_dim=72, nvocab=257, qk_norm=True), None, 2),
    ("text_all_norms", dict(nl=9, n_heads=4, nkv=1, hdim=16, dim=64, mlp_dim=96, nvocab=301, qk_norm=True,
                            mlp_pre=True, mlp_pst=True), None, 3),
    ("text_pre_only", dict(nl=1, n_heads=1, nkv=1, hdim=8, dim=33, mlp_dim=17, nvocab=50, mlp_pre=True), None, 4),
    ("mm_small", dict(nl=2, n_heads=2, nkv=1, hdim=32, dim=64, mlp_dim=96, nvocab=300, qk_norm=True, mlp_pre=True,
                      mlp_pst=True), dict(nl=2, n_heads=2, mlp_dim=80, dim=48, img_px=56, psize=14), 5),
    ("mm_odd", dict(nl=3, n_heads=2, nkv=1, hdim=20, dim=40, mlp_dim=56, nvocab=77),
     dict(nl=1, n_heads=1, mlp_dim=36, dim=24, img_px=30, psize=6), 6),
]


def main() -> None:
    if not oracle.build_ref():
        raise SystemExit("reference sources not found; cannot generate fixtures")
    R = oracle.Ref("native", threads=1)
    out = []
    for name, text, vision, seed in CASES:
        buf, _ = binfmt.image(text, vision, seed=seed)
        with tempfile.NamedTemporaryFile(suffix=".bin", delete=False) as f:
            f.write(buf.tobytes())
            path = f.name
        try:
            for allow_mm in ([True, False] if vision else [True]):
                out.append({"name": name, "text": text, "vision": vision, "seed": seed, "allow_mm": allow_mm,
                            "bytes": int(buf.nbytes), "qtensors": R.bin_layout(path, allow_mm)})
        finally:
            os.unlink(path)
    with open(os.path.join(HERE, "bin_layout.json"), "w") as f:
        json.dump(out, f, indent=0, separators=(",", ":"))
    print(f"{len(out)} layouts, {sum(len(c['qtensors']) for c in out)} QTensors")


if __name__ == "__main__":
    main()
