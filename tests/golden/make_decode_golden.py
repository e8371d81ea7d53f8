"""Generate tests/golden/decode.npz from the reference's own decode step.

gemma.c's forward_text_decode (gemma.c:4727-4978) runs, through
oracle/ref_harness.c's ref_decode_steps, on small seeded W8A8 decoders
(synth.decoder_model) for positions 0..7 with seeded input embeddings, and
its forward_text_chunk (gemma.c:4985-5455) over chunks of 5 and 11 tokens.
The fixture keeps every step's logits and final hidden state, and the RoPE
tables gemma.c's rope_freqs builds for each position, so the GPU decoder can
be fed the same angles.  Needs the reference sources (run where they are
mounted):

    python tests/golden/make_decode_golden.py
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

NPOS = 8
CHUNKS = [5, 11]  # forward_text_chunk calls from position 0
CASES = {
    # Gemma 3 style: QK norm, pre/post norms, a sliding layer (window 4) and a global one
    "gemma3": dict(tid=1000, nl=2, n_heads=2, nkv=1, hdim=64, dim=128, mlp_dim=256, nvocab=500, q_scale=64,
                   slide=4, swa=[1, 0], qk_norm=True, mlp_pre=True, mlp_pst=True, theta_l=10000.0,
                   theta_g=1000000.0, eps=1e-6, sc_att=0.0, sc_log=0.0),
    # Gemma 2 style: soft-capped scores and logits, no QK norm, 4 query heads over 2 kv heads
    "softcap": dict(tid=2000, nl=3, n_heads=4, nkv=2, hdim=64, dim=96, mlp_dim=192, nvocab=300, q_scale=48,
                    slide=3, swa=[1, 0, 1], qk_norm=False, mlp_pre=True, mlp_pst=True, theta_l=10000.0,
                    theta_g=10000.0, eps=1e-6, sc_att=50.0, sc_log=30.0),
}


def main() -> None:
    if not oracle.build_ref():
        raise SystemExit("reference sources not found; cannot generate fixtures")
    R = oracle.Ref("native", threads=2)
    out = {"meta": np.array(json.dumps({"cases": CASES, "npos": NPOS, "chunks": CHUNKS, "isa": R.isa}))}
    for name, cfg in CASES.items():
        layers, emb, fnorm = synth.decoder_model(cfg["tid"], cfg)
        x0 = synth.normal(cfg["tid"] + 999, (NPOS, cfg["dim"]))
        logits, hid = R.decode_steps(cfg, layers, emb, fnorm, x0)
        slid = np.empty((NPOS, cfg["hdim"]), np.float32)
        full = np.empty((NPOS, cfg["hdim"]), np.float32)
        for p in range(NPOS):
            s, f = R.rope_freqs(cfg["hdim"], cfg["theta_l"], cfg["theta_g"], p, 1)
            slid[p], full[p] = s[0], f[0]
        out.update({f"{name}_logits": logits, f"{name}_hid": hid, f"{name}_slid": slid, f"{name}_full": full})
        # prefill: the same decoder over chunks of CHUNKS tokens
        total = sum(CHUNKS)
        xp = synth.normal(cfg["tid"] + 777, (total, cfg["dim"]))
        plog, phid = R.prefill_chunks(cfg, layers, emb, fnorm, xp, CHUNKS)
        ps, pf = R.rope_freqs(cfg["hdim"], cfg["theta_l"], cfg["theta_g"], 0, total)
        out.update({f"{name}_pre_logits": plog, f"{name}_pre_hid": phid, f"{name}_pslid": ps, f"{name}_pfull": pf})
    np.savez_compressed(os.path.join(HERE, "decode.npz"), **out)
    print(f"{len(CASES)} decoders x {NPOS} positions")


if __name__ == "__main__":
    main()
