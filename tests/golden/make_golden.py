"""Generate tests/golden/golden.npz from the reference's own functions.

The reference ships no tests or golden vectors, so the fixtures are made by
running gemma.c's quantize_act / quantize_acts / gemv_int8 / gemv_int8_multi
/ gemm_int8 (gemma.c:2586-2837, 3937-4054), compiled by ``make -C oracle
ref`` with the reference Makefile's -O3 -ffast-math -fopenmp flags, on
seeded synthetic inputs.  Needs the reference sources (this runs where they
are mounted); the committed .npz is what the tests read everywhere else.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "gemma.c_b200"))

import oracle  # noqa: E402
import synth  # noqa: E402


def main() -> None:
    if not oracle.build_ref():
        raise SystemExit("reference sources not found; cannot generate fixtures")
    R = oracle.Ref("native", threads=4)
    out = {"meta_isa": np.array(R.isa), "meta_variant": np.array("native")}

    # quantize: random rows, an all-zero row, rounding-boundary values
    x = synth.activations(1, 6, 640, outliers=True)
    x[2] = 0.0
    x[3, :8] = [127.0, 63.5, -63.5, 0.5, -0.5, 1.5, -2.5, 126.5]
    x[3, 8:] = 0.25
    q, s = R.quantize_acts(x)
    out.update(quant_a_x=x, quant_a_q=q, quant_a_s=s)
    # odd width from a strided source (sstr = 40 floats per row, n = 33)
    xs = synth.activations(2, 3, 40)
    q, s = R.quantize_acts(xs, n=33, sstr=40)
    out.update(quant_b_x=xs, quant_b_q=q, quant_b_s=s)
    # single-vector quantize_act
    v = synth.activations(3, 1, 1152)[0]
    q, sc = R.quantize_act(v)
    out.update(quant_c_x=v, quant_c_q=q, quant_c_s=np.float32(sc))

    # gemv (decode): dense, and an odd reduction length
    for name, (n, k, tid) in {"gemv_a": (96, 640, 10), "gemv_b": (37, 33, 11)}.items():
        w, ws = synth.weight(tid, n, k)
        xq, xsc = R.quantize_act(synth.activations(tid + 100, 1, k)[0])
        y = R.gemv_int8(w, ws, xq, xsc)
        out.update({f"{name}_w": w, f"{name}_ws": ws, f"{name}_x": xq, f"{name}_xs": np.float32(xsc),
                    f"{name}_y": y})

    # gemv_int8_multi with Q/K/V-like jobs
    k = 640
    mats, scs = [], []
    for j, rows in enumerate((64, 16, 16)):
        w, ws = synth.weight(20 + j, rows, k)
        mats.append(w)
        scs.append(ws)
    xq, xsc = R.quantize_act(synth.activations(120, 1, k)[0])
    ys = R.gemv_int8_multi(mats, scs, xq, xsc)
    for j in range(3):
        out.update({f"multi_w{j}": mats[j], f"multi_ws{j}": scs[j], f"multi_y{j}": ys[j]})
    out.update(multi_x=xq, multi_xs=np.float32(xsc))

    # gemm (prefill): dense, ragged tails, strided operands, m beyond one tile
    for name, (m, n, k, tid) in {"gemm_a": (20, 40, 256, 30), "gemm_b": (13, 11, 40, 31),
                                 "gemm_d": (130, 24, 160, 32)}.items():
        w, ws = synth.weight(tid, n, k)
        xq, xsc = R.quantize_acts(synth.activations(tid + 100, m, k, outliers=True))
        y = R.gemm_int8(w, ws, xq, xsc)
        out.update({f"{name}_w": w, f"{name}_ws": ws, f"{name}_x": xq, f"{name}_xs": xsc, f"{name}_y": y})
    # strided: dstr 30, mstr 80, sstr 72 for m 9, n 24, k 64
    m, n, k, dstr, mstr, sstr = 9, 24, 64, 30, 80, 72
    wfull, wsc = synth.weight(33, n, mstr)
    xfull, xsc = R.quantize_acts(synth.activations(133, m, sstr))
    dst = np.full((m, dstr), -1.0, np.float32)
    R.gemm_int8(wfull.reshape(-1), wsc, xfull.reshape(-1), xsc, dst=dst, dstr=dstr, mstr=mstr, sstr=sstr,
                m=m, n=n, k=k)
    out.update(gemm_c_w=wfull, gemm_c_ws=wsc, gemm_c_x=xfull, gemm_c_xs=xsc, gemm_c_y=dst,
               gemm_c_dims=np.array([m, n, k, dstr, mstr, sstr], np.int32))

    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes, isa {R.isa})")


if __name__ == "__main__":
    main()
