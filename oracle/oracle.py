"""ctypes bindings to the CPU checkers (test infrastructure only).

Two libraries live here:

* ``liboracle.so`` -- the C restatement of Gemma.c's W8A8 hot path
  (``gemma_oracle.c``; each function cites the gemma.c lines it follows).
* ``_ref/libgemma_ref_<isa>.so`` -- the reference's own ``quantize_act``,
  ``quantize_acts``, ``gemv_int8``, ``gemv_int8_multi`` and ``gemm_int8``
  compiled from gemma.c (gemma.c:2586-2837, 3937-4054) with its Makefile's
  -O3 -ffast-math -fopenmp flags.  Present wherever ``make -C oracle ref`` ran
  (the build machine); it is shipped as a built file, the source is not.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this module.  The product (gemma.c_b200) never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

_i8p = ctypes.POINTER(ctypes.c_int8)
_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)


class GemvJob(ctypes.Structure):
    """gemma.c:2795 GemvJob with floatx = float."""
    _fields_ = [("w", ctypes.c_void_p), ("sc", _f32p), ("dst", _f32p), ("m", ctypes.c_int)]


def _ptr(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"] or a.ndim == 0
    return a.ctypes.data_as(t)


def build() -> None:
    """Compile liboracle.so (the restatement). Needs only gcc."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)


def ref_source_dir() -> str:
    """Where the reference sources lie: $GEMMA_REF_DIR, else the Makefile's
    REF_DIR default (the one place that default is written)."""
    env = os.environ.get("GEMMA_REF_DIR")
    if env:
        return env
    out = subprocess.run(["make", "-s", "--no-print-directory", "-C", HERE, "refdir"],
                         capture_output=True, text=True)
    return out.stdout.strip()


def build_ref(ref_dir: str | None = None) -> bool:
    """Compile the reference harness when the reference sources are present."""
    ref_dir = ref_dir or ref_source_dir()
    if not ref_dir or not os.path.isfile(os.path.join(ref_dir, "gemma.c")):
        return False
    subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF_DIR={ref_dir}"], check=True)
    # gemma.c with the CUDA drop-in, when libgcu.so has been built
    if os.path.exists(os.path.join(HERE, "..", "gemma.c_b200", "libgcu.so")):
        subprocess.run(["make", "-s", "-C", HERE, "dropin", f"REF_DIR={ref_dir}"], check=True)
    return True


_orc = None


def orc() -> ctypes.CDLL:
    global _orc
    if _orc is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        lib = ctypes.CDLL(path)
        lib.orc_quantize_act.restype = ctypes.c_float
        lib.orc_quantize_act.argtypes = [_i8p, _f32p, ctypes.c_int]
        lib.orc_quantize_acts.restype = None
        lib.orc_quantize_acts.argtypes = [_i8p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        lib.orc_acc_int8.restype = None
        lib.orc_acc_int8.argtypes = [_i32p, _i8p, ctypes.c_int, _i8p, ctypes.c_int,
                                     ctypes.c_int, ctypes.c_int, ctypes.c_int]
        lib.orc_gemv_int8.restype = None
        lib.orc_gemv_int8.argtypes = [_f32p, _i8p, _f32p, _i8p, ctypes.c_float, ctypes.c_int, ctypes.c_int]
        lib.orc_gemv_int8_multi.restype = None
        lib.orc_gemv_int8_multi.argtypes = [ctypes.POINTER(GemvJob), ctypes.c_int, _i8p,
                                            ctypes.c_float, ctypes.c_int]
        lib.orc_gemm_int8.restype = ctypes.c_int
        lib.orc_gemm_int8.argtypes = [_f32p, ctypes.c_int, _i8p, ctypes.c_int, _f32p, _i8p,
                                      ctypes.c_int, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        lib.orc_quantize_weight_rows.restype = None
        lib.orc_quantize_weight_rows.argtypes = [_i8p, _f32p, _f32p, ctypes.c_int, ctypes.c_int]
        lib.orc_rmsnorm_quantize.restype = None
        lib.orc_rmsnorm_quantize.argtypes = [_i8p, _f32p, _f32p, _f32p, _f32p, ctypes.c_float,
                                             ctypes.c_int, ctypes.c_int]
        lib.orc_geglu_quantize.restype = None
        lib.orc_geglu_quantize.argtypes = [_i8p, _f32p, _f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int]
        lib.orc_attention_decode.restype = None
        lib.orc_attention_decode.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_long] + [ctypes.c_int] * 5 + \
            [ctypes.c_float, ctypes.c_float, _f32p]
        lib.orc_attention_prefill.restype = None
        lib.orc_attention_prefill.argtypes = [_f32p, ctypes.c_int, _f32p, _f32p, _f32p, ctypes.c_long] + \
            [ctypes.c_int] * 6 + [ctypes.c_float, ctypes.c_int, _f32p]
        lib.orc_qk_norm_rope_cache.restype = None
        lib.orc_qk_norm_rope_cache.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_long, _f32p, _f32p,
                                               ctypes.c_float, _f32p, ctypes.c_float] + [ctypes.c_int] * 5
        lib.orc_patch_embed.restype = None
        lib.orc_patch_embed.argtypes = [_f32p, _f32p, _f32p, _f32p, _i8p, _f32p, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int]
        lib.orc_vision_pool.restype = None
        lib.orc_vision_pool.argtypes = [_i8p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_float,
                                        ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p]
        _orc = lib
    return _orc


# --------------------------------------------------------------------------
# restatement wrappers (numpy in, numpy out)
# --------------------------------------------------------------------------

def quantize_act(vec: np.ndarray):
    vec = np.ascontiguousarray(vec, dtype=np.float32)
    dst = np.empty(vec.shape[0], np.int8)
    sc = orc().orc_quantize_act(_ptr(dst, _i8p), _ptr(vec, _f32p), vec.shape[0])
    return dst, np.float32(sc)


def quantize_acts(src: np.ndarray, n: int | None = None, sstr: int = 0):
    """src is (m, sstr) fp32 (sstr >= n); returns int8 (m, n) and fp32 (m,)."""
    src = np.ascontiguousarray(src, dtype=np.float32)
    m = src.shape[0]
    n = src.shape[1] if n is None else n
    dst = np.empty((m, n), np.int8)
    dsc = np.empty(m, np.float32)
    orc().orc_quantize_acts(_ptr(dst, _i8p), _ptr(dsc, _f32p), _ptr(src, _f32p), sstr, m, n)
    return dst, dsc


def acc_int8(mat: np.ndarray, src: np.ndarray) -> np.ndarray:
    """int32 accumulators acc[i, j] = sum_l src[i, l] * mat[j, l] (dense)."""
    mat = np.ascontiguousarray(mat, np.int8)
    src = np.ascontiguousarray(src, np.int8)
    m, k = src.shape
    n = mat.shape[0]
    acc = np.empty((m, n), np.int32)
    orc().orc_acc_int8(_ptr(acc, _i32p), _ptr(mat, _i8p), k, _ptr(src, _i8p), k, m, n, k)
    return acc


def gemv_int8(mat, matsc, vec, vsc):
    mat = np.ascontiguousarray(mat, np.int8)
    matsc = np.ascontiguousarray(matsc, np.float32)
    vec = np.ascontiguousarray(vec, np.int8)
    m, n = mat.shape
    dst = np.empty(m, np.float32)
    orc().orc_gemv_int8(_ptr(dst, _f32p), _ptr(mat, _i8p), _ptr(matsc, _f32p), _ptr(vec, _i8p),
                        float(vsc), m, n)
    return dst


def gemv_int8_multi(mats, scs, vec, vsc):
    vec = np.ascontiguousarray(vec, np.int8)
    mats = [np.ascontiguousarray(w, np.int8) for w in mats]
    scs = [np.ascontiguousarray(s, np.float32) for s in scs]
    outs = [np.empty(w.shape[0], np.float32) for w in mats]
    jobs = (GemvJob * len(mats))()
    for j, (w, s, o) in enumerate(zip(mats, scs, outs)):
        jobs[j] = GemvJob(w.ctypes.data, _ptr(s, _f32p), _ptr(o, _f32p), w.shape[0])
    orc().orc_gemv_int8_multi(jobs, len(mats), _ptr(vec, _i8p), float(vsc), vec.shape[0])
    return outs


def gemm_int8(mat, matsc, src, ssc, dst=None, dstr=0, mstr=0, sstr=0, m=None, n=None, k=None):
    """NT GEMM; with strides the arrays are flat buffers and m, n, k are given."""
    mat = np.ascontiguousarray(mat, np.int8)
    src = np.ascontiguousarray(src, np.int8)
    matsc = np.ascontiguousarray(matsc, np.float32)
    ssc = np.ascontiguousarray(ssc, np.float32)
    if m is None:
        m, k = src.shape
        n = mat.shape[0]
    if dst is None:
        dst = np.zeros((m, n), np.float32)
    orc().orc_gemm_int8(_ptr(dst, _f32p), dstr, _ptr(mat, _i8p), mstr, _ptr(matsc, _f32p),
                        _ptr(src, _i8p), sstr, _ptr(ssc, _f32p), m, n, k)
    return dst


def quantize_weight_rows(w: np.ndarray):
    w = np.ascontiguousarray(w, np.float32)
    n, k = w.shape
    q = np.empty((n, k), np.int8)
    s = np.empty(n, np.float32)
    orc().orc_quantize_weight_rows(_ptr(q, _i8p), _ptr(s, _f32p), _ptr(w, _f32p), n, k)
    return q, s


def rmsnorm_quantize(x: np.ndarray, w: np.ndarray, eps: float):
    """(m, dim) fp32 rows -> RMSNorm'd rows, their int8 codes and scales."""
    x = np.ascontiguousarray(x, np.float32)
    m, dim = x.shape
    w = np.ascontiguousarray(w, np.float32)
    xn = np.empty((m, dim), np.float32)
    q = np.empty((m, dim), np.int8)
    s = np.empty(m, np.float32)
    orc().orc_rmsnorm_quantize(_ptr(q, _i8p), _ptr(s, _f32p), _ptr(xn, _f32p), _ptr(x, _f32p),
                               _ptr(w, _f32p), eps, m, dim)
    return xn, q, s


def geglu_quantize(gate: np.ndarray, up: np.ndarray):
    """(m, dim) gate and up rows -> gelu_tanh(gate) * up, its codes and scales."""
    gate = np.ascontiguousarray(gate, np.float32)
    up = np.ascontiguousarray(up, np.float32)
    m, dim = gate.shape
    h = np.empty((m, dim), np.float32)
    q = np.empty((m, dim), np.int8)
    s = np.empty(m, np.float32)
    orc().orc_geglu_quantize(_ptr(q, _i8p), _ptr(s, _f32p), _ptr(h, _f32p), _ptr(gate, _f32p),
                             _ptr(up, _f32p), m, dim)
    return h, q, s


def _cache(kc, vc):
    """(nkv, clen, hdim) K and V caches -> contiguous arrays and the head stride."""
    kc = np.ascontiguousarray(kc, np.float32)
    vc = np.ascontiguousarray(vc, np.float32)
    assert kc.shape == vc.shape and kc.ndim == 3
    return kc, vc, kc.shape[1] * kc.shape[2]


def attention_decode(xq, kc, vc, spos, attlen, asc, sc_att=0.0):
    """gemma.c:4836-4848: xq (n_heads, hdim); caches (nkv, clen, hdim);
    the window [spos, spos+attlen).  Returns xo (n_heads, hdim)."""
    xq = np.ascontiguousarray(xq, np.float32)
    kc, vc, stride = _cache(kc, vc)
    n_heads, hdim = xq.shape
    xo = np.empty((n_heads, hdim), np.float32)
    att = np.empty(n_heads * attlen, np.float32)
    orc().orc_attention_decode(_ptr(xo, _f32p), _ptr(xq, _f32p), _ptr(kc, _f32p), _ptr(vc, _f32p), stride,
                               n_heads, kc.shape[0], hdim, spos, attlen, asc, sc_att, _ptr(att, _f32p))
    return xo


def attention_prefill(xq, kc, vc, spos, slide=0, sc_att=0.0, mask=True):
    """gemma.c:5160-5295: xq (n_heads, ntok, hdim), rotated and scaled;
    caches (nkv, clen, hdim) holding this chunk at [spos, spos+ntok).
    Returns xo (ntok, n_heads*hdim)."""
    xq = np.ascontiguousarray(xq, np.float32)
    kc, vc, stride = _cache(kc, vc)
    n_heads, ntok, hdim = xq.shape
    xo = np.empty((ntok, n_heads * hdim), np.float32)
    att = np.empty(spos + ntok, np.float32)
    orc().orc_attention_prefill(_ptr(xo, _f32p), n_heads * hdim, _ptr(xq, _f32p), _ptr(kc, _f32p),
                                _ptr(vc, _f32p), stride, n_heads, kc.shape[0], hdim, spos, ntok, slide,
                                sc_att, int(mask), _ptr(att, _f32p))
    return xo


def qk_norm_rope_cache(xq, xk, xv, kc, vc, freqs, spos, q_scale=1.0, nq=None, nk=None, eps=1e-6):
    """gemma.c:4775-4818 / 5095-5145: returns (rotated xq, k cache, v cache)
    after writing the chunk at [spos, spos+ntok); inputs are not modified."""
    xq = np.array(xq, np.float32, copy=True)
    xk = np.array(xk, np.float32, copy=True)
    xv = np.ascontiguousarray(xv, np.float32)
    kc = np.array(kc, np.float32, copy=True)
    vc = np.array(vc, np.float32, copy=True)
    freqs = np.ascontiguousarray(freqs, np.float32)
    n_heads, ntok, hdim = xq.shape
    nq = None if nq is None else np.ascontiguousarray(nq, np.float32)
    nk = None if nk is None else np.ascontiguousarray(nk, np.float32)
    orc().orc_qk_norm_rope_cache(_ptr(xq, _f32p), _ptr(xk, _f32p), _ptr(xv, _f32p), _ptr(kc, _f32p), _ptr(vc, _f32p),
                                 kc.shape[1] * hdim, _ptr(nq, _f32p) if nq is not None else None,
                                 _ptr(nk, _f32p) if nk is not None else None, eps, _ptr(freqs, _f32p), q_scale,
                                 n_heads, kc.shape[0], hdim, spos, ntok)
    return xq, kc, vc


def patch_embed(v: dict):
    """gemma.c:4411-4466 on synth.vision_head_inputs: (npatch, dim) fp32."""
    ppi = v["img_px"] // v["psize"]
    dim = v["dim"]
    x = np.empty((ppi * ppi, dim), np.float32)
    orc().orc_patch_embed(_ptr(x, _f32p), _ptr(v["img"], _f32p), _ptr(v["pe"], _f32p), _ptr(v["pe_b"], _f32p),
                          _ptr(v["pos_q"], _i8p), _ptr(v["pos_s"], _f32p), v["img_px"], v["psize"], dim)
    return x


def vision_pool(x: np.ndarray, v: dict):
    """gemma.c:4660-4705 + the quantize of 4714: pooled rows, codes, scales."""
    x = np.ascontiguousarray(x, np.float32)
    ppi = v["img_px"] // v["psize"]
    side = int(round(np.sqrt(v["img_tok"])))
    dim = v["dim"]
    out = np.empty((side * side, dim), np.float32)
    q = np.empty((side * side, dim), np.int8)
    s = np.empty(side * side, np.float32)
    scratch = np.empty(dim, np.float32)
    orc().orc_vision_pool(_ptr(q, _i8p), _ptr(s, _f32p), _ptr(out, _f32p), _ptr(x, _f32p), _ptr(v["post_n"], _f32p),
                          _ptr(v["post_nb"], _f32p), _ptr(v["norm"], _f32p), v["eps"], ppi, side, dim,
                          _ptr(scratch, _f32p))
    return out, q, s


# --------------------------------------------------------------------------
# the compiled reference (gemma.c's own functions)
# --------------------------------------------------------------------------

def cpu_flags() -> set:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


def native_build_flags() -> set | None:
    """ISA flags of the CPU the native reference build was compiled for."""
    p = os.path.join(REF_DIR, "native_flags.txt")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        return {ln.strip() for ln in f if ln.strip()}


def native_build_cpu() -> str:
    p = os.path.join(REF_DIR, "native_cpu.txt")
    return open(p).read().strip().replace("\n", "; ") if os.path.exists(p) else "unknown"


def ref_build_desc(variant: str) -> str:
    """The compiler flags of a reference build, for benchmark records."""
    if variant == "native":
        return (f"gcc -Ofast -fopenmp -march=native -mtune=native, built for {native_build_cpu()}; "
                "this host has every ISA flag of that CPU")
    return f"gcc -Ofast -fopenmp -march=x86-64-{variant}"


def ref_variant() -> str | None:
    """Best reference build this host can run: native (-march=native of a
    CPU whose ISA flags this host has, every one of them: then it is this
    host's own -march=native build), v4 (AVX-512) or v3 (AVX2+FMA)."""
    flags = cpu_flags()
    avail = {v: os.path.join(REF_DIR, f"libgemma_ref_{v}.so") for v in ("native", "v4", "v3")}
    built_for = native_build_flags()
    if os.path.exists(avail["native"]) and built_for is not None and built_for <= flags:
        return "native"
    if {"avx512f", "avx512bw", "avx512cd", "avx512dq", "avx512vl"} <= flags and os.path.exists(avail["v4"]):
        return "v4"
    if {"avx2", "fma", "bmi2"} <= flags and os.path.exists(avail["v3"]):
        return "v3"
    return None


_refs: dict = {}


def ref(variant: str | None = None) -> ctypes.CDLL | None:
    variant = variant or ref_variant()
    if variant is None:
        return None
    if variant in _refs:
        return _refs[variant]
    path = os.path.join(REF_DIR, f"libgemma_ref_{variant}.so")
    if not os.path.exists(path):
        return None
    lib = ctypes.CDLL(path)
    lib.ref_quantize_act.restype = ctypes.c_float
    lib.ref_quantize_act.argtypes = [_i8p, _f32p, ctypes.c_int]
    lib.ref_quantize_acts.restype = None
    lib.ref_quantize_acts.argtypes = [_i8p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    lib.ref_gemv_int8.restype = None
    lib.ref_gemv_int8.argtypes = [_f32p, _i8p, _f32p, _i8p, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    lib.ref_gemv_int8_multi.restype = None
    lib.ref_gemv_int8_multi.argtypes = [ctypes.POINTER(GemvJob), ctypes.c_int, _i8p, ctypes.c_float,
                                        ctypes.c_int, ctypes.c_int]
    lib.ref_gemm_int8.restype = ctypes.c_int
    lib.ref_gemm_int8.argtypes = [_f32p, ctypes.c_int, _i8p, ctypes.c_int, _f32p, _i8p, ctypes.c_int,
                                  _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    lib.ref_setup.restype = None
    lib.ref_rmsnorm.restype = None
    lib.ref_rmsnorm.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_float]
    lib.ref_gelu_mul.restype = None
    lib.ref_gelu_mul.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int]
    lib.ref_isa.restype = ctypes.c_char_p
    if hasattr(lib, "ref_attention_decode"):
        lib.ref_attention_decode.restype = None
        lib.ref_attention_decode.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_long] + [ctypes.c_int] * 5 + \
            [ctypes.c_float, ctypes.c_float, _f32p, ctypes.c_int]
        lib.ref_attention_prefill.restype = ctypes.c_int
        lib.ref_attention_prefill.argtypes = [_f32p, ctypes.c_int, _f32p, _f32p, _f32p, ctypes.c_long] + \
            [ctypes.c_int] * 6 + [ctypes.c_float, ctypes.c_int, _f32p, ctypes.c_int]
    if hasattr(lib, "ref_vision_head"):
        lib.ref_vision_head.restype = ctypes.c_int
        lib.ref_vision_head.argtypes = [_f32p, _f32p, _i8p, _f32p, _f32p] + [ctypes.c_int] * 5 + \
            [ctypes.c_float, _f32p, _f32p, _i8p, _f32p, _f32p, _f32p, _f32p, _i8p, _f32p, ctypes.c_int]
    if hasattr(lib, "ref_qk_norm_rope_cache"):
        lib.ref_rope_freqs.restype = None
        lib.ref_rope_freqs.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                       ctypes.c_int, ctypes.c_int]
        lib.ref_qk_norm_rope_cache.restype = None
        lib.ref_qk_norm_rope_cache.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_long, _f32p, _f32p,
                                               ctypes.c_float, _f32p, ctypes.c_float] + [ctypes.c_int] * 5
    _model_args = [ctypes.POINTER(ctypes.c_int)] + [ctypes.c_int] * 3 + [ctypes.c_float] * 5 + \
        [ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p), _i8p, _f32p, _f32p, ctypes.c_int]
    if hasattr(lib, "ref_decode_steps"):
        lib.ref_decode_steps.restype = ctypes.c_int
        lib.ref_decode_steps.argtypes = [_f32p, _f32p, _f32p] + [ctypes.c_int] * 10 + _model_args
    if hasattr(lib, "ref_prefill_chunks"):
        lib.ref_prefill_chunks.restype = ctypes.c_int
        lib.ref_prefill_chunks.argtypes = [_f32p, _f32p, _f32p, ctypes.POINTER(ctypes.c_int)] + \
            [ctypes.c_int] * 10 + _model_args
    if hasattr(lib, "ref_read_model_seconds"):
        lib.ref_read_model_seconds.restype = ctypes.c_double
        lib.ref_read_model_seconds.argtypes = [ctypes.c_char_p, ctypes.c_int]
    if hasattr(lib, "ref_bin_layout"):
        lib.ref_bin_layout.restype = ctypes.c_int
        lib.ref_bin_layout.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_longlong),
                                       ctypes.c_int]
    if hasattr(lib, "ref_qkv_head_tasks"):
        lib.ref_qkv_head_tasks.restype = ctypes.c_int
        lib.ref_qkv_head_tasks.argtypes = [_f32p] * 3 + [_i8p, _f32p] * 3 + [_i8p, _f32p] + [ctypes.c_int] * 6
    lib.ref_gemv_job_size.restype = ctypes.c_int
    assert lib.ref_gemv_job_size() == ctypes.sizeof(GemvJob)
    lib.ref_setup()
    _refs[variant] = lib
    return lib


class Ref:
    """numpy-level calls into the compiled reference."""

    def __init__(self, variant: str | None = None, threads: int | None = None):
        self.lib = ref(variant)
        if self.lib is None:
            raise RuntimeError("reference build not available (run make -C oracle ref)")
        self.variant = variant or ref_variant()
        self.threads = threads or os.cpu_count() or 1

    @property
    def isa(self) -> str:
        return self.lib.ref_isa().decode()

    def quantize_act(self, vec):
        vec = np.ascontiguousarray(vec, np.float32)
        dst = np.empty(vec.shape[0], np.int8)
        sc = self.lib.ref_quantize_act(_ptr(dst, _i8p), _ptr(vec, _f32p), vec.shape[0])
        return dst, np.float32(sc)

    def quantize_acts(self, src, n=None, sstr=0):
        src = np.ascontiguousarray(src, np.float32)
        m = src.shape[0]
        n = src.shape[1] if n is None else n
        dst = np.empty((m, n), np.int8)
        dsc = np.empty(m, np.float32)
        self.lib.ref_quantize_acts(_ptr(dst, _i8p), _ptr(dsc, _f32p), _ptr(src, _f32p), sstr, m, n,
                                   self.threads)
        return dst, dsc

    def bin_layout(self, path: str, allow_mm: bool = True):
        """The matmul QTensors gemma.c's mmap_gemma_model finds in a model
        file, as gcu_bin_qtensors lists them (offsets from the file start)."""
        kinds = ("lm_head", "wq", "wk", "wv", "wo", "w1", "w2", "w3",
                 "vwq", "vwk", "vwv", "vwo", "vw1", "vw2", "vproj")
        n = self.lib.ref_bin_layout(path.encode(), int(allow_mm), None, 0)
        if n < 0:
            raise RuntimeError(f"the reference refused {path}")
        rec = (ctypes.c_longlong * (6 * max(n, 1)))()
        self.lib.ref_bin_layout(path.encode(), int(allow_mm), rec, n)
        return [{"kind": kinds[rec[6 * i]], "layer": int(rec[6 * i + 1]), "rows": int(rec[6 * i + 4]),
                 "k": int(rec[6 * i + 5]), "q_off": int(rec[6 * i + 2]), "s_off": int(rec[6 * i + 3])}
                for i in range(n)]

    def attention_decode(self, xq, kc, vc, spos, attlen, asc, sc_att=0.0):
        """gemma.c's decode attention (att_scores_gqa, att_finalize,
        att_values_gqa) on the same arguments as oracle.attention_decode."""
        xq = np.ascontiguousarray(xq, np.float32)
        kc, vc, stride = _cache(kc, vc)
        n_heads, hdim = xq.shape
        xo = np.empty((n_heads, hdim), np.float32)
        att = np.empty(spos + n_heads * attlen, np.float32)
        self.lib.ref_attention_decode(_ptr(xo, _f32p), _ptr(xq, _f32p), _ptr(kc, _f32p), _ptr(vc, _f32p), stride,
                                      n_heads, kc.shape[0], hdim, spos, attlen, asc, sc_att, _ptr(att, _f32p),
                                      self.threads)
        return xo

    def attention_prefill(self, xq, kc, vc, spos, slide=0, sc_att=0.0, mask=True):
        """gemma.c's prefill attention loop on the same arguments as
        oracle.attention_prefill."""
        xq = np.ascontiguousarray(xq, np.float32)
        kc, vc, stride = _cache(kc, vc)
        n_heads, ntok, hdim = xq.shape
        xo = np.empty((ntok, n_heads * hdim), np.float32)
        att = np.zeros(n_heads * ntok * (spos + ntok), np.float32)
        if self.lib.ref_attention_prefill(_ptr(xo, _f32p), n_heads * hdim, _ptr(xq, _f32p), _ptr(kc, _f32p),
                                          _ptr(vc, _f32p), stride, n_heads, kc.shape[0], hdim, spos, ntok, slide,
                                          sc_att, int(mask), _ptr(att, _f32p), self.threads):
            raise RuntimeError("reference attention_prefill failed")
        return xo

    def rope_freqs(self, hdim, theta_l, theta_g, pos, n):
        """gemma.c's rope_freqs: (sliding, full) tables, (n, hdim) each."""
        slid = np.empty((n, hdim), np.float32)
        full = np.empty((n, hdim), np.float32)
        self.lib.ref_rope_freqs(_ptr(slid, _f32p), _ptr(full, _f32p), hdim, hdim, theta_l, theta_g, pos, n)
        return slid, full

    def qk_norm_rope_cache(self, xq, xk, xv, kc, vc, freqs, spos, q_scale=1.0, nq=None, nk=None, eps=1e-6):
        """The reference's rmsnorm / rope_apply / cache copies on the same
        arguments as oracle.qk_norm_rope_cache."""
        xq = np.array(xq, np.float32, copy=True)
        xk = np.array(xk, np.float32, copy=True)
        xv = np.ascontiguousarray(xv, np.float32)
        kc = np.array(kc, np.float32, copy=True)
        vc = np.array(vc, np.float32, copy=True)
        freqs = np.ascontiguousarray(freqs, np.float32)
        n_heads, ntok, hdim = xq.shape
        nq = None if nq is None else np.ascontiguousarray(nq, np.float32)
        nk = None if nk is None else np.ascontiguousarray(nk, np.float32)
        self.lib.ref_qk_norm_rope_cache(_ptr(xq, _f32p), _ptr(xk, _f32p), _ptr(xv, _f32p), _ptr(kc, _f32p),
                                        _ptr(vc, _f32p), kc.shape[1] * hdim, _ptr(nq, _f32p) if nq is not None else None,
                                        _ptr(nk, _f32p) if nk is not None else None, eps, _ptr(freqs, _f32p), q_scale,
                                        n_heads, kc.shape[0], hdim, spos, ntok)
        return xq, kc, vc

    def _model(self, cfg, layers, emb, fnorm):
        """ctypes arguments describing a decoder (and the arrays they point into)."""
        keep = []
        qt = (ctypes.c_void_p * (14 * cfg["nl"]))()
        nrm = (ctypes.c_void_p * (6 * cfg["nl"]))()
        for l, lay in enumerate(layers):
            for j, k in enumerate(("wq", "wk", "wv", "wo", "w1", "w2", "w3")):
                q, s = np.ascontiguousarray(lay[k][0], np.int8), np.ascontiguousarray(lay[k][1], np.float32)
                keep += [q, s]
                qt[14 * l + 2 * j], qt[14 * l + 2 * j + 1] = q.ctypes.data, s.ctypes.data
            for j, k in enumerate(("n1", "n2", "n3", "n4", "nq", "nk")):
                v = np.ascontiguousarray(lay[k], np.float32)
                keep.append(v)
                nrm[6 * l + j] = v.ctypes.data
        swa = (ctypes.c_int * cfg["nl"])(*[int(b) for b in cfg["swa"]])
        eq, es = np.ascontiguousarray(emb[0], np.int8), np.ascontiguousarray(emb[1], np.float32)
        fn = np.ascontiguousarray(fnorm, np.float32)
        keep += [eq, es, fn, swa]
        dims = [cfg["nl"], cfg["n_heads"], cfg["nkv"], cfg["hdim"], cfg["dim"], cfg["mlp_dim"], cfg["nvocab"],
                cfg["q_scale"], cfg["slide"]]
        rest = [swa, int(cfg["qk_norm"]), int(cfg["mlp_pre"]), int(cfg["mlp_pst"]), cfg["theta_l"], cfg["theta_g"],
                cfg["eps"], cfg["sc_att"], cfg["sc_log"], qt, nrm, _ptr(eq, _i8p), _ptr(es, _f32p), _ptr(fn, _f32p),
                self.threads]
        return dims, rest, keep

    def decode_steps(self, cfg: dict, layers: list, emb, fnorm, x0):
        """gemma.c's forward_text_decode for positions 0 .. len(x0)-1 on a
        decoder built from synth.decoder_model-style tensors; returns the
        logits (npos, nvocab) and final hidden states (npos, dim)."""
        x0 = np.ascontiguousarray(x0, np.float32)
        npos = x0.shape[0]
        dims, rest, keep = self._model(cfg, layers, emb, fnorm)
        logits = np.empty((npos, cfg["nvocab"]), np.float32)
        hid = np.empty((npos, cfg["dim"]), np.float32)
        rc = self.lib.ref_decode_steps(_ptr(logits, _f32p), _ptr(hid, _f32p), _ptr(x0, _f32p), npos, *dims, *rest)
        del keep
        if rc:
            raise RuntimeError("reference forward_text_decode failed")
        return logits, hid

    def prefill_chunks(self, cfg: dict, layers: list, emb, fnorm, x0, chunks):
        """gemma.c's forward_text_chunk over consecutive chunks from position
        0; returns each chunk's last-token logits (len(chunks), nvocab) and
        every token's final hidden state (sum(chunks), dim)."""
        x0 = np.ascontiguousarray(x0, np.float32)
        assert x0.shape[0] == sum(chunks)
        dims, rest, keep = self._model(cfg, layers, emb, fnorm)
        ch = (ctypes.c_int * len(chunks))(*chunks)
        logits = np.empty((len(chunks), cfg["nvocab"]), np.float32)
        hid = np.empty((x0.shape[0], cfg["dim"]), np.float32)
        rc = self.lib.ref_prefill_chunks(_ptr(logits, _f32p), _ptr(hid, _f32p), _ptr(x0, _f32p), ch, len(chunks), *dims,
                                         *rest)
        del keep
        if rc:
            raise RuntimeError("reference forward_text_chunk failed")
        return logits, hid

    def vision_head(self, v: dict):
        """gemma.c's forward_vision with no encoder layers on
        synth.vision_head_inputs: (projection output, pooled rows, codes, scales)."""
        side = int(round(np.sqrt(v["img_tok"])))
        n, dim, tdim = side * side, v["dim"], v["tdim"]
        out = np.empty((n, tdim), np.float32)
        pooled = np.empty((n, dim), np.float32)
        q = np.empty((n, dim), np.int8)
        s = np.empty(n, np.float32)
        rc = self.lib.ref_vision_head(_ptr(out, _f32p), _ptr(pooled, _f32p), _ptr(q, _i8p), _ptr(s, _f32p),
                                      _ptr(v["img"], _f32p), v["img_px"], v["psize"], dim, v["img_tok"], tdim,
                                      v["eps"], _ptr(v["pe"], _f32p), _ptr(v["pe_b"], _f32p), _ptr(v["pos_q"], _i8p),
                                      _ptr(v["pos_s"], _f32p), _ptr(v["post_n"], _f32p), _ptr(v["post_nb"], _f32p),
                                      _ptr(v["norm"], _f32p), _ptr(v["proj_q"], _i8p), _ptr(v["proj_s"], _f32p),
                                      self.threads)
        if rc:
            raise RuntimeError("reference forward_vision failed")
        return out, pooled, q, s

    def read_model_seconds(self, path: str, allow_mm: bool = True) -> float:
        """Seconds gemma.c's read_gemma_model takes to load the file."""
        t = self.lib.ref_read_model_seconds(path.encode(), int(allow_mm))
        if t < 0:
            raise RuntimeError(f"the reference refused {path}")
        return t

    def rmsnorm_quantize(self, x, w, eps):
        """gemma.c's rmsnorm on each row, then its quantize_acts."""
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        xn = np.empty_like(x)
        for i in range(x.shape[0]):
            self.lib.ref_rmsnorm(_ptr(xn[i], _f32p), _ptr(x[i], _f32p), _ptr(w, _f32p), x.shape[1], eps)
        q, s = self.quantize_acts(xn)
        return xn, q, s

    def geglu_quantize(self, gate, up):
        """gemma.c's gelu with `mul` (gate * up), then its quantize_acts."""
        gate = np.ascontiguousarray(gate, np.float32)
        up = np.ascontiguousarray(up, np.float32)
        h = np.empty_like(gate)
        self.lib.ref_gelu_mul(_ptr(h, _f32p), _ptr(gate, _f32p), _ptr(up, _f32p), gate.shape[0], gate.shape[1])
        q, s = self.quantize_acts(h)
        return h, q, s

    def gemv_int8(self, mat, matsc, vec, vsc, dst=None):
        mat = np.ascontiguousarray(mat, np.int8)
        m, n = mat.shape
        if dst is None:
            dst = np.empty(m, np.float32)
        self.lib.ref_gemv_int8(_ptr(dst, _f32p), _ptr(mat, _i8p), _ptr(np.ascontiguousarray(matsc, np.float32), _f32p),
                               _ptr(np.ascontiguousarray(vec, np.int8), _i8p), float(vsc), m, n, self.threads)
        return dst

    def gemv_int8_multi(self, mats, scs, vec, vsc, outs=None):
        vec = np.ascontiguousarray(vec, np.int8)
        if outs is None:
            outs = [np.empty(w.shape[0], np.float32) for w in mats]
        jobs = (GemvJob * len(mats))()
        for j, (w, s, o) in enumerate(zip(mats, scs, outs)):
            jobs[j] = GemvJob(w.ctypes.data, _ptr(s, _f32p), _ptr(o, _f32p), w.shape[0])
        self.lib.ref_gemv_int8_multi(jobs, len(mats), _ptr(vec, _i8p), float(vsc), vec.shape[0], self.threads)
        return outs

    def qkv_head_tasks(self, wq, sq, wk, sk, wv, sv, q, s, hdim, outs=None):
        """The prefill Q/K/V projections in gemma.c's own task split
        (gemma.c:5037-5091): per (head, 128-token block) gemm_int8 tasks
        over the OpenMP threads.  Returns xq, xk, xv head-major
        ([heads][ntok][hdim])."""
        q = np.ascontiguousarray(q, np.int8)
        ntok, dim = q.shape
        nh, nkv = wq.shape[0] // hdim, wk.shape[0] // hdim
        if outs is None:
            outs = [np.empty((h, ntok, hdim), np.float32) for h in (nh, nkv, nkv)]
        args = []
        for w, sc in ((wq, sq), (wk, sk), (wv, sv)):
            args += [_ptr(np.ascontiguousarray(w, np.int8), _i8p), _ptr(np.ascontiguousarray(sc, np.float32), _f32p)]
        rc = self.lib.ref_qkv_head_tasks(*[_ptr(o, _f32p) for o in outs], *args, _ptr(q, _i8p),
                                         _ptr(np.ascontiguousarray(s, np.float32), _f32p), ntok, dim, nh, nkv,
                                         hdim, self.threads)
        if rc:
            raise RuntimeError("reference gemm_int8 task failed")
        return outs

    def gemm_int8(self, mat, matsc, src, ssc, dst=None, dstr=0, mstr=0, sstr=0, m=None, n=None, k=None,
                  omp: bool = True):
        mat = np.ascontiguousarray(mat, np.int8)
        src = np.ascontiguousarray(src, np.int8)
        if m is None:
            m, k = src.shape
            n = mat.shape[0]
        if dst is None:
            dst = np.zeros((m, n), np.float32)
        rc = self.lib.ref_gemm_int8(_ptr(dst, _f32p), dstr, _ptr(mat, _i8p), mstr,
                                    _ptr(np.ascontiguousarray(matsc, np.float32), _f32p), _ptr(src, _i8p), sstr,
                                    _ptr(np.ascontiguousarray(ssc, np.float32), _f32p), m, n, k,
                                    self.threads if omp else 1)
        if rc != 0:
            raise RuntimeError("reference gemm_int8 returned %d" % rc)
        return dst
