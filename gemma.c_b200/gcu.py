"""Python host binding of libgcu.so (ctypes over the C ABI in include/gcu.h).

The functions mirror gemma.c's hot-path interface -- same names, same
argument meaning (gemma.c:2590 quantize_act, 2656 quantize_acts, 2770
gemv_int8, 2818 gemv_int8_multi, 3943 gemm_int8) -- on numpy host arrays,
plus ``dev_*`` variants on CUDA tensors (torch is only the allocator and
stream provider here).  There is no CPU fallback: importing this module
without a built libgcu.so raises, and calls fail loudly on error.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libgcu.so")

_i8p = ctypes.POINTER(ctypes.c_int8)
_f32p = ctypes.POINTER(ctypes.c_float)
_vp = ctypes.c_void_p
_int = ctypes.c_int


class GemvJob(ctypes.Structure):
    """gcu_gemv_job == gemma.c:2795 GemvJob (floatx = float)."""
    _fields_ = [("w", ctypes.c_void_p), ("sc", ctypes.c_void_p), ("dst", ctypes.c_void_p), ("m", ctypes.c_int)]


class QGemmStep(ctypes.Structure):
    """gcu_qgemm_step: one quantize_acts -> gemm_int8 step of a chain."""
    _fields_ = [("x", ctypes.c_void_p), ("xstr", ctypes.c_int), ("q", ctypes.c_void_p), ("s", ctypes.c_void_p),
                ("m", ctypes.c_int), ("k", ctypes.c_int), ("njobs", ctypes.c_int), ("jobs", GemvJob * 4)]


class QTensor(ctypes.Structure):
    """gcu_qtensor: one matmul weight of a model image (gemma.c:1102 QTensor
    plus its shape and which weight it is)."""
    _fields_ = [("q", ctypes.c_void_p), ("scales", ctypes.c_void_p), ("rows", ctypes.c_int),
                ("k", ctypes.c_int), ("kind", ctypes.c_int), ("layer", ctypes.c_int)]


# gcu_qt_kind
QT_KINDS = ("lm_head", "wq", "wk", "wv", "wo", "w1", "w2", "w3",
            "vwq", "vwk", "vwv", "vwo", "vw1", "vw2", "vproj")


class GcuError(RuntimeError):
    pass


# every symbol include/gcu.h declares, with (restype, argtypes)
SIGNATURES = {
    "gcu_init": (_int, [_int]),
    "gcu_shutdown": (_int, []),
    "gcu_last_error": (ctypes.c_char_p, []),
    "gcu_check_device": (_int, []),
    "gcu_version": (ctypes.c_char_p, []),
    "gcu_register_weight": (_int, [_vp, _vp, _int, _int]),
    "gcu_unregister_weight": (_int, [_vp]),
    "gcu_registered_bytes": (ctypes.c_size_t, []),
    "gcu_bin_qtensors": (_int, [_vp, ctypes.c_size_t, _int, ctypes.POINTER(QTensor), _int]),
    "gcu_register_qtensors": (_int, [ctypes.POINTER(QTensor), _int, ctypes.POINTER(_int)]),
    "gcu_register_model": (_int, [_vp, ctypes.c_size_t, _int, ctypes.POINTER(_int)]),
    "gcu_unregister_arena": (_int, [_int]),
    "gcu_quantize_act": (ctypes.c_float, [_vp, _vp, _int]),
    "gcu_quantize_acts": (_int, [_vp, _vp, _vp, _int, _int, _int]),
    "gcu_gemv_int8": (_int, [_vp, _vp, _vp, _vp, ctypes.c_float, _int, _int]),
    "gcu_gemv_int8_multi": (_int, [ctypes.POINTER(GemvJob), _int, _vp, ctypes.c_float, _int]),
    "gcu_gemm_int8": (_int, [_vp, _int, _vp, _int, _vp, _vp, _int, _vp, _int, _int, _int]),
    "gcu_dev_quantize_acts": (_int, [_vp, _vp, _vp, _int, _int, _int, _vp]),
    "gcu_dev_gemv_int8": (_int, [_vp, _vp, _vp, _vp, _vp, _int, _int, _vp]),
    "gcu_dev_gemv_int8_multi": (_int, [ctypes.POINTER(GemvJob), _int, _vp, _vp, _int, _vp]),
    "gcu_dev_gemm_int8": (_int, [_vp, _int, _vp, _int, _vp, _vp, _int, _vp, _int, _int, _int, _vp]),
    "gcu_dev_gemm_int8_multi": (_int, [ctypes.POINTER(GemvJob), _int, _vp, _int, _vp, _int, _int, _vp]),
    "gcu_dev_gemm_int8_noalloc": (_int, [_vp, _int, _vp, _int, _vp, _vp, _int, _vp, _int, _int, _int, _vp]),
    "gcu_dev_quantize_gemm_int8_multi": (_int, [ctypes.POINTER(GemvJob), _int, _vp, _vp, _vp, _int, _int, _int,
                                                _vp]),
    "gcu_gemm_chain_create": (_int, [ctypes.POINTER(QGemmStep), _int, ctypes.POINTER(_int), ctypes.POINTER(_int)]),
    "gcu_gemm_chain_run": (_int, [_int, _vp]),
    "gcu_gemm_chain_plan": (_int, [_int, ctypes.POINTER(_int), _int]),
    "gcu_gemm_chain_destroy": (_int, [_int]),
    "gcu_dev_ffn_rowshard": (_int, [_vp, _vp, _vp, _int, _int, _int, _vp, _vp, _vp, _vp, _vp, _int, _vp, _vp]),
    "gcu_comm_unique_id": (_int, [ctypes.c_char_p]),
    "gcu_comm_init": (_int, [_int, _int, ctypes.c_char_p]),
    "gcu_comm_destroy": (_int, []),
    "gcu_comm_fused_allgather": (_int, []),
    "gcu_dev_gemm_int8_rowshard": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _int, _int, _int, _vp]),
    "gcu_dev_quantize_gemm_int8_rowshard_multi": (_int, [ctypes.POINTER(GemvJob), _int, _vp, _vp, _vp, _int,
                                                         _int, _int, _vp, _vp]),
    "gcu_dev_rmsnorm_quantize": (_int, [_vp, _vp, _vp, _vp, _int, _vp, ctypes.c_float, _int, _int, _vp]),
    "gcu_dev_geglu_quantize": (_int, [_vp, _vp, _vp, _vp, _vp, _int, _int, _vp]),
    "gcu_dev_attention_decode": (_int, [_vp, _vp, _vp, _vp, ctypes.c_long, _int, _int, _int, _int, _int,
                                        ctypes.c_float, ctypes.c_float, _vp]),
    "gcu_dev_attention_prefill": (_int, [_vp, _int, _vp, _vp, _vp, ctypes.c_long, _int, _int, _int, _int, _int,
                                         _int, ctypes.c_float, _int, _vp]),
    "gcu_dev_attention_decode_rope": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_long, _vp, _vp, ctypes.c_float,
                                             _vp, _int, _int, _int, _int, _int, ctypes.c_float, ctypes.c_float, _vp]),
    "gcu_dev_rmsnorm_residual": (_int, [_vp, _vp, _vp, _vp, ctypes.c_float, _int, _int, _vp]),
    "gcu_dev_softcap": (_int, [_vp, ctypes.c_long, ctypes.c_float, _vp]),
    "gcu_dev_residual_norm_quantize": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_float, _int, _int, _vp]),
    "gcu_dev_geglu_quantize_gemv_multi": (_int, [ctypes.POINTER(GemvJob), _int, _vp, _vp, _vp, _vp, _int, _vp]),
    "gcu_dev_residual_norm_quantize_gemv_multi": (_int, [ctypes.POINTER(GemvJob), _int, _vp, _vp, _vp, _vp, _vp,
                                                         _vp, _vp, ctypes.c_float, _int, _vp]),
    "gcu_dev_qk_norm_rope_cache": (_int, [_vp, _vp, _vp, _vp, _vp, ctypes.c_long, _vp, _vp, ctypes.c_float, _vp,
                                          ctypes.c_float, _int, _int, _int, _int, _int, _vp]),
    "gcu_dev_qkv_norm_rope_cache": (_int, [_vp, _vp, ctypes.c_long, _vp, _vp, ctypes.c_long, _vp, _vp, ctypes.c_float,
                                           _vp, ctypes.c_float, _int, _int, _int, _int, _int, _vp]),
    "gcu_dev_patch_embed": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _int, _int, _int, _vp]),
    "gcu_dev_vision_pool_quantize": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_float, _int, _int, _int,
                                            _vp]),
}
# exported but not part of the public header (benchmark sweeps, self-test)
EXTRA = {
    "gcu_selftest_bounded_wait": (_int, [_int, _int, ctypes.POINTER(ctypes.c_ulonglong), _vp]),
    "gcu_dev_gemm_int8_multi_tuned": (_int, [ctypes.POINTER(GemvJob), _int, _vp, _int, _vp, _int, _int, _int,
                                             _int, _int, _vp]),
    "gcu_dev_gemm_int8_tuned": (_int, [_vp, _int, _vp, _int, _vp, _vp, _int, _vp, _int, _int, _int,
                                       _int, _int, _int, _vp]),
    "gcu_dev_gemm_int8_raw_tuned": (_int, [_vp, _vp, _vp, _int, _int, _int, _int, _int, _int, _vp]),
    "gcu_dev_gemm_int8_noalloc_tuned": (_int, [_vp, _int, _vp, _int, _vp, _vp, _int, _vp, _int, _int,
                                               _int, _int, _int, _int, _vp]),
}


def build() -> None:
    """Compile libgcu.so in-tree (nvcc, sm_100a)."""
    subprocess.run(["make", "-s", "-C", HERE, "-j4"], check=True)


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise GcuError(f"libgcu.so not built ({LIB_PATH}); run make -C gemma.c_b200")
        l = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in {**SIGNATURES, **EXTRA}.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise GcuError(f"{what}: {lib().gcu_last_error().decode()}")


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def init(device: int = 0) -> None:
    _check(lib().gcu_init(device), "gcu_init")


def shutdown() -> None:
    _check(lib().gcu_shutdown(), "gcu_shutdown")


def check_device() -> None:
    _check(lib().gcu_check_device(), "device")


def selftest_bounded_wait(mode: int, budget_us: int, stream=None) -> int:
    """Run one device-side wait (mode 0: an mbarrier, 1: a global flag) on
    something that never completes, with a budget of `budget_us`; returns the
    nanoseconds the kernel waited.  Leaves the timeout code in the device error
    word for the next check to report."""
    ns = ctypes.c_ulonglong(0)
    _check(lib().gcu_selftest_bounded_wait(mode, budget_us, ctypes.byref(ns), _stream(stream)),
           "selftest_bounded_wait")
    return ns.value


def register_weight(q: np.ndarray, scales: np.ndarray) -> None:
    """Upload a QTensor (int8 [rows][k] + fp32 [rows]) once; the arrays must
    stay alive and unchanged while registered."""
    assert q.dtype == np.int8 and q.ndim == 2 and q.flags["C_CONTIGUOUS"]
    assert scales.dtype == np.float32 and scales.shape == (q.shape[0],)
    _check(lib().gcu_register_weight(_p(q), _p(scales), q.shape[0], q.shape[1]), "register_weight")


def unregister_weight(q: np.ndarray) -> None:
    _check(lib().gcu_unregister_weight(_p(q)), "unregister_weight")


def bin_qtensors(image: np.ndarray, allow_mm: bool = True) -> list[dict]:
    """The matmul QTensors of a `-q` model image (uint8 array): kind, layer,
    rows, k and the BYTE OFFSETS of the int8 values and scales in the image.
    Host only."""
    assert image.dtype == np.uint8 and image.flags["C_CONTIGUOUS"]
    n = lib().gcu_bin_qtensors(_p(image), image.nbytes, int(allow_mm), None, 0)
    if n < 0:
        raise GcuError(f"bin_qtensors: {lib().gcu_last_error().decode()}")
    recs = (QTensor * max(n, 1))()
    lib().gcu_bin_qtensors(_p(image), image.nbytes, int(allow_mm), recs, n)
    base = _p(image)
    return [{"kind": QT_KINDS[r.kind], "layer": r.layer, "rows": r.rows, "k": r.k,
             "q_off": r.q - base, "s_off": r.scales - base} for r in recs[:n]]


def register_model(image: np.ndarray, allow_mm: bool = True) -> int:
    """Upload every matmul weight of a model image as one arena; returns its
    handle.  The image must stay alive and unchanged while registered."""
    assert image.dtype == np.uint8 and image.flags["C_CONTIGUOUS"]
    arena = _int(0)
    _check(lib().gcu_register_model(_p(image), image.nbytes, int(allow_mm), ctypes.byref(arena)),
           "register_model")
    return arena.value


def register_qtensors(tensors) -> int:
    """Upload (q, scales) pairs of numpy arrays as one arena; returns its handle."""
    recs = (QTensor * len(tensors))()
    for r, (q, sc) in zip(recs, tensors):
        assert q.dtype == np.int8 and q.ndim == 2 and q.flags["C_CONTIGUOUS"]
        assert sc.dtype == np.float32 and sc.shape == (q.shape[0],)
        r.q, r.scales, r.rows, r.k, r.kind, r.layer = _p(q), _p(sc), q.shape[0], q.shape[1], 0, -1
    arena = _int(0)
    _check(lib().gcu_register_qtensors(recs, len(tensors), ctypes.byref(arena)), "register_qtensors")
    return arena.value


def unregister_arena(arena: int) -> None:
    _check(lib().gcu_unregister_arena(arena), "unregister_arena")


def registered_bytes() -> int:
    return lib().gcu_registered_bytes()


# --------------------------------------------------------------------------
# host-pointer API (gemma.c semantics; numpy in, numpy out)
# --------------------------------------------------------------------------

def quantize_act(vec: np.ndarray):
    """gemma.c:2590 -> (int8 codes, fp32 scale)."""
    vec = np.ascontiguousarray(vec, np.float32)
    dst = np.empty(vec.shape[0], np.int8)
    sc = lib().gcu_quantize_act(_p(dst), _p(vec), vec.shape[0])
    if np.isnan(sc):
        raise GcuError("quantize_act: " + lib().gcu_last_error().decode())
    return dst, np.float32(sc)


def quantize_acts(src: np.ndarray, n: int | None = None, sstr: int = 0, dst=None, dsc=None):
    """gemma.c:2656 on an (m, sstr) fp32 array -> int8 (m, n), fp32 (m,);
    dst / dsc: optional output arrays (for instance views of pinned memory)."""
    src = np.ascontiguousarray(src, np.float32)
    m = src.shape[0]
    n = src.shape[1] if n is None else n
    if dst is None:
        dst = np.empty((m, n), np.int8)
    if dsc is None:
        dsc = np.empty(m, np.float32)
    _check(lib().gcu_quantize_acts(_p(dst), _p(dsc), _p(src), sstr, m, n), "quantize_acts")
    return dst, dsc


def gemv_int8(mat, matsc, vec, vsc, dst=None):
    """gemma.c:2770: mat (m, n) int8, returns fp32 (m,)."""
    m, n = mat.shape
    if dst is None:
        dst = np.empty(m, np.float32)
    _check(lib().gcu_gemv_int8(_p(dst), _p(mat), _p(matsc), _p(vec), float(vsc), m, n), "gemv_int8")
    return dst


def gemv_int8_multi(mats, scs, vec, vsc, outs=None):
    """gemma.c:2818: several (rows_j, n) weights sharing vec."""
    if outs is None:
        outs = [np.empty(w.shape[0], np.float32) for w in mats]
    jobs = (GemvJob * len(mats))()
    for j, (w, s, o) in enumerate(zip(mats, scs, outs)):
        jobs[j] = GemvJob(_p(w), _p(s), _p(o), w.shape[0])
    _check(lib().gcu_gemv_int8_multi(jobs, len(mats), _p(vec), float(vsc), vec.shape[0]), "gemv_int8_multi")
    return outs


def gemm_int8(mat, matsc, src, ssc, dst=None, dstr=0, mstr=0, sstr=0, m=None, n=None, k=None):
    """gemma.c:3943 NT GEMM; with strides, pass flat buffers and m, n, k."""
    if m is None:
        m, k = src.shape
        n = mat.shape[0]
    if dst is None:
        dst = np.zeros((m, n), np.float32)
    _check(lib().gcu_gemm_int8(_p(dst), dstr, _p(mat), mstr, _p(matsc), _p(src), sstr, _p(ssc), m, n, k),
           "gemm_int8")
    return dst


# --------------------------------------------------------------------------
# device-pointer API on torch CUDA tensors (enqueued on torch's current stream)
# --------------------------------------------------------------------------

def _stream(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def dev_quantize_acts(dst, dsc, src, m, n, sstr=0, stream=None):
    _check(lib().gcu_dev_quantize_acts(dst.data_ptr(), dsc.data_ptr(), src.data_ptr(), sstr, m, n,
                                       _stream(stream)), "dev_quantize_acts")


def dev_gemv_int8(dst, mat, matsc, vec, vsc, m, n, stream=None):
    _check(lib().gcu_dev_gemv_int8(dst.data_ptr(), mat.data_ptr(), matsc.data_ptr(), vec.data_ptr(),
                                   vsc.data_ptr(), m, n, _stream(stream)), "dev_gemv_int8")


def dev_gemv_int8_multi(jobs_t, vec, vsc, n, stream=None):
    """jobs_t: list of (w, sc, dst) device tensors."""
    jobs = (GemvJob * len(jobs_t))()
    for j, (w, s, o) in enumerate(jobs_t):
        jobs[j] = GemvJob(w.data_ptr(), s.data_ptr(), o.data_ptr(), w.shape[0])
    _check(lib().gcu_dev_gemv_int8_multi(jobs, len(jobs_t), vec.data_ptr(), vsc.data_ptr(), n,
                                         _stream(stream)), "dev_gemv_int8_multi")


def dev_gemm_int8(dst, mat, matsc, src, ssc, m, n, k, dstr=0, mstr=0, sstr=0, stream=None):
    _check(lib().gcu_dev_gemm_int8(dst.data_ptr(), dstr, mat.data_ptr(), mstr, matsc.data_ptr(),
                                   src.data_ptr(), sstr, ssc.data_ptr(), m, n, k, _stream(stream)),
           "dev_gemm_int8")


def dev_quantize_gemm_int8_multi(jobs_t, q, s, x, m, k, xstr=0, stream=None):
    """quantize_acts(x) -> (q, s) and every job's gemm_int8 on it, in one launch.
    jobs_t: list of (w, sc, dst) device tensors."""
    jobs = (GemvJob * len(jobs_t))()
    for j, (w, sc, o) in enumerate(jobs_t):
        jobs[j] = GemvJob(w.data_ptr(), sc.data_ptr(), o.data_ptr(), w.shape[0])
    _check(lib().gcu_dev_quantize_gemm_int8_multi(jobs, len(jobs_t), q.data_ptr(), s.data_ptr(), x.data_ptr(),
                                                  xstr, m, k, _stream(stream)), "dev_quantize_gemm_int8_multi")


def dev_gemm_int8_noalloc(dst, mat, matsc, src, ssc, m, n, k, dstr=0, mstr=0, sstr=0, stream=None):
    """gemm_int8 on device tensors with no device allocation: split-K scratch
    comes from a fixed array inside libgcu.so (see include/gcu.h)."""
    _check(lib().gcu_dev_gemm_int8_noalloc(dst.data_ptr(), dstr, mat.data_ptr(), mstr, matsc.data_ptr(),
                                           src.data_ptr(), sstr, ssc.data_ptr(), m, n, k, _stream(stream)),
           "dev_gemm_int8_noalloc")


def dev_gemm_int8_multi(jobs_t, src, ssc, m, k, sstr=0, stream=None):
    jobs = (GemvJob * len(jobs_t))()
    for j, (w, s, o) in enumerate(jobs_t):
        jobs[j] = GemvJob(w.data_ptr(), s.data_ptr(), o.data_ptr(), w.shape[0])
    _check(lib().gcu_dev_gemm_int8_multi(jobs, len(jobs_t), src.data_ptr(), sstr, ssc.data_ptr(), m, k,
                                         _stream(stream)), "dev_gemm_int8_multi")


def dev_gemm_int8_tuned(dst, mat, matsc, src, ssc, m, n, k, bn, split, mb=1, stream=None):
    """Force the tile shape ((128*mb) x bn) and K split (benchmark sweeps)."""
    _check(lib().gcu_dev_gemm_int8_tuned(dst.data_ptr(), 0, mat.data_ptr(), 0, matsc.data_ptr(),
                                         src.data_ptr(), 0, ssc.data_ptr(), m, n, k, bn, split, mb,
                                         _stream(stream)), "dev_gemm_int8_tuned")


def dev_gemm_int8_noalloc_tuned(dst, mat, matsc, src, ssc, m, n, k, bn, split, mb=1, stream=None):
    """dev_gemm_int8_noalloc with a forced tile shape and K split (tests)."""
    _check(lib().gcu_dev_gemm_int8_noalloc_tuned(dst.data_ptr(), 0, mat.data_ptr(), 0, matsc.data_ptr(),
                                                 src.data_ptr(), 0, ssc.data_ptr(), m, n, k, bn, split, mb,
                                                 _stream(stream)), "dev_gemm_int8_noalloc_tuned")


def dev_gemm_int8_multi_tuned(jobs_t, src, ssc, m, k, bn, split, mb=1, stream=None):
    """Multi-job GEMM with a forced tile shape and K split (benchmark sweeps)."""
    jobs = (GemvJob * len(jobs_t))()
    for j, (w, s, o) in enumerate(jobs_t):
        jobs[j] = GemvJob(w.data_ptr(), s.data_ptr(), o.data_ptr(), w.shape[0])
    _check(lib().gcu_dev_gemm_int8_multi_tuned(jobs, len(jobs_t), src.data_ptr(), 0, ssc.data_ptr(), m, k, bn,
                                               split, mb, _stream(stream)), "dev_gemm_int8_multi_tuned")


class GemmChain:
    """A chain of quantize_acts -> gemm_int8 steps run as one launch
    (gcu_gemm_chain_*).  steps: list of (x, q, s, jobs) with device tensors
    x [m][k] fp32, q [m][k] int8, s [m] fp32 and jobs [(w, sc, dst), ...];
    force: None or per step (bn, mb, splits)."""

    def __init__(self, steps, force=None):
        self.handle = 0
        arr = (QGemmStep * len(steps))()
        for i, (x, q, s, jobs) in enumerate(steps):
            st = arr[i]
            st.x, st.xstr, st.q, st.s = x.data_ptr(), 0, q.data_ptr(), s.data_ptr()
            st.m, st.k, st.njobs = x.shape[0], x.shape[1], len(jobs)
            for j, (w, sc, o) in enumerate(jobs[:4]):  # more than 4: the library refuses njobs
                st.jobs[j] = GemvJob(w.data_ptr(), sc.data_ptr(), o.data_ptr(), w.shape[0])
        self._keep = steps
        self.n = len(steps)
        f = None
        if force is not None:
            f = (_int * (3 * len(steps)))(*[v for t in force for v in t])
        h = _int(0)
        _check(lib().gcu_gemm_chain_create(arr, len(steps), f, ctypes.byref(h)), "gemm_chain_create")
        self.handle = h.value

    def run(self, stream=None):
        _check(lib().gcu_gemm_chain_run(self.handle, _stream(stream)), "gemm_chain_run")

    def plan(self):
        out = (_int * (3 * self.n))()
        _check(lib().gcu_gemm_chain_plan(self.handle, out, self.n), "gemm_chain_plan")
        return [tuple(out[3 * i:3 * i + 3]) for i in range(self.n)]

    def close(self):
        if self.handle:
            _check(lib().gcu_gemm_chain_destroy(self.handle), "gemm_chain_destroy")
            self.handle = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def dev_ffn_rowshard(out, xq, xs, m, dim, ffn, w_up, s_up, w_gate, s_gate, w_down, s_down, w_down_stride=0,
                     stream=None):
    """Gemma's FFN (up, gate, GeGLU, quantize, down) with the hidden dimension
    split over the ranks of comm_init; unsharded without it."""
    _check(lib().gcu_dev_ffn_rowshard(out.data_ptr(), xq.data_ptr(), xs.data_ptr(), m, dim, ffn, w_up.data_ptr(),
                                      s_up.data_ptr(), w_gate.data_ptr(), s_gate.data_ptr(), w_down.data_ptr(),
                                      w_down_stride, s_down.data_ptr(), _stream(stream)), "dev_ffn_rowshard")


def dev_gemm_int8_raw_tuned(dst, mat, src, m, n, k, bn=0, split=0, mb=0, stream=None):
    """The int32 sums of gemm_int8 (dst: int32 tensor), forced tile shape (tests)."""
    _check(lib().gcu_dev_gemm_int8_raw_tuned(dst.data_ptr(), mat.data_ptr(), src.data_ptr(), m, n, k, bn, split, mb,
                                             _stream(stream)), "dev_gemm_int8_raw_tuned")


def comm_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    _check(lib().gcu_comm_unique_id(buf), "comm_unique_id")
    return buf.raw


def comm_init(rank: int, world: int, uid: bytes) -> None:
    _check(lib().gcu_comm_init(rank, world, uid), "comm_init")


def comm_fused_allgather() -> bool:
    return bool(lib().gcu_comm_fused_allgather())


def comm_destroy() -> None:
    _check(lib().gcu_comm_destroy(), "comm_destroy")


def dev_gemm_int8_rowshard(dst, work, mat_local, matsc_local, src, ssc, m, n, k, stream=None):
    _check(lib().gcu_dev_gemm_int8_rowshard(dst.data_ptr(), work.data_ptr(), mat_local.data_ptr(),
                                            matsc_local.data_ptr(), src.data_ptr(), ssc.data_ptr(),
                                            m, n, k, _stream(stream)), "dev_gemm_int8_rowshard")


def dev_quantize_gemm_int8_rowshard_multi(jobs_t, q, s, x, m, k, work=None, xstr=0, stream=None):
    """quantize_acts(x) -> (q, s) and the row-sharded GEMM of every job on it.
    jobs_t: list of (w_local, sc_local, dst, rows) with rows the FULL row count."""
    jobs = (GemvJob * len(jobs_t))()
    for j, (w, sc, o, rows) in enumerate(jobs_t):
        jobs[j] = GemvJob(w.data_ptr(), sc.data_ptr(), o.data_ptr(), rows)
    _check(lib().gcu_dev_quantize_gemm_int8_rowshard_multi(jobs, len(jobs_t), q.data_ptr(), s.data_ptr(),
                                                           x.data_ptr(), xstr, m, k,
                                                           work.data_ptr() if work is not None else None,
                                                           _stream(stream)),
           "dev_quantize_gemm_int8_rowshard_multi")


def dev_rmsnorm_quantize(q, s, x, weight, eps, m, dim, out=None, xstr=0, stream=None):
    """gemma.c's rmsnorm then quantize_acts, fused: codes -> q, scales -> s,
    the normalized rows -> out (optional)."""
    _check(lib().gcu_dev_rmsnorm_quantize(q.data_ptr(), s.data_ptr(), out.data_ptr() if out is not None else None,
                                          x.data_ptr(), xstr, weight.data_ptr(), float(eps), m, dim,
                                          _stream(stream)), "dev_rmsnorm_quantize")


def dev_geglu_quantize(q, s, gate, up, m, dim, out=None, stream=None):
    """gemma.c's gelu(gate) * up then quantize_acts, fused."""
    _check(lib().gcu_dev_geglu_quantize(q.data_ptr(), s.data_ptr(), out.data_ptr() if out is not None else None,
                                        gate.data_ptr(), up.data_ptr(), m, dim, _stream(stream)),
           "dev_geglu_quantize")


def dev_attention_decode(xo, xq, kc, vc, spos, attlen, asc, sc_att=0.0, stream=None):
    """gemma.c:4836-4848 on CUDA tensors: xq (n_heads, hdim); kc, vc
    (nkv, clen, hdim) caches; writes xo (n_heads, hdim)."""
    n_heads, hdim = xq.shape
    nkv, clen, _ = kc.shape
    _check(lib().gcu_dev_attention_decode(xo.data_ptr(), xq.data_ptr(), kc.data_ptr(), vc.data_ptr(), clen * hdim,
                                          n_heads, nkv, hdim, spos, attlen, asc, sc_att, _stream(stream)),
           "dev_attention_decode")


def dev_attention_decode_rope(xo, xq, xk, xv, kc, vc, freqs, spos, attlen, asc, sc_att=0.0, nq=None, nk=None,
                              eps=1e-6, stream=None):
    """dev_qk_norm_rope_cache at position spos + attlen - 1 and
    dev_attention_decode in one launch: xq (n_heads, hdim), xk / xv (nkv,
    hdim) as the Q/K/V GEMVs wrote them; kc, vc (nkv, clen, hdim); freqs the
    position's (hdim,) table.  xq is not rotated in place."""
    n_heads, hdim = xq.shape[-2], xq.shape[-1]
    nkv, clen, _ = kc.shape
    _check(lib().gcu_dev_attention_decode_rope(xo.data_ptr(), xq.data_ptr(), xk.data_ptr(), xv.data_ptr(),
                                               kc.data_ptr(), vc.data_ptr(), clen * hdim,
                                               nq.data_ptr() if nq is not None else None,
                                               nk.data_ptr() if nk is not None else None, eps, freqs.data_ptr(),
                                               n_heads, nkv, hdim, spos, attlen, asc, sc_att, _stream(stream)),
           "dev_attention_decode_rope")


def dev_attention_prefill(xo, xq, kc, vc, spos, slide=0, sc_att=0.0, mask=True, xostr=0, stream=None):
    """gemma.c:5160-5295 on CUDA tensors: xq (n_heads, ntok, hdim) rotated and
    scaled; kc, vc (nkv, clen, hdim) holding the chunk at [spos, spos+ntok);
    writes xo rows (ntok, >= n_heads*hdim)."""
    n_heads, ntok, hdim = xq.shape
    nkv, clen, _ = kc.shape
    _check(lib().gcu_dev_attention_prefill(xo.data_ptr(), xostr, xq.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                           clen * hdim, n_heads, nkv, hdim, spos, ntok, slide, sc_att, int(mask),
                                           _stream(stream)),
           "dev_attention_prefill")


def dev_patch_embed(x, img, pe, pe_b, pos_q, pos_s, img_px, psize, dim, stream=None):
    """gemma.c:4411-4466 on CUDA tensors: x (npatch, dim) from the image
    (img_px, img_px, 3), pe (dim, 3, psize, psize), pe_b and the int8
    position embedding (pos_q, pos_s)."""
    _check(lib().gcu_dev_patch_embed(x.data_ptr(), img.data_ptr(), pe.data_ptr(), pe_b.data_ptr(), pos_q.data_ptr(),
                                     pos_s.data_ptr(), img_px, psize, dim, _stream(stream)), "dev_patch_embed")


def dev_vision_pool_quantize(q, s, x, post_n, post_nb, norm, eps, ppi, side, dim, out=None, stream=None):
    """gemma.c:4660-4705 + 4714 on CUDA tensors: codes q (side*side, dim),
    scales s, optional fp32 rows out, from the patch rows x (ppi*ppi, dim)."""
    _check(lib().gcu_dev_vision_pool_quantize(q.data_ptr(), s.data_ptr(), out.data_ptr() if out is not None else None,
                                              x.data_ptr(), post_n.data_ptr(), post_nb.data_ptr(), norm.data_ptr(),
                                              eps, ppi, side, dim, _stream(stream)), "dev_vision_pool_quantize")


def dev_qk_norm_rope_cache(xq, xk, xv, kc, vc, freqs, spos, q_scale=1.0, nq=None, nk=None, eps=1e-6, stream=None):
    """gemma.c:4775-4818 / 5095-5145 on CUDA tensors: xq (n_heads, ntok, hdim)
    rotated in place; xk, xv (nkv, ntok, hdim) normed/rotated keys and the
    values written into kc, vc (nkv, clen, hdim) at [spos, spos+ntok);
    freqs (ntok, hdim)."""
    n_heads, ntok, hdim = xq.shape
    nkv, clen, _ = kc.shape
    _check(lib().gcu_dev_qk_norm_rope_cache(xq.data_ptr(), xk.data_ptr(), xv.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                            clen * hdim, nq.data_ptr() if nq is not None else None,
                                            nk.data_ptr() if nk is not None else None, eps, freqs.data_ptr(),
                                            q_scale, n_heads, nkv, hdim, spos, ntok, _stream(stream)),
           "dev_qk_norm_rope_cache")


def dev_rmsnorm_residual(x, y, resid, weight, eps, m, dim, stream=None):
    """gemma.c:4862-4881 / 4950-4962 on CUDA tensors: x = clamp(resid + rmsnorm(y, weight)),
    weight None = no post-norm."""
    _check(lib().gcu_dev_rmsnorm_residual(x.data_ptr(), y.data_ptr(), resid.data_ptr(),
                                          weight.data_ptr() if weight is not None else None, eps, m, dim,
                                          _stream(stream)), "dev_rmsnorm_residual")


def dev_softcap(x, cap, stream=None):
    """gemma.c:4971-4976 on a CUDA tensor, in place."""
    _check(lib().gcu_dev_softcap(x.data_ptr(), x.numel(), cap, _stream(stream)), "dev_softcap")


def dev_residual_norm_quantize(x, q, s, y, resid, w_post, w_next, eps, m, dim, stream=None):
    """x = clamp(resid + rmsnorm(y, w_post)); q, s = quantize(rmsnorm(x, w_next)), one launch."""
    _check(lib().gcu_dev_residual_norm_quantize(x.data_ptr(), q.data_ptr(), s.data_ptr(), y.data_ptr(),
                                                resid.data_ptr(), w_post.data_ptr() if w_post is not None else None,
                                                w_next.data_ptr(), eps, m, dim, _stream(stream)),
           "dev_residual_norm_quantize")


def _gemv_jobs(jobs_t):
    jobs = (GemvJob * len(jobs_t))()
    for j, (w, sc, o) in enumerate(jobs_t):
        jobs[j] = GemvJob(w.data_ptr(), sc.data_ptr(), o.data_ptr(), w.shape[0])
    return jobs


def dev_geglu_quantize_gemv_multi(jobs_t, q, s, gate, up, k, stream=None):
    """One token: h = gelu(gate) * up quantized into (q, s) and every job's
    GEMV on it, in one launch.  jobs_t: list of (w, sc, dst) device tensors."""
    jobs = _gemv_jobs(jobs_t)
    _check(lib().gcu_dev_geglu_quantize_gemv_multi(jobs, len(jobs_t), q.data_ptr(), s.data_ptr(), gate.data_ptr(),
                                                   up.data_ptr(), k, _stream(stream)), "dev_geglu_quantize_gemv_multi")


def dev_residual_norm_quantize_gemv_multi(jobs_t, x, q, s, y, resid, w_post, w_next, eps, dim, stream=None):
    """One token: x = clamp(resid + rmsnorm(y, w_post)), then rmsnorm(x, w_next)
    quantized into (q, s) and every job's GEMV on it, in one launch.  x must
    be a buffer other than resid and y."""
    jobs = _gemv_jobs(jobs_t)
    _check(lib().gcu_dev_residual_norm_quantize_gemv_multi(
        jobs, len(jobs_t), x.data_ptr(), q.data_ptr(), s.data_ptr(), y.data_ptr(), resid.data_ptr(),
        w_post.data_ptr() if w_post is not None else None, w_next.data_ptr(), eps, dim, _stream(stream)),
        "dev_residual_norm_quantize_gemv_multi")


def dev_qkv_norm_rope_cache(xq, qkv, kc, vc, freqs, spos, n_heads, q_scale=1.0, nq=None, nk=None, eps=1e-6,
                            stream=None):
    """Token-major variant: qkv (ntok, >= (n_heads+2*nkv)*hdim) rows of the fused
    projection; rotated queries to xq (n_heads, ntok, hdim), keys/values to the
    caches kc, vc (nkv, clen, hdim)."""
    nkv, clen, hdim = kc.shape
    ntok = qkv.shape[0]
    _check(lib().gcu_dev_qkv_norm_rope_cache(xq.data_ptr(), qkv.data_ptr(), qkv.stride(0), kc.data_ptr(),
                                             vc.data_ptr(), clen * hdim, nq.data_ptr() if nq is not None else None,
                                             nk.data_ptr() if nk is not None else None, eps, freqs.data_ptr(),
                                             q_scale, n_heads, nkv, hdim, spos, ntok, _stream(stream)),
           "dev_qkv_norm_rope_cache")
