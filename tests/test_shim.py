"""The reference-side drop-in header gemma.c_b200/host/gemma_gcu.h: the five
gemma.c hot-path functions with their exact static signatures, compiled in a
gemma.c-like context (tests/shim/shim_harness.c) and called like gemma.c's
forward passes call them."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

import gcu
import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CC = "/usr/bin/gcc" if os.path.exists("/usr/bin/gcc") else "gcc"


@pytest.fixture(scope="module")
def shim(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("shim") / "libshim.so")
    pkg = os.path.join(ROOT, "gemma.c_b200")
    subprocess.run([CC, "-std=gnu11", "-O2", "-Wall", "-Werror", "-fPIC", "-shared",
                    "-I", os.path.join(ROOT, "include"), "-I", os.path.join(pkg, "host"),
                    os.path.join(ROOT, "tests", "shim", "shim_harness.c"), "-o", out,
                    "-L", pkg, "-lgcu", f"-Wl,-rpath,{pkg}"], check=True)
    lib = ctypes.CDLL(out)
    lib.shim_quantize_act.restype = ctypes.c_float
    lib.shim_quantize_act.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    lib.shim_gemv_int8.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_float, ctypes.c_int, ctypes.c_int]
    lib.shim_gemv_int8_multi.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_float,
                                         ctypes.c_int]
    lib.shim_gemm_int8.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                   ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_int]
    lib.shim_error.restype = ctypes.c_char_p
    lib.shim_perf_count.restype = ctypes.c_long
    return lib


def test_shim_compiles_and_exports(shim):
    for name in ("shim_quantize_act", "shim_quantize_acts", "shim_gemv_int8", "shim_gemv_int8_multi",
                 "shim_gemm_int8", "shim_register"):
        assert hasattr(shim, name)


def test_shim_error_convention_without_device(shim):
    # gemm_int8 with k <= 0 fails before touching a GPU: returns 1 and sets
    # the thread's error text like gemma.c:3977-3982
    d = np.zeros(4, np.float32)
    a = np.zeros(4, np.int8)
    rc = shim.shim_gemm_int8(d.ctypes.data, 0, a.ctypes.data, 0, d.ctypes.data, a.ctypes.data, 0,
                             d.ctypes.data, 1, 1, 0)
    assert rc == 1
    assert shim.shim_error().startswith(b"cuda gemm_int8:")


@pytest.mark.gpu
def test_shim_matches_reference_golden(shim, golden):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    bits = lambda a: np.ascontiguousarray(a, np.float32).view(np.uint32)
    # quantize_act (decode) and quantize_acts (prefill)
    v = golden["quant_c_x"]
    q = np.empty(v.shape[0], np.int8)
    sc = shim.shim_quantize_act(q.ctypes.data, v.ctypes.data, v.shape[0])
    assert np.array_equal(q, golden["quant_c_q"]) and np.float32(sc) == golden["quant_c_s"]
    x = golden["quant_a_x"]
    qa = np.empty(x.shape, np.int8)
    sa = np.empty(x.shape[0], np.float32)
    shim.shim_quantize_acts(qa.ctypes.data, sa.ctypes.data, x.ctypes.data, 0, x.shape[0], x.shape[1])
    assert np.array_equal(qa, golden["quant_a_q"]) and np.array_equal(bits(sa), bits(golden["quant_a_s"]))
    # gemv_int8 after registering the weight (the setup_gemma_model hook)
    w, ws, xv, xs = (golden[f"gemv_a_{k}"] for k in ("w", "ws", "x", "xs"))
    assert shim.shim_register(w.ctypes.data, ws.ctypes.data, w.shape[0], w.shape[1]) == 0
    y = np.empty(w.shape[0], np.float32)
    shim.shim_gemv_int8(y.ctypes.data, w.ctypes.data, ws.ctypes.data, xv.ctypes.data, float(xs), w.shape[0],
                        w.shape[1])
    assert np.array_equal(bits(y), bits(golden["gemv_a_y"]))
    # gemv_int8_multi with GemvJob records
    mats = [golden[f"multi_w{j}"] for j in range(3)]
    scs = [golden[f"multi_ws{j}"] for j in range(3)]
    outs = [np.empty(m.shape[0], np.float32) for m in mats]
    jobs = (gcu.GemvJob * 3)(*[gcu.GemvJob(m.ctypes.data, s.ctypes.data, o.ctypes.data, m.shape[0])
                               for m, s, o in zip(mats, scs, outs)])
    mx = golden["multi_x"]  # keep the array alive across the call
    shim.shim_gemv_int8_multi(jobs, 3, mx.ctypes.data, float(golden["multi_xs"]), 640)
    for j in range(3):
        assert np.array_equal(bits(outs[j]), bits(golden[f"multi_y{j}"]))
    # gemm_int8, strided (gemma.c's dstr/mstr/sstr)
    m, n, k, dstr, mstr, sstr = (int(t) for t in golden["gemm_c_dims"])
    dst = np.full((m, dstr), -1.0, np.float32)
    cw, cws, cx, cxs = (golden[f"gemm_c_{t}"] for t in ("w", "ws", "x", "xs"))
    rc = shim.shim_gemm_int8(dst.ctypes.data, dstr, cw.ctypes.data, mstr, cws.ctypes.data, cx.ctypes.data, sstr,
                             cxs.ctypes.data, m, n, k)
    assert rc == 0
    assert np.array_equal(bits(dst), bits(golden["gemm_c_y"]))
    assert shim.shim_failed() == 0
    # PerfBench accounting kept (gemma.c:2648, 2787, 4052)
    assert shim.shim_perf_count(0) >= 2 and shim.shim_perf_count(1) >= 2 and shim.shim_perf_count(2) >= 1
