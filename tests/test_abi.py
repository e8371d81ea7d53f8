"""The C ABI boundary without a GPU: libgcu.so loads, exports every entry
point include/gcu.h declares, and reports errors instead of crashing."""
import ctypes
import os
import re

import numpy as np
import pytest

import gcu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    text = open(os.path.join(ROOT, "include", "gcu.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gcu_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(gcu.LIB_PATH)
    names = header_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    assert set(header_functions()) == set(gcu.SIGNATURES)


def test_version_and_error_string():
    assert gcu.lib().gcu_version().decode().startswith("gcu")
    assert isinstance(gcu.lib().gcu_last_error(), bytes)


def test_bad_arguments_are_errors_not_crashes():
    # argument checks run before any CUDA call
    rc = gcu.lib().gcu_register_weight(None, None, 0, 0)
    assert rc == 1
    assert b"bad arguments" in gcu.lib().gcu_last_error()
    jobs = (gcu.GemvJob * 9)()
    x = np.zeros(16, np.int8)
    assert gcu.lib().gcu_gemv_int8_multi(jobs, 9, x.ctypes.data, 1.0, 16) == 1
    assert b"at most" in gcu.lib().gcu_last_error()


def test_zero_sized_calls_are_noops():
    assert gcu.lib().gcu_quantize_acts(None, None, None, 0, 0, 16) == 0
    assert gcu.lib().gcu_gemm_int8(None, 0, None, 0, None, None, 0, None, 0, 8, 8) == 0


def test_init_without_gpu_reports_error():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert gcu.lib().gcu_init(0) == 1
    assert gcu.lib().gcu_last_error() != b""


def test_product_does_not_import_oracle():
    pkg = os.path.join(ROOT, "gemma.c_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".c", ".h")):
                src = open(os.path.join(dirpath, f), errors="ignore").read()
                assert "import oracle" not in src and "oracle/" not in src, f
