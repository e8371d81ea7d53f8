"""CPU checks of the drop-in build (oracle/_ref/libgemma_dropin.so, gemma.c
with its hot path replaced by gemma_gcu.h): it loads, says it is the drop-in
build, and the reference build of the same harness runs gemma.c's whole
model path on the synthetic models the GPU test uses.  The GPU comparison
itself is tests/test_gpu_dropin.py."""
import numpy as np
import pytest

import dropin_cases as D


def test_dropin_build_loads_without_a_gpu():
    lib = D.load("dropin")
    if lib is None:
        pytest.skip("oracle/_ref/libgemma_dropin.so not built (make -C oracle dropin)")
    assert lib.ref_dropin() == 1
    native = D.load("native")
    if native is not None:
        assert native.ref_dropin() == 0


@pytest.mark.parametrize("name", list(D.CASES))
@pytest.mark.parametrize("mmap_on", [0, 1])
def test_reference_model_path_runs(tmp_path, name, mmap_on):
    lib = D.load("native")
    if lib is None:
        pytest.skip("oracle/_ref/libgemma_ref_native.so not built")
    path = D.write_model(tmp_path, name)
    out = D.run(lib, path, name, mmap_on)
    assert np.isfinite(out).all() and np.abs(out).max() > 0
    # mapping and reading the same file give the same forward passes
    other = D.run(lib, path, name, 1 - mmap_on)
    assert np.array_equal(out.view(np.uint32), other.view(np.uint32))
