"""gemma.c's own forward passes with the CUDA drop-in (row a8 of the hot path:
the call sites gemma.c:4497-4717 vision, 4768-4966 decode, 5034-5437 prefill).

oracle/_ref/libgemma_dropin.so is the reference's gemma.c with its five
hot-path definitions (gemma.c:2586-2837, 3937-4054) replaced by
gemma.c_b200/host/gemma_gcu.h and the model hooks of gemma_gcu_model.h in
setup_gemma_model / cleanup_gemma_model (oracle/make_dropin.py applies the
patch; oracle/Makefile builds it with the reference build's own flags).
Both builds run gemma.c's model path on the same synthetic `-q` file --
setup_gemma_model (read or mmap), forward_gemma_image for the multimodal
model, forward_gemma_prefill of a prompt in chunks (the Q/K/V projections as
concurrent per-(head, 128-token) gemm_int8 tasks from OpenMP workers,
gemma.c:5045-5091), then forward_gemma_decode steps -- and the logits must be
IDENTICAL: the drop-in's quantize, GEMV and GEMM results are bit-exact
against gemma.c's, and every other stage is the same C code with the same
flags, so no tolerance is needed."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import binfmt  # noqa: E402
import dropin_cases as D  # noqa: E402
import gcu  # noqa: E402


@pytest.fixture(scope="module")
def libs():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    native, dropin = D.load("native"), D.load("dropin")
    if native is None or dropin is None:
        pytest.skip("oracle/_ref reference builds missing (make -C oracle ref dropin)")
    gcu.init(0)
    return native, dropin


@pytest.mark.parametrize("name", list(D.CASES))
@pytest.mark.parametrize("mmap_on", [0, 1])
def test_dropin_forward_equals_reference(tmp_path, libs, name, mmap_on):
    native, dropin = libs
    path = D.write_model(tmp_path, name)
    want = D.run(native, path, name, mmap_on)
    for _ in range(2):  # the second run re-registers after the release hook
        got = D.run(dropin, path, name, mmap_on)
        gcu.check_device()
        diff = got.view(np.uint32) != want.view(np.uint32)
        assert not diff.any(), (f"{diff.sum()} of {diff.size} logits differ; max |d| "
                                f"{np.abs(got - want).max():.3g} of max |x| {np.abs(want).max():.3g}")


@pytest.mark.parametrize("mmap_on", [0, 1])
def test_setup_hook_registers_every_matmul_weight(tmp_path, libs, mmap_on):
    _, dropin = libs
    c = D.CASES["vision"]
    path = D.write_model(tmp_path, "vision")
    lib = gcu.lib()
    lib.gcu_registered_bytes.restype = ctypes.c_size_t
    before = lib.gcu_registered_bytes()
    held = dropin.ref_model_registered_bytes(path.encode(), mmap_on, 1, 1024, c["chunk"]) - before
    hdr = binfmt.image(c["text"], c["vision"], seed=c["seed"])[1]
    recs = binfmt.expected_qtensors(c["text"], c["vision"], hdr)
    need = sum(r["rows"] * r["k"] + 4 * r["rows"] for r in recs)
    assert need <= held <= need + 512 * len(recs), (held, need)
    assert lib.gcu_registered_bytes() == before  # cleanup_gemma_model released them
