"""Model images registered as one arena (gcu_register_model) on the GPU.

After registering a synthetic `-q` model image, every matmul QTensor of it is
used through the host entry points with pointers INTO the image, exactly as
gemma.c passes its mmap'd weights (mmap_qtensor, gemma.c:1156-1171).  The
host copy of the weights is then overwritten, so a result that still matches
the oracle on the original weights came from the arena, not from a transient
upload.  Results are bit-exact against the CPU oracle.
"""
import json
import os

import numpy as np
import pytest

import binfmt
import oracle as O
import synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import gcu  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
with open(os.path.join(HERE, "golden", "bin_layout.json")) as _f:
    GOLDEN = {(c["name"], c["allow_mm"]): c for c in json.load(_f)}


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    gcu.init(0)
    yield
    gcu.check_device()


def _bits_equal(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def _check_all(buf, recs, orig, m, seed):
    """Every QTensor through gemm_int8 (m > 8: tensor cores; m <= 8: GEMV)
    with host pointers into `buf`; the oracle uses `orig`."""
    for i, r in enumerate(recs):
        q, s = binfmt.qtensor_arrays(buf, r)
        q0, s0 = binfmt.qtensor_arrays(orig, r)
        x = synth.activations(seed + i, m, r["k"])
        xq, xs = O.quantize_acts(x)
        got = gcu.gemm_int8(q, s, xq, xs)
        want = O.gemm_int8(np.ascontiguousarray(q0), np.ascontiguousarray(s0), xq, xs)
        assert _bits_equal(got, want), (r["kind"], r["layer"], m)


@pytest.mark.parametrize("name,allow_mm", [("mm_small", True), ("mm_small", False), ("text_all_norms", True),
                                           ("mm_odd", True)])
def test_register_model_serves_every_weight(name, allow_mm):
    case = GOLDEN[(name, allow_mm)]
    orig, _ = binfmt.image(case["text"], case["vision"], seed=case["seed"])
    buf = orig.copy()
    before = gcu.registered_bytes()
    arena = gcu.register_model(buf, allow_mm)
    try:
        recs = gcu.bin_qtensors(buf, allow_mm)
        assert recs == case["qtensors"]
        need = sum(r["rows"] * r["k"] + 4 * r["rows"] for r in recs)
        assert need <= gcu.registered_bytes() - before <= need + 512 * len(recs)
        # the host copy changes: results must still be those of the registered weights
        for r in recs:
            q, s = binfmt.qtensor_arrays(buf, r)
            q[...] = 0
            s[...] = 0.0
        _check_all(buf, recs, orig, 40, 100)
        _check_all(buf, recs, orig, 3, 200)
    finally:
        gcu.unregister_arena(arena)
    assert gcu.registered_bytes() == before


def test_arena_rules():
    case = GOLDEN[("mm_small", True)]
    buf, _ = binfmt.image(case["text"], case["vision"], seed=case["seed"])
    arena = gcu.register_model(buf)
    try:
        with pytest.raises(gcu.GcuError, match="overlaps"):
            gcu.register_model(buf)
        r = case["qtensors"][3]
        q, s = binfmt.qtensor_arrays(buf, r)
        with pytest.raises(gcu.GcuError, match="arena"):
            gcu.unregister_weight(q)
        gcu.register_weight(q, s)  # the same tensor again: already registered, a no-op
    finally:
        gcu.unregister_arena(arena)
    with pytest.raises(gcu.GcuError, match="no arena"):
        gcu.unregister_arena(arena)
    arena = gcu.register_model(buf)  # registrable again once dropped
    gcu.unregister_arena(arena)


def test_register_qtensors_list():
    # the read_gemma_model case: tensors in separate buffers (gemma.c:1134-1153)
    ws = [synth.weight(900 + i, n, k) for i, (n, k) in enumerate([(1024, 640), (256, 640), (640, 1024), (33, 48)])]
    arena = gcu.register_qtensors(ws)
    try:
        saved = [(q.copy(), s.copy()) for q, s in ws]
        for q, s in ws:
            q[...] = 0
        for i, ((q, s), (q0, s0)) in enumerate(zip(ws, saved)):
            xq, xs = O.quantize_acts(synth.activations(950 + i, 20, q.shape[1]))
            assert _bits_equal(gcu.gemm_int8(q, s, xq, xs), O.gemm_int8(q0, s0, xq, xs))
    finally:
        gcu.unregister_arena(arena)


def test_lm_head_of_a_full_size_image():
    # Gemma 3 1B text decoder at full size (1.0 GB image); the tied lm_head
    # (262144 x 1152) and a sample of layers checked bit-exact
    buf, _ = binfmt.image(binfmt.TEXT_1B, None, seed=7, fast=True)
    arena = gcu.register_model(buf)
    try:
        recs = gcu.bin_qtensors(buf)
        assert len(recs) == 1 + 7 * binfmt.TEXT_1B["nl"]
        head = recs[0]
        q, s = binfmt.qtensor_arrays(buf, head)
        xq, xs = O.quantize_acts(synth.activations(77, 1, head["k"]))
        assert _bits_equal(gcu.gemv_int8(q, s, xq[0], xs[0]), O.gemv_int8(q, s, xq[0], xs[0]))
        for r in [recs[1], recs[5], recs[7], recs[-1]]:
            q, s = binfmt.qtensor_arrays(buf, r)
            xq, xs = O.quantize_acts(synth.activations(78, 64, r["k"]))
            assert _bits_equal(gcu.gemm_int8(q, s, xq, xs),
                               O.gemm_int8(np.ascontiguousarray(q), np.ascontiguousarray(s), xq, xs))
    finally:
        gcu.unregister_arena(arena)


def test_register_rejects_bad_lists():
    with pytest.raises(gcu.GcuError, match="no tensors"):
        gcu.register_qtensors([])
    with pytest.raises(gcu.GcuError, match="W8A8"):
        gcu.register_model(np.frombuffer(b"GEMAf32U" + bytes(64), np.uint8).copy())
