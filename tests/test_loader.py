"""The `-q` model-image parser (gcu_bin_qtensors) against gemma.c's own loader.

tests/golden/bin_layout.json holds, for synthetic model files, where the
reference's mmap_gemma_model (gemma.c:1946-2043) finds every matmul QTensor;
make_bin_layout.py made it with the compiled reference.  The parser must
return the same records (kind, layer, rows, k, byte offsets of the int8
values and of the scales) for the same bytes, and refuse the malformed
images gemma.c refuses.  Host only: no GPU is touched.
"""
import json
import os
import tempfile

import numpy as np
import pytest

import binfmt
import gcu
import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
with open(os.path.join(HERE, "golden", "bin_layout.json")) as _f:
    GOLDEN = json.load(_f)


def _ref_with_layout():
    try:
        lib = O.ref()
    except OSError:
        return None
    if lib is None or not hasattr(lib, "ref_bin_layout"):
        return None
    return O.Ref(threads=1)


def _image(case):
    buf, _ = binfmt.image(case["text"], case["vision"], seed=case["seed"])
    return buf


@pytest.mark.parametrize("case", GOLDEN, ids=lambda c: f"{c['name']}-mm{int(c['allow_mm'])}")
def test_parser_matches_reference_fixture(case):
    buf = _image(case)
    assert buf.nbytes == case["bytes"]
    assert gcu.bin_qtensors(buf, case["allow_mm"]) == case["qtensors"]


@pytest.mark.parametrize("case", GOLDEN, ids=lambda c: f"{c['name']}-mm{int(c['allow_mm'])}")
def test_writer_layout_matches_reference_fixture(case):
    buf, hl = binfmt.image(case["text"], case["vision"], seed=case["seed"])
    assert binfmt.expected_qtensors(case["text"], case["vision"], hl, case["allow_mm"]) == case["qtensors"]


def test_parser_matches_live_reference():
    R = _ref_with_layout()
    if R is None:
        pytest.skip("reference build not available")
    text = dict(nl=4, n_heads=3, nkv=3, hdim=24, dim=72, mlp_dim=40, nvocab=999, qk_norm=True, mlp_pst=True)
    vision = dict(nl=3, n_heads=2, mlp_dim=64, dim=32, img_px=40, psize=8)
    buf, _ = binfmt.image(text, vision, seed=11)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.bin")
        buf.tofile(path)
        for allow_mm in (True, False):
            assert gcu.bin_qtensors(buf, allow_mm) == R.bin_layout(path, allow_mm)


def test_trailing_bytes_are_ignored():
    case = GOLDEN[0]
    buf, _ = binfmt.image(case["text"], case["vision"], seed=case["seed"], pad=4096)
    assert gcu.bin_qtensors(buf, True) == case["qtensors"]


def _malformed():
    text = dict(nl=2, n_heads=2, nkv=1, hdim=16, dim=32, mlp_dim=48, nvocab=40)
    vision = dict(nl=1, n_heads=1, mlp_dim=32, dim=16, img_px=28, psize=14)
    good, hl = binfmt.image(text, vision, seed=9)
    cases = {}
    b = good.copy(); b[0:4] = np.frombuffer(b"GEMX", np.uint8); cases["magic"] = (b, "magic", True)
    b = good.copy(); b[4:7] = np.frombuffer(b"f16", np.uint8); cases["dtype"] = (b, "dtype", True)
    b = good.copy(); b[7] = ord("U"); cases["unquantized"] = (b, "W8A8", False)
    b = good.copy(); b[7] = ord("X"); cases["flag"] = (b, "flag", True)
    b = good.copy(); b[8 + 3 + 12 + 8 + 20] = 0; cases["swa_bytes"] = (b, "att_layers", True)
    cases["header_only"] = (good[:8].copy(), "truncated", True)
    cases["in_tokenizer"] = (good[:hl - 5].copy(), "truncated", True)
    cases["in_tensors"] = (good[:-1].copy(), "ends before", False)
    cases["empty"] = (good[:0].copy(), "no header", True)
    return cases


@pytest.mark.parametrize("name", list(_malformed()))
def test_malformed_images_are_refused(name):
    buf, msg, ref_refuses = _malformed()[name]
    with pytest.raises(gcu.GcuError, match=msg):
        gcu.bin_qtensors(buf)
    R = _ref_with_layout()
    if R is None or not ref_refuses or buf.nbytes == 0:
        return
    # gemma.c refuses the same file (a 'U' file it would load unquantized,
    # and it maps past a short file's end without reading it, so those two
    # are this library's own checks)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.bin")
        buf.tofile(path)
        with pytest.raises(RuntimeError, match="refused"):
            R.bin_layout(path)


def test_capacity_and_counting():
    case = next(c for c in GOLDEN if c["vision"] and c["allow_mm"])
    buf = _image(case)
    n = gcu.lib().gcu_bin_qtensors(buf.ctypes.data, buf.nbytes, 1, None, 0)
    assert n == len(case["qtensors"])
    recs = (gcu.QTensor * 3)()
    assert gcu.lib().gcu_bin_qtensors(buf.ctypes.data, buf.nbytes, 1, recs, 3) == n
    assert [r.kind for r in recs] == [0, 1, 2]


def test_parser_matches_live_reference_on_drawn_configs():
    # hypothesis draws decoder and SigLIP configurations (head layouts, odd
    # widths and vocabularies, every norm flag, with and without a vision
    # tower); the parser and gemma.c's mmap_gemma_model must find the same
    # records in the same bytes
    pytest.importorskip("hypothesis")
    from hypothesis import given, settings, strategies as st
    R = _ref_with_layout()
    if R is None:
        pytest.skip("reference build not available")

    @settings(max_examples=12, deadline=None, derandomize=True)
    @given(st.data())
    def run(data):
        nkv = data.draw(st.integers(1, 3))
        text = dict(nl=data.draw(st.integers(1, 3)), n_heads=nkv * data.draw(st.integers(1, 3)), nkv=nkv,
                    hdim=2 * data.draw(st.integers(2, 16)), dim=data.draw(st.integers(8, 80)),
                    mlp_dim=data.draw(st.integers(4, 64)), nvocab=data.draw(st.integers(20, 700)),
                    qk_norm=data.draw(st.booleans()), mlp_pre=data.draw(st.booleans()),
                    mlp_pst=data.draw(st.booleans()))
        vision = None
        if data.draw(st.booleans()):
            psize = data.draw(st.integers(1, 8))
            vision = dict(nl=data.draw(st.integers(0, 2)), n_heads=data.draw(st.integers(1, 2)),
                          mlp_dim=data.draw(st.integers(4, 40)), dim=data.draw(st.integers(4, 40)),
                          img_px=psize * data.draw(st.integers(1, 6)), psize=psize)
        buf, _ = binfmt.image(text, vision, seed=data.draw(st.integers(0, 99)))
        with tempfile.TemporaryDirectory() as d:
            path = os.path.join(d, "m.bin")
            buf.tofile(path)
            for allow_mm in (True, False):
                assert gcu.bin_qtensors(buf, allow_mm) == R.bin_layout(path, allow_mm)

    run()
