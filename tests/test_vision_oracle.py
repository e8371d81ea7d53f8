"""The SigLIP-head restatement (oracle) against gemma.c's own forward_vision.

tests/golden/vision.npz holds what the reference's forward_vision computes on
an encoder with no layers (make_vision_golden.py): the pooled, RMSNorm'd
rows, their int8 codes and scales (quantize_acts), and the int8 projection.
The patch embedding, LayerNorm and RMSNorm are fp32 sums that the reference
vectorizes under -ffast-math, so the rows agree to fp32 reassociation
(max |oracle - reference| <= 1e-5 * max |reference|); an int8 code may then
differ by one where a value sits on a rounding boundary.  The projection is
the exact int8 path: on the reference's own codes it is bit-exact.  Host only.
"""
import json
import os

import numpy as np
import pytest

import oracle as O
import synth

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "vision.npz"))
CASES = json.loads(str(GOLD["meta"]))["cases"]
TOL = 1e-5


def assert_rows_close(got, want, tol=TOL):
    err = float(np.max(np.abs(got - want)))
    assert err <= tol * float(np.max(np.abs(want))), err


def assert_codes_close(got, want):
    d = np.abs(got.astype(np.int32) - want.astype(np.int32))
    assert d.max() <= 1 and (d != 0).sum() <= max(2, got.size // 1000), (int(d.max()), int((d != 0).sum()))


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"vision{c[0]}")
def test_oracle_head_matches_reference_fixture(case):
    tid = case[0]
    v = synth.vision_head_inputs(*case)
    pooled, q, s = O.vision_pool(O.patch_embed(v), v)
    assert_rows_close(pooled, GOLD[f"pooled_{tid}"])
    assert_codes_close(q, GOLD[f"q_{tid}"])
    assert_rows_close(s, GOLD[f"s_{tid}"])


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"vision{c[0]}")
def test_projection_on_reference_codes_is_exact(case):
    tid = case[0]
    v = synth.vision_head_inputs(*case)
    y = O.gemm_int8(v["proj_q"], v["proj_s"], GOLD[f"q_{tid}"], GOLD[f"s_{tid}"])
    assert np.array_equal(y.view(np.uint32), GOLD[f"proj_{tid}"].view(np.uint32))


def test_oracle_head_matches_live_reference():
    try:
        lib = O.ref()
    except OSError:
        lib = None
    if lib is None or not hasattr(lib, "ref_vision_head"):
        pytest.skip("reference build not available")
    v = synth.vision_head_inputs(650, 280, 14, 256, 100, 96)  # 20 x 20 patches pooled 2 x 2
    y, pooled, q, s = O.Ref(threads=4).vision_head(v)
    po, qo, so = O.vision_pool(O.patch_embed(v), v)
    assert_rows_close(po, pooled)
    assert_codes_close(qo, q)


def test_pooling_identity_window():
    # ksize 1: the pooled row is RMSNorm(LayerNorm(patch row)), checked by hand
    v = synth.vision_head_inputs(660, 56, 14, 64, 16, 32)
    x = O.patch_embed(v)
    pooled, _, _ = O.vision_pool(x, v)
    mu = x.mean(axis=1, keepdims=True, dtype=np.float64)
    ln = (x - mu) / np.sqrt(((x - mu) ** 2).mean(axis=1, keepdims=True) + v["eps"]) * v["post_n"] + v["post_nb"]
    rms = ln / np.sqrt((ln ** 2).mean(axis=1, keepdims=True) + v["eps"]) * (v["norm"] + 1.0)
    assert np.max(np.abs(pooled - rms)) <= 1e-5 * np.max(np.abs(rms))


def test_oracle_head_matches_live_reference_on_drawn_shapes():
    # hypothesis draws patch sizes, patch grids, pooling windows and widths;
    # the restatement stays within the fp32 bound of gemma.c's forward_vision
    # head, with at most a few +-1 codes on rounding boundaries
    pytest.importorskip("hypothesis")
    from hypothesis import given, settings, strategies as st
    try:
        lib = O.ref()
    except OSError:
        lib = None
    if lib is None or not hasattr(lib, "ref_vision_head"):
        pytest.skip("reference build not available")
    R = O.Ref(threads=4)

    @settings(max_examples=15, deadline=None, derandomize=True)
    @given(st.data())
    def run(data):
        psize = data.draw(st.integers(1, 16))
        side = data.draw(st.integers(1, 6))
        ppi = side * data.draw(st.integers(1, 4))
        dim = 4 * data.draw(st.integers(1, 48))
        tdim = data.draw(st.integers(1, 40))
        v = synth.vision_head_inputs(700 + ppi * psize, ppi * psize, psize, dim, side * side, tdim)
        _, pooled, q, s = R.vision_head(v)
        po, qo, so = O.vision_pool(O.patch_embed(v), v)
        assert_rows_close(po, pooled)
        assert_codes_close(qo, q)
        assert_rows_close(so, s)

    run()
