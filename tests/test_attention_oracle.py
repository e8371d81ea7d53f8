"""The fp32 attention restatement (oracle) against gemma.c's own attention.

tests/golden/attention.npz holds the outputs of the reference's decode
attention (gemma.c:4836-4848) and prefill attention loop (gemma.c:5160-5295)
on seeded inputs (make_attention_golden.py).  The reference is compiled with
-ffast-math and vectorizes its fp32 dot products, so agreement is to fp32
reassociation: max |oracle - reference| <= 1e-5 * max |reference| (measured
1e-7 .. 3e-6 on these cases).  Host only.
"""
import json
import os

import numpy as np
import pytest

import oracle as O
import synth

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "attention.npz"))
META = json.loads(str(GOLD["meta"]))
TOL = 1e-5  # of the output's largest magnitude


def assert_attn_close(got, want, tol=TOL):
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    assert got.shape == want.shape
    err = float(np.max(np.abs(got - want)))
    scale = float(np.max(np.abs(want)))
    assert np.all(np.isfinite(got)) and err <= tol * scale, f"max err {err:.3g} vs {tol} x {scale:.3g}"


@pytest.mark.parametrize("case", META["decode"], ids=lambda c: f"decode{c[0]}")
def test_oracle_decode_matches_reference_fixture(case):
    tid, nh, nkv, hd, clen, spos, attlen, sc = case
    xq, kc, vc = synth.attention_inputs(tid, nh, nkv, hd, clen)
    got = O.attention_decode(xq, kc, vc, spos, attlen, np.float32(1.0 / np.sqrt(hd)), sc)
    assert_attn_close(got, GOLD[f"decode_{tid}"])


@pytest.mark.parametrize("case", META["prefill"], ids=lambda c: f"prefill{c[0]}")
def test_oracle_prefill_matches_reference_fixture(case):
    tid, nh, nkv, hd, spos, ntok, slide, sc, mask = case
    xq, kc, vc = synth.attention_inputs(tid, nh, nkv, hd, spos + ntok + 3, ntok)
    got = O.attention_prefill(xq, kc, vc, spos, slide, sc, bool(mask))
    assert_attn_close(got, GOLD[f"prefill_{tid}"])


def _ref():
    try:
        lib = O.ref()
    except OSError:
        return None
    if lib is None or not hasattr(lib, "ref_attention_decode"):
        return None
    return O.Ref(threads=4)


@pytest.mark.parametrize("nh,nkv,hd,clen,spos,attlen,sc", [(4, 1, 256, 700, 200, 300, 0.0),
                                                          (16, 8, 256, 1500, 0, 1500, 30.0),
                                                          (6, 3, 64, 90, 17, 73, 0.0),
                                                          (6, 4, 128, 300, 0, 300, 0.0)])  # uneven groups
def test_oracle_decode_matches_live_reference(nh, nkv, hd, clen, spos, attlen, sc):
    R = _ref()
    if R is None:
        pytest.skip("reference build not available")
    xq, kc, vc = synth.attention_inputs(7 + attlen, nh, nkv, hd, clen)
    asc = np.float32(1.0 / np.sqrt(hd))
    assert_attn_close(O.attention_decode(xq, kc, vc, spos, attlen, asc, sc),
                      R.attention_decode(xq, kc, vc, spos, attlen, asc, sc))


@pytest.mark.parametrize("nh,nkv,hd,spos,ntok,slide,sc,mask", [(4, 1, 256, 0, 150, 64, 0.0, True),
                                                               (8, 2, 128, 64, 96, 0, 20.0, True),
                                                               (2, 1, 64, 30, 45, 16, 0.0, False),
                                                               (6, 4, 64, 0, 70, 0, 0.0, True)])  # uneven
def test_oracle_prefill_matches_live_reference(nh, nkv, hd, spos, ntok, slide, sc, mask):
    R = _ref()
    if R is None:
        pytest.skip("reference build not available")
    xq, kc, vc = synth.attention_inputs(9 + ntok, nh, nkv, hd, spos + ntok, ntok)
    assert_attn_close(O.attention_prefill(xq, kc, vc, spos, slide, sc, mask),
                      R.attention_prefill(xq, kc, vc, spos, slide, sc, mask))


def test_oracle_single_position_returns_the_value_row():
    # one visible position: weight fast_expf(0) = 1, so xo is V's row exactly
    xq, kc, vc = synth.attention_inputs(3, 4, 2, 64, 10)
    got = O.attention_decode(xq, kc, vc, 6, 1, np.float32(0.125))
    want = np.repeat(vc[:, 6, :], 2, axis=0)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("case", META.get("rope", []), ids=lambda c: f"rope{c[0]}")
def test_oracle_rope_matches_reference_fixture(case):
    # QK norm + RoPE + cache write (gemma.c:4775-4818, 5095-5145) on the
    # reference's own rope_freqs table
    tid, nh, nkv, hd, clen, spos, ntok, qs, norm, _, _ = case
    xq, xk, xv, kc, vc, nq, nk = synth.rope_inputs(tid, nh, nkv, hd, clen, ntok, norm)
    gq, gk, gv = O.qk_norm_rope_cache(xq, xk, xv, kc, vc, GOLD[f"rope_{tid}_freqs"], spos, qs, nq, nk)
    assert_attn_close(gq, GOLD[f"rope_{tid}_xq"])
    assert_attn_close(gk[:, spos:spos + ntok], GOLD[f"rope_{tid}_k"])
    assert np.array_equal(gv[:, spos:spos + ntok], xv)  # values are copied
    assert np.array_equal(gk[:, :spos], kc[:, :spos]) and np.array_equal(gk[:, spos + ntok:], kc[:, spos + ntok:])


def test_oracle_rope_matches_live_reference():
    R = _ref()
    if R is None or not hasattr(R.lib, "ref_qk_norm_rope_cache"):
        pytest.skip("reference build not available")
    slid, full = R.rope_freqs(128, 10000.0, 1e6, 700, 33)
    xq, xk, xv, kc, vc, nq, nk = synth.rope_inputs(340, 6, 2, 128, 800, 33, True)
    for fr in (slid, full):
        a = O.qk_norm_rope_cache(xq, xk, xv, kc, vc, fr, 700, 0.088, nq, nk)
        b = R.qk_norm_rope_cache(xq, xk, xv, kc, vc, fr, 700, 0.088, nq, nk)
        for x, y in zip(a, b):
            assert_attn_close(x, y)


# ---- size-independent properties of the two restatements

@pytest.mark.parametrize("nh,nkv,hd,spos,ntok,slide,sc", [(4, 1, 256, 0, 40, 0, 0.0), (6, 2, 64, 30, 50, 16, 0.0),
                                                          (4, 4, 128, 100, 20, 64, 25.0)])
def test_oracle_prefill_row_is_decode_over_its_window(nh, nkv, hd, spos, ntok, slide, sc):
    # causal prefill row i (queries pre-scaled) attends to exactly the window
    # decode attention sees at position spos + i with a unit score scale
    xq, kc, vc = synth.attention_inputs(40 + ntok, nh, nkv, hd, spos + ntok, ntok)
    pre = O.attention_prefill(xq, kc, vc, spos, slide, sc, True)
    for i in range(ntok):
        pos = spos + i
        t0 = pos + 1 - slide if slide > 0 and pos >= slide else 0
        dec = O.attention_decode(np.ascontiguousarray(xq[:, i, :]), kc, vc, t0, pos + 1 - t0, np.float32(1.0), sc)
        assert_attn_close(pre[i].reshape(nh, hd), dec)


def test_oracle_output_is_linear_in_values():
    # weights do not depend on V: scaling V by a power of two scales the output exactly
    xq, kc, vc = synth.attention_inputs(77, 8, 2, 128, 300)
    a = O.attention_decode(xq, kc, vc, 10, 250, np.float32(0.088))
    b = O.attention_decode(xq, kc, (vc * np.float32(4.0)).astype(np.float32), 10, 250, np.float32(0.088))
    assert np.array_equal(b, a * np.float32(4.0))
    xq, kc, vc = synth.attention_inputs(78, 4, 1, 64, 60, 60)
    a = O.attention_prefill(xq, kc, vc, 0, 16)
    b = O.attention_prefill(xq, kc, (vc * np.float32(0.5)).astype(np.float32), 0, 16)
    assert np.array_equal(b, a * np.float32(0.5))


def test_oracle_weights_sum_to_one():
    xq, kc, _ = synth.attention_inputs(79, 4, 2, 256, 2000)
    out = O.attention_decode(xq, kc, np.ones_like(kc), 0, 2000, np.float32(1 / 16), 30.0)
    assert np.max(np.abs(out - 1.0)) < 1e-5
    xq, kc, _ = synth.attention_inputs(80, 2, 1, 64, 300, 300)
    out = O.attention_prefill(xq, kc, np.ones_like(kc), 0, 100)
    assert np.max(np.abs(out - 1.0)) < 1e-5


def test_oracle_matches_live_reference_on_drawn_shapes():
    # hypothesis draws head layouts (uneven groups included), head sizes,
    # windows, sliding spans, softcaps and the dense path; the restatement
    # stays within the fp32 bound of gemma.c's own compiled attention
    hyp = pytest.importorskip("hypothesis")
    from hypothesis import given, settings, strategies as st
    R = _ref()
    if R is None:
        pytest.skip("reference build not available")

    @settings(max_examples=25, deadline=None, derandomize=True)
    @given(st.data())
    def run(data):
        nkv = data.draw(st.integers(1, 4))
        nh = data.draw(st.integers(nkv, 4 * nkv))
        hd = data.draw(st.sampled_from([64, 128, 256]))
        sc = data.draw(st.sampled_from([0.0, 30.0]))
        clen = data.draw(st.integers(1, 600))
        spos = data.draw(st.integers(0, clen - 1))
        attlen = data.draw(st.integers(1, clen - spos))
        xq, kc, vc = synth.attention_inputs(1000 + clen, nh, nkv, hd, clen)
        asc = np.float32(1.0 / np.sqrt(hd))
        assert_attn_close(O.attention_decode(xq, kc, vc, spos, attlen, asc, sc),
                          R.attention_decode(xq, kc, vc, spos, attlen, asc, sc))
        ntok = data.draw(st.integers(1, 120))
        pspos = data.draw(st.integers(0, 150))
        slide = data.draw(st.sampled_from([0, 16, 64]))
        mask = data.draw(st.booleans())
        xq, kc, vc = synth.attention_inputs(2000 + ntok, nh, nkv, hd, pspos + ntok, ntok)
        assert_attn_close(O.attention_prefill(xq, kc, vc, pspos, slide, sc, mask),
                          R.attention_prefill(xq, kc, vc, pspos, slide, sc, mask))

    run()


def test_oracle_rope_matches_live_reference_on_drawn_shapes():
    # QK norm + RoPE + cache write on drawn head layouts, head sizes,
    # positions, chunk lengths and norm settings, with the reference's own
    # rope_freqs tables (local and global theta)
    pytest.importorskip("hypothesis")
    from hypothesis import given, settings, strategies as st
    R = _ref()
    if R is None or not hasattr(R.lib, "ref_qk_norm_rope_cache"):
        pytest.skip("reference build not available")

    @settings(max_examples=15, deadline=None, derandomize=True)
    @given(st.data())
    def run(data):
        nkv = data.draw(st.integers(1, 4))
        nh = data.draw(st.integers(nkv, 3 * nkv))
        hd = data.draw(st.sampled_from([64, 128, 256]))
        ntok = data.draw(st.integers(1, 40))
        spos = data.draw(st.integers(0, 3000))
        norm = data.draw(st.booleans())
        qs = data.draw(st.sampled_from([1.0, 0.0625, 0.088]))
        slid, full = R.rope_freqs(hd, 10000.0, 1e6, spos, ntok)
        xq, xk, xv, kc, vc, nq, nk = synth.rope_inputs(3000 + ntok, nh, nkv, hd, spos + ntok + 2, ntok, norm)
        for fr in (slid, full):
            a = O.qk_norm_rope_cache(xq, xk, xv, kc, vc, fr, spos, qs, nq, nk)
            b = R.qk_norm_rope_cache(xq, xk, xv, kc, vc, fr, spos, qs, nq, nk)
            for x, y in zip(a, b):
                assert_attn_close(x, y)

    run()
