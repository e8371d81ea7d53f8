"""Size-independent properties of the CPU oracle (CPU only).

The golden vectors pin the oracle on fixed inputs; these properties hold on
any input, so hypothesis draws the shapes and values:

- quantize_act (gemma.c:2586-2650): codes in [-127, 127], the sign of each
  code follows its element, the largest |element| maps to +-127, and the
  reconstruction error |q * scale - x| is at most half a step (plus the
  float error of scale * inv != 1); a row of zeros gives scale 1 and zero
  codes; quantize_acts is quantize_act row by row (gemma.c:2652-2674).
- gemv / gemm (gemma.c:2754-2788, 3937-4054): row m of gemm_int8 equals
  gemv_int8 of activation row m bit for bit (both dequantize (float)acc *
  (xs * ws)); gemv_int8_multi equals its jobs run one by one; the int32
  sums are linear in the activation codes.
- where the reference build is present: drawn inputs (values on rounding
  boundaries among them) give the same bits through the restatement and
  through gemma.c's own compiled quantize_acts, gemv_int8 and gemm_int8.
"""
import numpy as np
import pytest

hyp = pytest.importorskip("hypothesis")
from hypothesis import given, settings, strategies as st  # noqa: E402
from hypothesis.extra import numpy as hnp  # noqa: E402

import oracle as O  # noqa: E402

SETTINGS = settings(max_examples=40, deadline=None, derandomize=True)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


finite32 = st.floats(min_value=-1e4, max_value=1e4, allow_nan=False, allow_infinity=False, width=32)


@SETTINGS
@given(hnp.arrays(np.float32, st.tuples(st.integers(1, 6), st.integers(1, 300)), elements=finite32))
def test_quantize_bounds_sign_and_error(x):
    q, s = O.quantize_acts(x)
    assert q.dtype == np.int8 and q.shape == x.shape
    assert q.min() >= -127 and q.max() <= 127
    for r in range(x.shape[0]):
        row, qr, sc = x[r].astype(np.float64), q[r].astype(np.int64), float(s[r])
        amax = float(np.max(np.abs(row)))
        if amax == 0.0:  # gemma.c:2615: an all-zero row has scale 1 and zero codes
            assert sc == 1.0 and not qr.any()
            continue
        assert np.all(qr * np.sign(row) >= 0)  # no code has the opposite sign of its element
        assert np.abs(qr[np.argmax(np.abs(row))]) == 127
        err = np.abs(qr * sc - row)
        assert np.all(err <= 0.5 * sc * (1 + 1e-5) + amax * 1e-6)


@SETTINGS
@given(hnp.arrays(np.float32, st.integers(1, 500), elements=finite32))
def test_quantize_act_is_one_row_of_quantize_acts(v):
    q1, s1 = O.quantize_act(v)
    q2, s2 = O.quantize_acts(v[None, :])
    assert np.array_equal(q1, q2[0]) and bits(s1) == bits(s2[0])


def _operands(data, m, n, k):
    i8 = st.integers(-127, 127)
    mat = data.draw(hnp.arrays(np.int8, (n, k), elements=i8))
    src = data.draw(hnp.arrays(np.int8, (m, k), elements=i8))
    pos = st.floats(min_value=float(np.float32(1e-4)), max_value=4.0, allow_nan=False, width=32)
    matsc = data.draw(hnp.arrays(np.float32, n, elements=pos))
    ssc = data.draw(hnp.arrays(np.float32, m, elements=pos))
    return mat, matsc, src, ssc


@SETTINGS
@given(st.data(), st.integers(1, 9), st.integers(1, 40), st.integers(1, 200))
def test_gemm_rows_are_gemv(data, m, n, k):
    mat, matsc, src, ssc = _operands(data, m, n, k)
    y = O.gemm_int8(mat, matsc, src, ssc)
    for r in range(m):
        assert np.array_equal(bits(y[r]), bits(O.gemv_int8(mat, matsc, src[r], ssc[r])))


@SETTINGS
@given(st.data(), st.lists(st.integers(1, 30), min_size=1, max_size=4), st.integers(1, 150))
def test_gemv_multi_is_its_jobs_one_by_one(data, rows, k):
    i8 = st.integers(-127, 127)
    pos = st.floats(min_value=float(np.float32(1e-4)), max_value=4.0, allow_nan=False, width=32)
    mats = [data.draw(hnp.arrays(np.int8, (n, k), elements=i8)) for n in rows]
    scs = [data.draw(hnp.arrays(np.float32, n, elements=pos)) for n in rows]
    vec = data.draw(hnp.arrays(np.int8, k, elements=i8))
    vsc = np.float32(data.draw(pos))
    outs = O.gemv_int8_multi(mats, scs, vec, vsc)
    for mat, sc, out in zip(mats, scs, outs):
        assert np.array_equal(bits(out), bits(O.gemv_int8(mat, sc, vec, vsc)))


@SETTINGS
@given(st.data(), st.integers(1, 6), st.integers(1, 30), st.integers(1, 120))
def test_int32_sums_are_linear_in_the_codes(data, m, n, k):
    half = st.integers(-63, 63)  # a + b stays inside int8
    mat = data.draw(hnp.arrays(np.int8, (n, k), elements=st.integers(-127, 127)))
    a = data.draw(hnp.arrays(np.int8, (m, k), elements=half))
    b = data.draw(hnp.arrays(np.int8, (m, k), elements=half))
    lhs = O.acc_int8(mat, (a.astype(np.int16) + b).astype(np.int8))
    assert np.array_equal(lhs, O.acc_int8(mat, a) + O.acc_int8(mat, b))


_REF = O.ref()


@pytest.mark.skipif(_REF is None, reason="reference build not present on this host")
@settings(max_examples=30, deadline=None, derandomize=True)
@given(st.data(), st.integers(1, 6), st.integers(1, 24), st.integers(1, 260))
def test_oracle_matches_live_reference_on_drawn_inputs(data, m, n, k):
    # drawn activations (no subnormals: the reference is built with fast math)
    # through quantize_acts, gemv_int8 and gemm_int8 of the compiled
    # reference and of the restatement: the same bits
    R = O.Ref(threads=2)
    el = st.one_of(st.floats(min_value=-1e4, max_value=1e4, allow_nan=False, allow_subnormal=False, width=32),
                   st.sampled_from([0.0, 0.5, -0.5, 1.5, -2.5, 127.0]))
    x = data.draw(hnp.arrays(np.float32, (m, k), elements=el))
    q1, s1 = O.quantize_acts(x)
    q2, s2 = R.quantize_acts(x)
    assert np.array_equal(q1, q2) and np.array_equal(bits(s1), bits(s2))
    w = data.draw(hnp.arrays(np.int8, (n, k), elements=st.integers(-127, 127)))
    pos = st.floats(min_value=float(np.float32(1e-4)), max_value=4.0, allow_nan=False, width=32)
    ws = data.draw(hnp.arrays(np.float32, n, elements=pos))
    assert np.array_equal(bits(O.gemm_int8(w, ws, q1, s1)), bits(R.gemm_int8(w, ws, q2, s2)))
    assert np.array_equal(bits(O.gemv_int8(w, ws, q1[0], s1[0])), bits(R.gemv_int8(w, ws, q2[0], s2[0])))
