"""The CPU oracle against the reference's golden vectors (CPU only).

The oracle (oracle/gemma_oracle.c) is what every GPU parity test compares
with, so it is pinned here first: bit-exact against fixtures produced by the
reference's own compiled functions (tests/golden/make_golden.py), against an
independent numpy int64 accumulator, and -- where the reference build is
present -- against the reference itself on fresh random inputs.
"""
import numpy as np
import pytest

import oracle as O
import synth


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_quantize_matches_golden(golden):
    q, s = O.quantize_acts(golden["quant_a_x"])
    assert np.array_equal(q, golden["quant_a_q"])
    assert np.array_equal(bits(s), bits(golden["quant_a_s"]))
    # the all-zero row: scale 1, codes 0 (gemma.c:2615)
    assert s[2] == 1.0 and not q[2].any()
    # round half away from zero at the boundaries (gemma.c:2642-2645)
    assert list(q[3, :8]) == [127, 64, -64, 1, -1, 2, -3, 127]


def test_quantize_strided_odd_width(golden):
    q, s = O.quantize_acts(golden["quant_b_x"], n=33, sstr=40)
    assert np.array_equal(q, golden["quant_b_q"])
    assert np.array_equal(bits(s), bits(golden["quant_b_s"]))


def test_quantize_act_single(golden):
    q, s = O.quantize_act(golden["quant_c_x"])
    assert np.array_equal(q, golden["quant_c_q"])
    assert bits(s) == bits(golden["quant_c_s"])


@pytest.mark.parametrize("name", ["gemv_a", "gemv_b"])
def test_gemv_matches_golden(golden, name):
    g = lambda k: golden[f"{name}_{k}"]
    y = O.gemv_int8(g("w"), g("ws"), g("x"), g("xs"))
    assert np.array_equal(bits(y), bits(g("y")))


def test_gemv_multi_matches_golden(golden):
    mats = [golden[f"multi_w{j}"] for j in range(3)]
    scs = [golden[f"multi_ws{j}"] for j in range(3)]
    ys = O.gemv_int8_multi(mats, scs, golden["multi_x"], golden["multi_xs"])
    for j in range(3):
        assert np.array_equal(bits(ys[j]), bits(golden[f"multi_y{j}"]))


@pytest.mark.parametrize("name", ["gemm_a", "gemm_b", "gemm_d"])
def test_gemm_matches_golden(golden, name):
    g = lambda k: golden[f"{name}_{k}"]
    y = O.gemm_int8(g("w"), g("ws"), g("x"), g("xs"))
    assert np.array_equal(bits(y), bits(g("y")))


def test_gemm_strided_matches_golden(golden):
    m, n, k, dstr, mstr, sstr = (int(v) for v in golden["gemm_c_dims"])
    dst = np.full((m, dstr), -1.0, np.float32)
    O.gemm_int8(golden["gemm_c_w"].reshape(-1), golden["gemm_c_ws"], golden["gemm_c_x"].reshape(-1),
                golden["gemm_c_xs"], dst=dst, dstr=dstr, mstr=mstr, sstr=sstr, m=m, n=n, k=k)
    assert np.array_equal(bits(dst), bits(golden["gemm_c_y"]))
    assert (dst[:, n:] == -1.0).all()  # padding columns untouched


def test_acc_int8_matches_int64_matmul():
    rng = np.random.default_rng(5)
    a = rng.integers(-127, 128, (17, 300), dtype=np.int8)
    b = rng.integers(-127, 128, (23, 300), dtype=np.int8)
    ref = a.astype(np.int64) @ b.astype(np.int64).T
    assert np.array_equal(O.acc_int8(b, a), ref.astype(np.int32))


def test_dequant_is_acc_times_scale_product(golden):
    # (float)acc * (xs*ws): the epilogue form the -ffast-math build runs
    g = lambda k: golden[f"gemm_a_{k}"]
    acc = O.acc_int8(g("w"), g("x"))
    y = acc.astype(np.float32) * (g("xs")[:, None] * g("ws")[None, :])
    assert np.array_equal(bits(y), bits(g("y")))


def test_weight_quantizer_c_matches_numpy():
    w = synth.normal(9, (64, 640), 0.02)
    q1, s1 = O.quantize_weight_rows(w)
    q2, s2 = synth.quantize_weight_rows(w)
    assert np.array_equal(q1, q2) and np.array_equal(bits(s1), bits(s2))


def test_weight_quantizer_matches_model_py_semantics():
    torch = pytest.importorskip("torch")
    w = synth.normal(12, (32, 256), 0.02)
    t = torch.from_numpy(w)
    amax = t.abs().amax(1, keepdim=True).clamp_min(1e-8)  # model.py:100-103
    sc = amax / 127.0
    q = torch.round(t / sc).clamp(-127, 127).to(torch.int8)
    q2, s2 = synth.quantize_weight_rows(w)
    assert np.array_equal(q.numpy(), q2)
    assert np.array_equal(bits(sc.squeeze(1).numpy()), bits(s2))


ref_lib = O.ref()


@pytest.mark.skipif(ref_lib is None, reason="reference build not present on this host")
def test_oracle_matches_reference_random():
    R = O.Ref(threads=4)
    for it, (m, k) in enumerate([(1, 640), (7, 1152), (33, 2560), (5, 4304), (3, 24)]):
        x = synth.activations(500 + it, m, k, outliers=True)
        q1, s1 = O.quantize_acts(x)
        q2, s2 = R.quantize_acts(x)
        assert np.array_equal(q1, q2) and np.array_equal(bits(s1), bits(s2))
        w, ws = synth.weight(600 + it, 48, k)
        y1 = O.gemm_int8(w, ws, q1, s1)
        y2 = R.gemm_int8(w, ws, q2, s2)
        assert np.array_equal(bits(y1), bits(y2))
        y1 = O.gemv_int8(w, ws, q1[0], s1[0])
        y2 = R.gemv_int8(w, ws, q2[0], s2[0])
        assert np.array_equal(bits(y1), bits(y2))


def rel_err(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.skipif(ref_lib is None, reason="reference build not present on this host")
@pytest.mark.parametrize("m,dim", [(4, 640), (3, 1152), (2, 2560), (2, 3840), (2, 15360), (5, 40)])
def test_producer_restatements_match_reference(m, dim):
    # rmsnorm and gelu*up then quantize_acts: the restatement sums squares in
    # order and uses this libm's tanhf; gemma.c's -ffast-math build
    # vectorizes the sum, so fp32 values agree within BASELINE's 1e-5
    # relative tolerance (1e-6 in practice) and the codes all but identically
    R = O.Ref(threads=4)
    x = synth.activations(70 + dim, m, dim, outliers=True)
    w = (synth.activations(71 + dim, 1, dim)[0] * 0.1).astype(np.float32)
    xn0, q0, s0 = R.rmsnorm_quantize(x, w, 1e-6)
    xn1, q1, s1 = O.rmsnorm_quantize(x, w, 1e-6)
    assert rel_err(xn1, xn0) < 1e-5
    assert rel_err(s1, s0) < 1e-5
    assert np.abs(q1.astype(int) - q0).max() <= 1 and (q1 != q0).mean() < 1e-3
    g = synth.activations(72 + dim, m, dim)
    u = synth.activations(73 + dim, m, dim)
    h0, qg0, sg0 = R.geglu_quantize(g, u)
    h1, qg1, sg1 = O.geglu_quantize(g, u)
    assert rel_err(h1, h0) < 1e-5
    assert rel_err(sg1, sg0) < 1e-5
    assert np.abs(qg1.astype(int) - qg0).max() <= 1 and (qg1 != qg0).mean() < 1e-3


def test_producer_quantize_step_is_quantize_act():
    # the restated producers quantize exactly as quantize_acts does
    x = synth.activations(80, 3, 1152, outliers=True)
    w = (synth.activations(81, 1, 1152)[0] * 0.1).astype(np.float32)
    xn, q, s = O.rmsnorm_quantize(x, w, 1e-6)
    q2, s2 = O.quantize_acts(xn)
    assert np.array_equal(q, q2) and np.array_equal(bits(s), bits(s2))
    h, qg, sg = O.geglu_quantize(x, x * 0.5)
    q3, s3 = O.quantize_acts(h)
    assert np.array_equal(qg, q3) and np.array_equal(bits(sg), bits(s3))


def test_synth_generator_is_deterministic():
    a = synth.normal(3, (1000,))
    b = synth.normal(3, (1000,))
    assert np.array_equal(a, b)
    assert abs(float(a.mean())) < 0.1 and 0.9 < float(a.std()) < 1.1
    cols = synth.outlier_columns(1, 1152)
    assert len(cols) == 12 and len(set(cols.tolist())) == 12
