"""GPU parity: libgcu.so (sm_100a kernels) against the CPU oracle.

Every check is bit-exact: int8 codes and scales of the quantize kernel, the
fp32 outputs of the GEMV and GEMM kernels (the reference's -ffast-math build
evaluates (float)acc * (xs*ws), and so do the kernels), and the int32
accumulators themselves (recovered exactly with unit scales).  Inputs are
seeded synthetic tensors; the golden fixtures come from the reference's own
compiled functions.  Calls go through the C ABI (gcu.py is a ctypes binding).
"""
import threading

import numpy as np
import pytest

import oracle as O
import synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import gcu  # noqa: E402


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def assert_bits(got, want):
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    assert got.shape == want.shape
    bad = bits(got) != bits(want)
    if bad.any():
        idx = np.argwhere(bad)[:5]
        raise AssertionError(f"{bad.sum()} of {bad.size} differ, first {idx.tolist()}: "
                             f"{got[tuple(idx[0])]} vs {want[tuple(idx[0])]}")


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    gcu.init(0)
    yield
    gcu.check_device()


def big_weight(tid, n, k):
    """Seeded quantized weight; large ones are drawn on the GPU (same
    quantizer) so the host-side generator stays fast."""
    if n * k <= 8 << 20:
        return synth.weight(tid, n, k)
    gen = torch.Generator(device="cuda").manual_seed(tid)
    w, s = synth.weight_torch(n, k, gen, "cuda")
    return w.cpu().numpy(), s.cpu().numpy()


# ---------------------------------------------------------------- quantize

def test_quantize_golden(golden):
    q, s = gcu.quantize_acts(golden["quant_a_x"])
    assert np.array_equal(q, golden["quant_a_q"])
    assert_bits(s, golden["quant_a_s"])
    q, s = gcu.quantize_acts(golden["quant_b_x"], n=33, sstr=40)
    assert np.array_equal(q, golden["quant_b_q"])
    assert_bits(s, golden["quant_b_s"])
    q, s = gcu.quantize_act(golden["quant_c_x"])
    assert np.array_equal(q, golden["quant_c_q"])
    assert bits(s) == bits(golden["quant_c_s"])


@pytest.mark.parametrize("m,k", [(1, 640), (1, 15360), (4, 1152), (64, 2560), (37, 6912), (3, 33),
                                 (2, 40000), (512, 1024), (700, 2048), (509, 6912)])
def test_quantize_random(m, k):
    x = synth.activations(1000 + k + m, m, k, outliers=True)
    q, s = gcu.quantize_acts(x)
    q0, s0 = O.quantize_acts(x)
    assert np.array_equal(q, q0)
    assert_bits(s, s0)


def test_quantize_host_strided_pipelined():
    # > 4 MB of input: the host call copies, quantizes and copies back in row
    # chunks on separate streams; rows are read at a stride of 2053 floats
    m, n, sstr = 611, 2000, 2053
    full = synth.activations(1500, m, sstr, outliers=True)
    q, s = gcu.quantize_acts(full, n=n, sstr=sstr)
    q0, s0 = O.quantize_acts(np.ascontiguousarray(full[:, :n]))
    assert np.array_equal(q, q0)
    assert_bits(s, s0)


def test_quantize_device_api():
    x = synth.activations(77, 300, 2560, outliers=True)
    xt = torch.from_numpy(x).cuda()
    q = torch.empty((300, 2560), dtype=torch.int8, device="cuda")
    s = torch.empty(300, dtype=torch.float32, device="cuda")
    gcu.dev_quantize_acts(q, s, xt, 300, 2560)
    torch.cuda.synchronize()
    q0, s0 = O.quantize_acts(x)
    assert np.array_equal(q.cpu().numpy(), q0)
    assert_bits(s.cpu().numpy(), s0)


# ---------------------------------------------------------------- GEMV

@pytest.mark.parametrize("name", ["gemv_a", "gemv_b"])
def test_gemv_golden(golden, name):
    g = lambda k: golden[f"{name}_{k}"]
    y = gcu.gemv_int8(g("w"), g("ws"), g("x"), g("xs"))  # unregistered: transient upload
    assert_bits(y, g("y"))


def test_gemv_multi_golden(golden):
    mats = [golden[f"multi_w{j}"] for j in range(3)]
    scs = [golden[f"multi_ws{j}"] for j in range(3)]
    for reg in (False, True):
        if reg:
            for w, s in zip(mats, scs):
                gcu.register_weight(w, s)
        ys = gcu.gemv_int8_multi(mats, scs, golden["multi_x"], golden["multi_xs"])
        for j in range(3):
            assert_bits(ys[j], golden[f"multi_y{j}"])
    for w in mats:
        gcu.unregister_weight(w)


@pytest.mark.parametrize("n,k", [(262144, 640), (262144, 2560), (2048, 640), (640, 2048), (1536, 1152),
                                 (3840, 15360), (1000, 4304), (257, 1024), (77, 48),
                                 # streamed sets whose row fits one round of 5 / 8 chunks per lane
                                 (262144, 1152), (40000, 896), (20000, 1920)])
def test_gemv_registered(n, k):
    w, ws = big_weight(2000 + n % 997 + k, n, k)
    gcu.register_weight(w, ws)
    try:
        xq, xs = O.quantize_act(synth.activations(3000 + k, 1, k)[0])
        y = gcu.gemv_int8(w, ws, xq, xs)
        assert_bits(y, O.gemv_int8(w, ws, xq, xs))
        # interior pointer of the registered range (gemma.c:5080-5086 style)
        r0 = n // 2
        y2 = gcu.gemv_int8(w[r0:], ws[r0:], xq, xs)
        assert_bits(y2, O.gemv_int8(w[r0:], ws[r0:], xq, xs))
    finally:
        gcu.unregister_weight(w)


@pytest.mark.parametrize("m", [2, 3, 4, 5, 8])
def test_small_batch_gemm_uses_gemv_kernel(m):
    n, k = 4096, 2560
    w, ws = synth.weight(4000 + m, n, k)
    xq, xs = O.quantize_acts(synth.activations(4100 + m, m, k))
    y = gcu.gemm_int8(w, ws, xq, xs)
    assert_bits(y, O.gemm_int8(w, ws, xq, xs))


@pytest.mark.parametrize("m,n,k", [(3, 16384, 2560), (8, 16384, 2560), (6, 60000, 640)])
def test_small_batch_gemm_streamed_set(m, n, k):
    # weight sets above the L2 prefetch bound take the four-chunk streaming split
    w, ws = big_weight(4200 + m + k, n, k)
    xq, xs = O.quantize_acts(synth.activations(4300 + m, m, k))
    y = gcu.gemm_int8(w, ws, xq, xs)
    assert_bits(y, O.gemm_int8(w, ws, xq, xs))


# ---------------------------------------------------------------- GEMM

@pytest.mark.parametrize("name", ["gemm_a", "gemm_b", "gemm_d"])
def test_gemm_golden(golden, name):
    g = lambda k: golden[f"{name}_{k}"]
    y = gcu.gemm_int8(g("w"), g("ws"), g("x"), g("xs"))
    assert_bits(y, g("y"))


def test_gemm_strided_golden(golden):
    m, n, k, dstr, mstr, sstr = (int(v) for v in golden["gemm_c_dims"])
    dst = np.full((m, dstr), -1.0, np.float32)
    gcu.gemm_int8(golden["gemm_c_w"].reshape(-1), golden["gemm_c_ws"], golden["gemm_c_x"].reshape(-1),
                  golden["gemm_c_xs"], dst=dst, dstr=dstr, mstr=mstr, sstr=sstr, m=m, n=n, k=k)
    assert_bits(dst, golden["gemm_c_y"])


@pytest.mark.parametrize("m,n,k", [(128, 256, 640), (512, 1024, 1152), (512, 6912, 1152), (512, 1152, 6912),
                                   (77, 100, 4304), (300, 520, 1040), (9, 16, 128), (130, 24, 160),
                                   (1000, 260, 33), (256, 4304, 1152)])
def test_gemm_random(m, n, k):
    w, ws = synth.weight(5000 + n + k, n, k)
    xq, xs = O.quantize_acts(synth.activations(5100 + m + k, m, k, outliers=True))
    gcu.register_weight(w, ws)
    try:
        y = gcu.gemm_int8(w, ws, xq, xs)
    finally:
        gcu.unregister_weight(w)
    assert_bits(y, O.gemm_int8(w, ws, xq, xs))


@pytest.mark.parametrize("m,n,k,pad", [(4, 4096, 2560, 2), (1, 640, 1024, 0), (300, 1000, 1168, 3),
                                       (512, 1024, 1152, 0), (512, 1152, 6912, 0), (130, 24, 160, 1),
                                       (77, 100, 4304, 0), (512, 6912, 1152, 0)])
def test_host_calls_write_pinned_outputs(m, n, k, pad):
    # the host-pointer entry points with page-locked caller buffers (the
    # transfers then run straight from and into them), a padded output
    # stride, the GEMV, one-CTA, split-K and row-chunked GEMM paths
    x = synth.activations(3700 + m + k, m, k, outliers=True)
    w, ws = synth.weight(3701 + n + k, n, k)
    gcu.register_weight(w, ws)
    try:
        q = torch.empty((m, k), dtype=torch.int8, pin_memory=True).numpy()
        s = torch.empty(m, dtype=torch.float32, pin_memory=True).numpy()
        dst = torch.full((m, n + pad), float("nan"), dtype=torch.float32, pin_memory=True).numpy()
        q0, s0 = O.quantize_acts(x)
        y0 = O.gemm_int8(w, ws, q0, s0)
        for _ in range(2):
            q[:] = 99
            gcu.quantize_acts(x, dst=q, dsc=s)
            assert np.array_equal(q, q0) and np.array_equal(bits(s), bits(s0))
            dst[:, :n] = float("nan")
            gcu.gemm_int8(w, ws, q, s, dst=dst, dstr=n + pad, m=m, n=n, k=k)
            assert_bits(dst[:, :n], y0)
            assert np.isnan(dst[:, n:]).all()  # the padding columns are left alone
    finally:
        gcu.unregister_weight(w)


@pytest.mark.parametrize("m,n,k,pad", [(600, 2500, 640, 0), (300, 4000, 640, 5), (129, 9000, 128, 3)])
def test_gemm_host_pipelined(m, n, k, pad):
    # > 4 MB of output: the host call runs 128-row chunks whose copies overlap
    # the GEMM of the next chunk; a padded dst stride keeps the gaps untouched
    w, ws = synth.weight(5600 + n, n, k)
    xq, xs = O.quantize_acts(synth.activations(5700 + m, m, k, outliers=True))
    dst = np.full((m, n + pad), -7.0, np.float32)
    gcu.register_weight(w, ws)
    try:
        gcu.gemm_int8(w.reshape(-1), ws, xq.reshape(-1), xs, dst=dst, dstr=n + pad, m=m, n=n, k=k)
    finally:
        gcu.unregister_weight(w)
    assert_bits(dst[:, :n], O.gemm_int8(w, ws, xq, xs))
    assert (dst[:, n:] == -7.0).all()


def test_gemm_prefill_qkv_head_blocks():
    # gemma.c:5045-5091: per (head, 128-token block) calls with interior
    # weight/scale pointers and dst stride hdim, from several host threads
    ntok, dim, hdim, heads = 300, 1152, 256, 4
    w, ws = synth.weight(6000, heads * hdim, dim)
    xq, xs = O.quantize_acts(synth.activations(6001, ntok, dim))
    gcu.register_weight(w, ws)
    out = np.zeros((heads, ntok, hdim), np.float32)
    errs = []

    def task(h, t0):
        tn = min(128, ntok - t0)
        try:
            dst = out[h, t0:t0 + tn]
            gcu.gemm_int8(w[h * hdim:(h + 1) * hdim], ws[h * hdim:(h + 1) * hdim], xq[t0:t0 + tn],
                          xs[t0:t0 + tn], dst=dst)
        except Exception as e:  # noqa: BLE001
            errs.append(e)

    threads = [threading.Thread(target=task, args=(h, t0)) for h in range(heads) for t0 in range(0, ntok, 128)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    gcu.unregister_weight(w)
    assert not errs, errs
    ref = O.gemm_int8(w, ws, xq, xs).reshape(ntok, heads, hdim).transpose(1, 0, 2)
    assert_bits(out, ref)


def test_int32_accumulators_exact():
    # unit scales make the fp32 output the int32 sum itself (|acc| < 2^24)
    m, n, k = 256, 384, 1024
    rng = np.random.default_rng(7)
    a = rng.integers(-127, 128, (m, k), dtype=np.int8)
    b = rng.integers(-127, 128, (n, k), dtype=np.int8)
    one_m = np.ones(m, np.float32)
    one_n = np.ones(n, np.float32)
    y = gcu.gemm_int8(b, one_n, a, one_m)
    acc = O.acc_int8(b, a)
    assert np.abs(acc).max() < 2 ** 24
    assert np.array_equal(y.astype(np.int64), acc.astype(np.int64))
    yv = gcu.gemv_int8(b, one_n, a[0], 1.0)
    assert np.array_equal(yv.astype(np.int64), acc[0].astype(np.int64))


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("bn,split,mb", [(128, 1, 1), (256, 1, 1), (128, 3, 1), (256, 2, 1), (128, 7, 1),
                                         (64, 1, 1), (64, 3, 1), (128, 1, 2), (192, 1, 2), (256, 1, 2),
                                         (192, 3, 2), (128, 2, 2),
                                         (128, 1, 4), (192, 1, 4), (256, 1, 4)])  # mb 4: CTA-pair tiles
def test_gemm_tile_and_split_variants(bn, split, mb):
    # m = 384 leaves a half-empty last 256-row tile for mb = 2
    m, n, k = 384, 1000, 2304
    w, ws = synth.weight(7000 + bn + split, n, k)
    xq, xs = O.quantize_acts(synth.activations(7100, m, k, outliers=True))
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    gcu.dev_gemm_int8_tuned(y, _dev(w), _dev(ws), _dev(xq), _dev(xs), m, n, k, bn, split, mb)
    torch.cuda.synchronize()
    gcu.check_device()
    assert_bits(y.cpu().numpy(), O.gemm_int8(w, ws, xq, xs))


@pytest.mark.parametrize("m,n,bn,split,mb", [
    (128, 1000, 64, 9, 1),    # one wave, more splits than 32x32 blocks per tile
    (384, 1000, 256, 8, 1),   # one wave, splits summed in two batches of four
    (40, 1000, 128, 4, 1),    # rows past m in every tile
    (384, 999, 128, 3, 1),    # odd row stride: plain stores instead of TMA
    (384, 999, 128, 9, 1),    # more units than SMs: the last split reduces
])
def test_gemm_split_k_reductions(m, n, bn, split, mb):
    k = 2304
    w, ws = synth.weight(7200 + n + split, n, k)
    xq, xs = O.quantize_acts(synth.activations(7300 + m, m, k, outliers=True))
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    for _ in range(2):  # the second call checks the counters were reset
        y.fill_(float("nan"))
        gcu.dev_gemm_int8_tuned(y, _dev(w), _dev(ws), _dev(xq), _dev(xs), m, n, k, bn, split, mb)
        torch.cuda.synchronize()
        gcu.check_device()
        assert_bits(y.cpu().numpy(), O.gemm_int8(w, ws, xq, xs))


def test_device_chain_quantize_then_multi_gemm():
    # prefill Q/K/V as one launch over three weights sharing the input
    m, dim = 512, 1152
    x = synth.activations(8000, m, dim, outliers=True)
    shapes = [("wq", 1024), ("wk", 256), ("wv", 256)]
    ws_np = [synth.weight(8001 + i, n, dim) for i, (_, n) in enumerate(shapes)]
    xt = _dev(x)
    q = torch.empty((m, dim), dtype=torch.int8, device="cuda")
    s = torch.empty(m, dtype=torch.float32, device="cuda")
    gcu.dev_quantize_acts(q, s, xt, m, dim)
    outs = [torch.empty((m, n), dtype=torch.float32, device="cuda") for _, n in shapes]
    jobs = [(_dev(w), _dev(sc), o) for (w, sc), o in zip(ws_np, outs)]
    gcu.dev_gemm_int8_multi(jobs, q, s, m, dim)
    torch.cuda.synchronize()
    gcu.check_device()
    xq, xs = O.quantize_acts(x)
    assert np.array_equal(q.cpu().numpy(), xq)
    for (w, sc), o in zip(ws_np, outs):
        assert_bits(o.cpu().numpy(), O.gemm_int8(w, sc, xq, xs))


def test_device_gemv_multi_and_scale_pointer():
    k = 640
    x = synth.activations(8100, 1, k)[0]
    ws_np = [synth.weight(8101 + i, n, k) for i, n in enumerate((1024, 256, 256))]
    q = torch.empty(k, dtype=torch.int8, device="cuda")
    s = torch.empty(1, dtype=torch.float32, device="cuda")
    gcu.dev_quantize_acts(q, s, _dev(x), 1, k)
    outs = [torch.empty(w.shape[0], dtype=torch.float32, device="cuda") for w, _ in ws_np]
    gcu.dev_gemv_int8_multi([(_dev(w), _dev(sc), o) for (w, sc), o in zip(ws_np, outs)], q, s, k)
    torch.cuda.synchronize()
    xq, xs = O.quantize_act(x)
    for (w, sc), o in zip(ws_np, outs):
        assert_bits(o.cpu().numpy(), O.gemv_int8(w, sc, xq, xs))


def test_full_size_gemm_sampled_rows():
    # 12B prefill gate at full size (M=4096, N=15360, K=3840): the oracle
    # recomputes a seeded sample of rows; every sampled output must match.
    m, n, k = 4096, 15360, 3840
    gen = torch.Generator(device="cuda").manual_seed(11)
    w, ws = synth.weight_torch(n, k, gen, "cuda")
    x = synth.activations_torch(m, k, gen, "cuda")
    q = torch.empty((m, k), dtype=torch.int8, device="cuda")
    s = torch.empty(m, dtype=torch.float32, device="cuda")
    gcu.dev_quantize_acts(q, s, x, m, k)
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    gcu.dev_gemm_int8(y, w, ws, q, s, m, n, k)
    torch.cuda.synchronize()
    gcu.check_device()
    rows = np.random.default_rng(3).choice(m, 12, replace=False)
    rows.sort()
    xq, xs = O.quantize_acts(x[rows].cpu().numpy())
    assert np.array_equal(q[rows].cpu().numpy(), xq)
    ref = O.gemm_int8(w.cpu().numpy(), ws.cpu().numpy(), xq, xs)
    assert_bits(y[rows].cpu().numpy(), ref)


# every distinct GEMM of BASELINE configs[3] (Gemma-3-4B text at M=2048 and
# the SigLIP-So400m tower at M=4096, projector at M=256) and configs[4]
# (Gemma-3-12B at M=4096, FFN row slices of 2/4/8 GPUs), at full size
FULL_SHAPES = [
    (2048, (2048, 1024, 1024), 2560), (2048, (2560,), 2048), (2048, (10240, 10240), 2560),
    (2048, (2560,), 10240),
    (4096, (1152, 1152, 1152), 1152), (4096, (1152,), 1152), (4096, (4304,), 1152), (4096, (1152,), 4304),
    (256, (2560,), 1152),
    (4096, (4096, 2048, 2048), 3840), (4096, (3840,), 4096), (4096, (15360, 15360), 3840),
    (4096, (3840,), 15360),
    (4096, (7680, 7680), 3840), (4096, (1920, 1920), 3840), (4096, (1920,), 15360), (4096, (480,), 15360),
]


@pytest.mark.parametrize("m,ns,k", FULL_SHAPES)
def test_full_size_config_shapes_sampled_rows(m, ns, k):
    # the quantize kernel and one multi-weight launch at full size; the oracle
    # recomputes a seeded sample of rows of every output
    gen = torch.Generator(device="cuda").manual_seed(m + k + sum(ns))
    ws_t = [synth.weight_torch(n, k, gen, "cuda") for n in ns]
    x = synth.activations_torch(m, k, gen, "cuda", outliers=True)
    q = torch.empty((m, k), dtype=torch.int8, device="cuda")
    s = torch.empty(m, dtype=torch.float32, device="cuda")
    ys = [torch.empty((m, n), dtype=torch.float32, device="cuda") for n in ns]
    gcu.dev_quantize_gemm_int8_multi([(w, sc, y) for (w, sc), y in zip(ws_t, ys)], q, s, x, m, k)
    torch.cuda.synchronize()
    gcu.check_device()
    rows = np.sort(np.random.default_rng(m + k).choice(m, 8, replace=False))
    xq, xs = O.quantize_acts(x[rows].cpu().numpy())
    assert np.array_equal(q[rows].cpu().numpy(), xq)
    assert_bits(s[rows].cpu().numpy(), xs)
    for (w, sc), y in zip(ws_t, ys):
        assert_bits(y[rows].cpu().numpy(), O.gemm_int8(w.cpu().numpy(), sc.cpu().numpy(), xq, xs))


def _rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("m,dim,xpad", [(1, 640, 0), (4, 1152, 0), (37, 2560, 8), (5, 3840, 0),
                                        (3, 15360, 0), (300, 1152, 4), (2, 40, 0)])
def test_rmsnorm_quantize_fused(m, dim, xpad):
    # the fused kernel's fp32 output within BASELINE's 1e-5 relative of the
    # reference's rmsnorm; its codes and scales are exactly quantize_acts of
    # that output; against the reference the codes differ by at most one
    xstr = dim + xpad
    x = synth.activations(3300 + dim, m, xstr, outliers=True)
    w = (synth.activations(3301 + dim, 1, dim)[0] * 0.1).astype(np.float32)
    xt, wt = _dev(x), _dev(w)
    q = torch.empty((m, dim), dtype=torch.int8, device="cuda")
    s = torch.empty(m, dtype=torch.float32, device="cuda")
    xn = torch.empty((m, dim), dtype=torch.float32, device="cuda")
    gcu.dev_rmsnorm_quantize(q, s, xt, wt, 1e-6, m, dim, out=xn, xstr=xstr)
    torch.cuda.synchronize()
    gcu.check_device()
    xn_g, q_g, s_g = xn.cpu().numpy(), q.cpu().numpy(), s.cpu().numpy()
    q_e, s_e = O.quantize_acts(xn_g)
    assert np.array_equal(q_g, q_e) and np.array_equal(bits(s_g), bits(s_e))
    xn_o, q_o, s_o = O.rmsnorm_quantize(np.ascontiguousarray(x[:, :dim]), w, 1e-6)
    assert _rel(xn_g, xn_o) < 1e-5 and _rel(s_g, s_o) < 1e-5
    assert np.abs(q_g.astype(int) - q_o).max() <= 1 and (q_g != q_o).mean() < 1e-3


@pytest.mark.parametrize("m,dim", [(1, 2048), (2, 6912), (8, 10240), (512, 6912), (3, 15360), (5, 40)])
def test_geglu_quantize_fused(m, dim):
    g = synth.activations(3400 + dim, m, dim)
    u = synth.activations(3401 + dim, m, dim)
    q = torch.empty((m, dim), dtype=torch.int8, device="cuda")
    s = torch.empty(m, dtype=torch.float32, device="cuda")
    h = torch.empty((m, dim), dtype=torch.float32, device="cuda")
    gcu.dev_geglu_quantize(q, s, _dev(g), _dev(u), m, dim, out=h)
    torch.cuda.synchronize()
    gcu.check_device()
    h_g, q_g, s_g = h.cpu().numpy(), q.cpu().numpy(), s.cpu().numpy()
    q_e, s_e = O.quantize_acts(h_g)
    assert np.array_equal(q_g, q_e) and np.array_equal(bits(s_g), bits(s_e))
    h_o, q_o, s_o = O.geglu_quantize(g, u)
    assert _rel(h_g, h_o) < 1e-5 and _rel(s_g, s_o) < 1e-5
    assert np.abs(q_g.astype(int) - q_o).max() <= 1 and (q_g != q_o).mean() < 1e-3
    # without the optional fp32 output the codes are the same
    q2 = torch.empty_like(q)
    s2 = torch.empty_like(s)
    gcu.dev_geglu_quantize(q2, s2, _dev(g), _dev(u), m, dim)
    torch.cuda.synchronize()
    assert torch.equal(q2, q) and torch.equal(s2, s)


def test_producers_reject_unsupported_rows():
    x = torch.zeros((2, 18), dtype=torch.float32, device="cuda")
    q = torch.empty((2, 18), dtype=torch.int8, device="cuda")
    s = torch.empty(2, dtype=torch.float32, device="cuda")
    with pytest.raises(gcu.GcuError, match="multiple of 4"):
        gcu.dev_rmsnorm_quantize(q, s, x, x[0], 1e-6, 2, 18)
    with pytest.raises(gcu.GcuError, match="multiple of 4"):
        gcu.dev_geglu_quantize(q, s, x, x, 2, 18)


def test_scale_linearity_property():
    # doubling every weight scale doubles every output exactly
    m, n, k = 256, 2048, 2048
    w, ws = synth.weight(9000, n, k)
    xq, xs = O.quantize_acts(synth.activations(9001, m, k))
    y1 = gcu.gemm_int8(w, ws, xq, xs)
    y2 = gcu.gemm_int8(w, (ws * 2).astype(np.float32), xq, xs)
    assert np.array_equal(bits(y2), bits(y1 * 2))


def test_error_reported_for_unsupported_device_call():
    w = torch.zeros((16, 64), dtype=torch.int8, device="cuda")
    sc = torch.ones(16, device="cuda")
    x = torch.zeros((2, 64), dtype=torch.int8, device="cuda")
    xs = torch.ones(2, device="cuda")
    y = torch.empty((2, 16), device="cuda")
    with pytest.raises(gcu.GcuError, match="dense weight rows"):
        gcu.dev_gemm_int8(y, w, sc, x, xs, 2, 16, 32, mstr=64)


# ---------------------------------------------------------------- fused quantize + matmul

@pytest.mark.parametrize("m,k,rows", [(1, 640, (1024, 256, 256)), (1, 2560, (262144,)), (4, 1152, (2048,)),
                                      (3, 1152, (512, 256)), (300, 1152, (1024, 256, 256)),
                                      (512, 1152, (6912, 6912)), (512, 6912, (1152,)), (1000, 2560, (640,)),
                                      (6, 40, (48,)), (77, 4304, (100, 60)), (1, 640, (262144,)),
                                      (2, 1152, (40000,))])
def test_fused_quantize_gemm(m, k, rows):
    x = synth.activations(9100 + m + k, m, k, outliers=True)
    ws_np = [big_weight(9200 + i + k, n, k) for i, n in enumerate(rows)]
    q = torch.full((m, k), 99, dtype=torch.int8, device="cuda")
    s = torch.zeros(m, dtype=torch.float32, device="cuda")
    outs = [torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda") for n in rows]
    jobs = [(_dev(w), _dev(sc), o) for (w, sc), o in zip(ws_np, outs)]
    xt = _dev(x)
    for _ in range(2):  # the grid barrier and counters are reused by the second call
        gcu.dev_quantize_gemm_int8_multi(jobs, q, s, xt, m, k)
        torch.cuda.synchronize()
    gcu.check_device()
    xq, xs = O.quantize_acts(x)
    assert np.array_equal(q.cpu().numpy(), xq)
    assert_bits(s.cpu().numpy(), xs)
    for (w, sc), o in zip(ws_np, outs):
        assert_bits(o.cpu().numpy(), O.gemm_int8(w, sc, xq, xs))


def test_fused_quantize_gemm_rejects_odd_k_on_tensor_cores():
    m, k = 130, 40
    x = torch.zeros((m, k), dtype=torch.float32, device="cuda")
    q = torch.empty((m, k), dtype=torch.int8, device="cuda")
    s = torch.empty(m, dtype=torch.float32, device="cuda")
    w = torch.zeros((48, k), dtype=torch.int8, device="cuda")
    sc = torch.ones(48, device="cuda")
    o = torch.empty((m, 48), device="cuda")
    with pytest.raises(gcu.GcuError, match="k % 16 == 0"):
        gcu.dev_quantize_gemm_int8_multi([(w, sc, o)], q, s, x, m, k)
