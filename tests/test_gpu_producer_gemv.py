"""A producer row and the decode GEMV that consumes it, in one launch
(gcu_dev_geglu_quantize_gemv_multi, gcu_dev_residual_norm_quantize_gemv_multi).

Every CTA of the GEMV computes the producer row itself -- GeGLU (gemma.c:4921-
4927), or the residual update with the next block's RMSNorm (gemma.c:4862-4910,
4950-4962 + 4754-4768) -- with the arithmetic of the standalone producer
kernels, so the codes, the scale, the updated residual and every GEMV output
must be bit for bit those of the two-launch sequence (gcu_dev_geglu_quantize /
gcu_dev_residual_norm_quantize, then gcu_dev_gemv_int8_multi), which the
parity tests pin to the reference.  The oracle also recomputes sampled output
rows from the fused launch's own codes.  Shapes: the Gemma 3 270m / 1B / 4B /
12B hidden and FFN widths.
"""
import numpy as np
import pytest

import oracle as O
import synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import gcu  # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    gcu.init(0)
    yield
    gcu.check_device()


def same(got, want, what):
    g = got.contiguous().view(torch.int32) if got.dtype == torch.float32 else got.contiguous()
    w = want.contiguous().view(torch.int32) if want.dtype == torch.float32 else want.contiguous()
    bad = g != w
    if bool(bad.any()):
        raise AssertionError(f"{what}: {int(bad.sum())} of {bad.numel()} differ, first "
                             f"{torch.nonzero(bad)[:3].tolist()}")


def weights(gen, ns, k):
    return [synth.weight_torch(n, k, gen, "cuda") for n in ns]


def oracle_rows(ws, q, s, outs, nrows=24, seed=0):
    rng = np.random.default_rng(seed)
    qn, sn = q.view(1, -1).cpu().numpy(), s.view(1).cpu().numpy()
    for (w, sc), o in zip(ws, outs):
        rows = np.sort(rng.choice(w.shape[0], min(nrows, w.shape[0]), replace=False))
        want = O.gemm_int8(w[rows].cpu().numpy(), sc[rows].cpu().numpy(), qn, sn)[0]
        got = o.view(-1)[rows].cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# (k = the FFN width, down-projection rows = the hidden width)
@pytest.mark.parametrize("k,ns", [(2048, (640,)), (6912, (1152,)), (10240, (2560,)), (15360, (3840,)),
                                  (16384, (100, 60)), (48, (16,))])
def test_geglu_gemv_equals_two_launches(k, ns):
    gen = torch.Generator(device="cuda").manual_seed(k + sum(ns))
    gate = synth.activations_torch(1, k, gen, "cuda")
    up = synth.activations_torch(1, k, gen, "cuda")
    ws = weights(gen, ns, k)
    # two launches: the producer kernel, then the GEMV
    q0 = torch.empty((1, k), dtype=torch.int8, device="cuda")
    s0 = torch.empty(1, device="cuda")
    gcu.dev_geglu_quantize(q0, s0, gate, up, 1, k)
    ref = [torch.empty(n, device="cuda") for n in ns]
    gcu.dev_gemv_int8_multi([(w, sc, o) for (w, sc), o in zip(ws, ref)], q0, s0, k)
    # one launch
    q = torch.full((1, k), 99, dtype=torch.int8, device="cuda")
    s = torch.full((1,), float("nan"), device="cuda")
    outs = [torch.full((n,), float("nan"), device="cuda") for n in ns]
    for _ in range(2):
        gcu.dev_geglu_quantize_gemv_multi([(w, sc, o) for (w, sc), o in zip(ws, outs)], q, s, gate, up, k)
    torch.cuda.synchronize()
    gcu.check_device()
    same(q, q0, "codes")
    same(s, s0, "scale")
    for i, (o, r) in enumerate(zip(outs, ref)):
        same(o, r, f"job {i}")
    oracle_rows(ws, q, s, outs)


@pytest.mark.parametrize("dim,ns,post", [(640, (2048, 2048), True), (1152, (1024, 256, 256), True),
                                         (1152, (6912, 6912), False), (2560, (2048, 1024, 1024), True),
                                         (3840, (4096,), True), (4096, (32,), False), (48, (16,), True),
                                         # streamed weight sets (over 32 MB): one round of 5 / 8 chunks
                                         (2560, (10240, 10240), True), (3840, (15360,), False)])
def test_residual_norm_gemv_equals_two_launches(dim, ns, post):
    gen = torch.Generator(device="cuda").manual_seed(dim + len(ns))
    y = synth.activations_torch(1, dim, gen, "cuda", outliers=True)
    resid = synth.activations_torch(1, dim, gen, "cuda")
    w_post = (synth.activations_torch(1, dim, gen, "cuda")[0] * 0.1).contiguous() if post else None
    w_next = (synth.activations_torch(1, dim, gen, "cuda")[0] * 0.1).contiguous()
    ws = weights(gen, ns, dim)
    # two launches (x in place over a copy of resid, as the decoder did)
    x0 = resid.clone()
    q0 = torch.empty((1, dim), dtype=torch.int8, device="cuda")
    s0 = torch.empty(1, device="cuda")
    gcu.dev_residual_norm_quantize(x0, q0, s0, y, x0, w_post, w_next, 1e-6, 1, dim)
    ref = [torch.empty(n, device="cuda") for n in ns]
    gcu.dev_gemv_int8_multi([(w, sc, o) for (w, sc), o in zip(ws, ref)], q0, s0, dim)
    # one launch, x out of place
    x = torch.full((1, dim), float("nan"), device="cuda")
    q = torch.full((1, dim), 99, dtype=torch.int8, device="cuda")
    s = torch.full((1,), float("nan"), device="cuda")
    outs = [torch.full((n,), float("nan"), device="cuda") for n in ns]
    for _ in range(2):
        gcu.dev_residual_norm_quantize_gemv_multi([(w, sc, o) for (w, sc), o in zip(ws, outs)], x, q, s, y, resid,
                                                  w_post, w_next, 1e-6, dim)
    torch.cuda.synchronize()
    gcu.check_device()
    same(x, x0, "residual")
    same(q, q0, "codes")
    same(s, s0, "scale")
    for i, (o, r) in enumerate(zip(outs, ref)):
        same(o, r, f"job {i}")
    oracle_rows(ws, q, s, outs, seed=1)


def test_staged_gemv_argument_checks():
    gen = torch.Generator(device="cuda").manual_seed(7)
    (w, sc), = weights(gen, (64,), 640)
    o = torch.empty(64, device="cuda")
    v = torch.zeros((1, 640), device="cuda")
    q = torch.empty((1, 640), dtype=torch.int8, device="cuda")
    s = torch.empty(1, device="cuda")
    # x may not alias the residual or y: other CTAs still read them
    with pytest.raises(gcu.GcuError, match="overlap"):
        gcu.dev_residual_norm_quantize_gemv_multi([(w, sc, o)], v, q, s, torch.zeros_like(v), v, None, v[0], 1e-6,
                                                  640)
    with pytest.raises(gcu.GcuError, match="multiple of 16"):
        gcu.dev_residual_norm_quantize_gemv_multi([(w, sc, o)], torch.zeros_like(v), q, s, v, v, None, v[0], 1e-6,
                                                  632)
    big = torch.zeros((1, 16400), device="cuda")
    with pytest.raises(gcu.GcuError, match="16384"):
        gcu.dev_geglu_quantize_gemv_multi([(w, sc, o)], q, s, big, big, 16400)
