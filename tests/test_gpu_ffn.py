"""The FFN block entry point and the raw int32 GEMM mode it is built on.

gcu_dev_ffn_rowshard runs Gemma's feed-forward block (up and gate, GeGLU,
quantize_acts, down) with the hidden dimension split over the ranks of
gcu_comm_init; without it, unsharded.  The sharded form sums the down
projection's int32 partial products over the ranks, so the GEMM must be able
to write the int32 sums themselves: those are checked against the oracle's
exact accumulators on every one-CTA tile shape and K split, and the
unsharded block against the step-by-step calls bit for bit.  The two-rank
form is tests/test_gpu_ffn_rowshard.py.
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


@pytest.mark.parametrize("m,n,k,bn,split,mb", [
    (300, 1000, 1168, 64, 1, 1), (512, 1152, 7680, 128, 4, 1), (512, 1152, 7680, 0, 0, 0),
    (256, 2048, 1920, 192, 1, 2), (1024, 3840, 1920, 256, 1, 2), (130, 480, 3840, 128, 3, 1),
    (4096, 3840, 7680, 0, 0, 0)])
def test_raw_int32_sums_are_exact(m, n, k, bn, split, mb):
    # the sums past 2^24 (k = 7680: up to 1.2e8) that an fp32 output could not hold
    gen = torch.Generator(device="cuda").manual_seed(m + n + k)
    w = torch.randint(-127, 128, (n, k), generator=gen, device="cuda", dtype=torch.int8)
    x = torch.randint(-127, 128, (m, k), generator=gen, device="cuda", dtype=torch.int8)
    # saturated rows: sums of +-k * 127^2 (past 2^24 once k > 1040)
    x[0], x[1], w[0], w[1] = 127, -127, 127, -127
    if m * n * k > (1 << 33):  # the oracle recomputes sampled rows of the largest case
        rows = np.sort(np.concatenate([[0, 1], np.random.default_rng(1).choice(np.arange(2, m), 14, replace=False)]))
    else:
        rows = np.arange(m)
    acc = torch.empty((m, n), dtype=torch.int32, device="cuda")
    gcu.dev_gemm_int8_raw_tuned(acc, w, x, m, n, k, bn, split, mb)
    torch.cuda.synchronize()
    gcu.check_device()
    want = O.acc_int8(w.cpu().numpy(), x[rows].cpu().numpy())
    got = acc[rows].cpu().numpy()
    assert np.array_equal(got, want), f"{int((got != want).sum())} of {got.size} sums differ"
    assert abs(int(want[0, 0])) == k * 127 * 127 and (k * 127 * 127 > (1 << 24) or k < 1100)


def test_raw_int32_sums_have_no_pair_tile():
    w = torch.zeros((256, 1024), dtype=torch.int8, device="cuda")
    x = torch.zeros((256, 1024), dtype=torch.int8, device="cuda")
    acc = torch.empty((256, 256), dtype=torch.int32, device="cuda")
    with pytest.raises(gcu.GcuError, match="CTA-pair"):
        gcu.dev_gemm_int8_raw_tuned(acc, w, x, 256, 256, 1024, 256, 1, 4)


def _ffn_weights(gen, dim, ffn):
    w1 = synth.weight_torch(ffn, dim, gen, "cuda")   # up
    w2 = synth.weight_torch(ffn, dim, gen, "cuda")   # gate
    w3 = synth.weight_torch(dim, ffn, gen, "cuda")   # down
    return w1, w2, w3


def _stepwise(xq, xs, m, dim, ffn, w1, w2, w3):
    up = torch.empty((m, ffn), device="cuda")
    gate = torch.empty((m, ffn), device="cuda")
    gcu.dev_gemm_int8_multi([(w1[0], w1[1], up), (w2[0], w2[1], gate)], xq, xs, m, dim)
    hq = torch.empty((m, ffn), dtype=torch.int8, device="cuda")
    hs = torch.empty(m, device="cuda")
    gcu.dev_geglu_quantize(hq, hs, gate, up, m, ffn)
    out = torch.empty((m, dim), device="cuda")
    gcu.dev_gemm_int8(out, w3[0], w3[1], hq, hs, m, dim, ffn)
    return out, hq, hs


@pytest.mark.parametrize("m,dim,ffn", [(512, 1152, 6912), (300, 640, 2048), (2048, 2560, 10240)])
def test_ffn_unsharded_equals_the_step_by_step_calls(m, dim, ffn):
    gen = torch.Generator(device="cuda").manual_seed(m + dim)
    w1, w2, w3 = _ffn_weights(gen, dim, ffn)
    x = synth.activations_torch(m, dim, gen, "cuda", outliers=True)
    xq = torch.empty((m, dim), dtype=torch.int8, device="cuda")
    xs = torch.empty(m, device="cuda")
    gcu.dev_quantize_acts(xq, xs, x, m, dim)
    want, _, _ = _stepwise(xq, xs, m, dim, ffn, w1, w2, w3)
    out = torch.full((m, dim), float("nan"), device="cuda")
    for _ in range(2):
        gcu.dev_ffn_rowshard(out, xq, xs, m, dim, ffn, w1[0], w1[1], w2[0], w2[1], w3[0], w3[1])
    torch.cuda.synchronize()
    gcu.check_device()
    assert torch.equal(out.view(torch.int32), want.view(torch.int32))


def test_ffn_rejects_what_it_cannot_run():
    gen = torch.Generator(device="cuda").manual_seed(3)
    w1, w2, w3 = _ffn_weights(gen, 640, 2048)
    xq = torch.zeros((8, 640), dtype=torch.int8, device="cuda")
    xs = torch.ones(8, device="cuda")
    out = torch.empty((8, 640), device="cuda")
    with pytest.raises(gcu.GcuError, match="m > 8"):
        gcu.dev_ffn_rowshard(out, xq, xs, 8, 640, 2048, w1[0], w1[1], w2[0], w2[1], w3[0], w3[1])
