"""GPU attention kernels (k_attention.cu) against the reference and the oracle.

Decode (gemma.c:4836-4848) and prefill (gemma.c:5160-5295) attention in fp32
through the C ABI.  The reference's dot products are vectorized under
-ffast-math, so agreement is to fp32 reassociation: max |gpu - reference|
<= 1e-5 * max |reference|, against the golden fixture made by the compiled
reference and against the oracle on larger seeded cases.  Size-independent
checks: all-ones V gives ones (the weights sum to one), a single visible
position returns its V row exactly.
"""
import json
import os

import numpy as np
import pytest

import oracle as O
import synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import gcu  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "attention.npz"))
META = json.loads(str(GOLD["meta"]))
TOL = 1e-5


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    gcu.init(0)
    yield
    gcu.check_device()


def assert_attn_close(got, want, tol=TOL):
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    assert got.shape == want.shape
    err = float(np.max(np.abs(got - want)))
    scale = float(np.max(np.abs(want)))
    assert np.all(np.isfinite(got)) and err <= tol * scale, f"max err {err:.3g} vs {tol} x {scale:.3g}"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_decode(xq, kc, vc, spos, attlen, asc, sc=0.0):
    xo = torch.empty(xq.shape, device="cuda")
    gcu.dev_attention_decode(xo, dev(xq), dev(kc), dev(vc), spos, attlen, float(asc), sc)
    torch.cuda.synchronize()
    return xo.cpu().numpy()


def run_prefill(xq, kc, vc, spos, slide=0, sc=0.0, mask=True):
    nh, ntok, hd = xq.shape
    xo = torch.empty((ntok, nh * hd), device="cuda")
    gcu.dev_attention_prefill(xo, dev(xq), dev(kc), dev(vc), spos, slide, sc, mask)
    torch.cuda.synchronize()
    return xo.cpu().numpy()


@pytest.mark.parametrize("case", META["decode"], ids=lambda c: f"decode{c[0]}")
def test_decode_matches_reference_fixture(case):
    tid, nh, nkv, hd, clen, spos, attlen, sc = case
    xq, kc, vc = synth.attention_inputs(tid, nh, nkv, hd, clen)
    assert_attn_close(run_decode(xq, kc, vc, spos, attlen, np.float32(1.0 / np.sqrt(hd)), sc),
                      GOLD[f"decode_{tid}"])


@pytest.mark.parametrize("case", META["prefill"], ids=lambda c: f"prefill{c[0]}")
def test_prefill_matches_reference_fixture(case):
    tid, nh, nkv, hd, spos, ntok, slide, sc, mask = case
    xq, kc, vc = synth.attention_inputs(tid, nh, nkv, hd, spos + ntok + 3, ntok)
    assert_attn_close(run_prefill(xq, kc, vc, spos, slide, sc, bool(mask)), GOLD[f"prefill_{tid}"])


# Gemma 3 decode shapes (heads, kv heads, head size) at several window lengths,
# including windows that split over many CTAs and a sliding-window start
@pytest.mark.parametrize("nh,nkv,hd,clen,spos,attlen,sc", [
    (4, 1, 256, 64, 0, 64, 0.0), (4, 1, 256, 65, 0, 65, 0.0), (4, 1, 256, 4096, 3000, 512, 0.0),
    (8, 4, 256, 8192, 0, 8192, 0.0), (16, 8, 256, 6000, 0, 6000, 50.0), (16, 8, 128, 777, 11, 700, 0.0),
    (5, 1, 64, 3000, 0, 2999, 0.0), (6, 4, 128, 2000, 0, 2000, 0.0)])  # last: uneven groups
def test_decode_matches_oracle(nh, nkv, hd, clen, spos, attlen, sc):
    xq, kc, vc = synth.attention_inputs(300 + attlen, nh, nkv, hd, clen)
    asc = np.float32(1.0 / np.sqrt(hd))
    assert_attn_close(run_decode(xq, kc, vc, spos, attlen, asc, sc),
                      O.attention_decode(xq, kc, vc, spos, attlen, asc, sc))


@pytest.mark.parametrize("nh,nkv,hd,spos,ntok,slide,sc,mask", [
    (4, 1, 256, 0, 512, 512, 0.0, True),     # Gemma-3-1B prefill chunk (config 1 shape)
    (4, 1, 256, 600, 200, 512, 0.0, True),   # a later chunk on a sliding layer
    (8, 4, 256, 0, 300, 0, 0.0, True),       # 4B heads, global layer
    (8, 4, 128, 13, 77, 20, 30.0, True),
    (2, 1, 64, 0, 100, 0, 0.0, False),
    (6, 4, 64, 0, 70, 0, 0.0, True),       # uneven query-head groups
    (4, 1, 256, 0, 2048, 0, 0.0, True),    # 32 key tiles: chunks of 4 tiles each
    (2, 1, 128, 0, 700, 0, 0.0, False)])   # 11 tiles: chunks of 2, the last of one
def test_prefill_matches_oracle(nh, nkv, hd, spos, ntok, slide, sc, mask):
    xq, kc, vc = synth.attention_inputs(400 + ntok, nh, nkv, hd, spos + ntok, ntok)
    assert_attn_close(run_prefill(xq, kc, vc, spos, slide, sc, mask),
                      O.attention_prefill(xq, kc, vc, spos, slide, sc, mask))


def test_weights_sum_to_one():
    # all-ones V: every output is sum(p_t)/sum(p_t), 1 to rounding, at any length
    xq, kc, _ = synth.attention_inputs(500, 4, 2, 256, 32768)
    ones = np.ones_like(kc)
    out = run_decode(xq, kc, ones, 0, 32768, np.float32(1 / 16))
    assert np.max(np.abs(out - 1.0)) < 1e-5
    xq, kc, _ = synth.attention_inputs(501, 4, 1, 256, 2048, 1024)
    out = run_prefill(xq, kc, np.ones_like(kc), 1024, 512)
    assert np.max(np.abs(out - 1.0)) < 1e-5


def test_single_position_returns_value_row():
    xq, kc, vc = synth.attention_inputs(502, 4, 2, 64, 10)
    got = run_decode(xq, kc, vc, 6, 1, np.float32(0.125))
    assert np.array_equal(got, np.repeat(vc[:, 6, :], 2, axis=0))
    xq, kc, vc = synth.attention_inputs(503, 2, 1, 128, 1, 1)
    assert np.array_equal(run_prefill(xq, kc, vc, 0), np.concatenate([vc[0, 0], vc[0, 0]])[None])


def test_prefill_output_stride():
    xq, kc, vc = synth.attention_inputs(504, 2, 1, 64, 20, 20)
    xo = torch.full((20, 200), 7.0, device="cuda")
    gcu.dev_attention_prefill(xo, dev(xq), dev(kc), dev(vc), 0, xostr=200)
    torch.cuda.synchronize()
    got = xo.cpu().numpy()
    assert_attn_close(got[:, :128], O.attention_prefill(xq, kc, vc, 0))
    assert np.all(got[:, 128:] == 7.0)


def test_rejections():
    xq, kc, vc = (dev(a) for a in synth.attention_inputs(505, 4, 1, 96, 10))
    xo = torch.empty_like(xq)
    with pytest.raises(gcu.GcuError, match="head size"):
        gcu.dev_attention_decode(xo, xq, kc, vc, 0, 10, 0.1)
    xq, kc, vc = (dev(a) for a in synth.attention_inputs(506, 4, 1, 64, 10))
    with pytest.raises(gcu.GcuError, match="window"):
        gcu.dev_attention_decode(torch.empty_like(xq), xq, kc, vc, 5, 6, 0.1)
    with pytest.raises(gcu.GcuError, match="window"):
        gcu.dev_attention_decode(torch.empty_like(xq), xq, kc, vc, 0, 0, 0.1)
    xq9, kc9, vc9 = (dev(a) for a in synth.attention_inputs(507, 18, 2, 64, 10))
    with pytest.raises(gcu.GcuError, match="per kv head"):
        gcu.dev_attention_decode(torch.empty_like(xq9), xq9, kc9, vc9, 0, 10, 0.1)
    xqp, kcp, vcp = (dev(a) for a in synth.attention_inputs(508, 2, 1, 64, 8, 8))
    with pytest.raises(gcu.GcuError, match="outside a cache"):
        gcu.dev_attention_prefill(torch.empty((8, 128), device="cuda"), xqp, kcp, vcp, 4)
    gcu.check_device()


def run_rope(xq, xk, xv, kc, vc, freqs, spos, qs, nq, nk):
    q, k, v = dev(xq), dev(xk), dev(xv)
    kcd, vcd = dev(kc), dev(vc)
    gcu.dev_qk_norm_rope_cache(q, k, v, kcd, vcd, dev(freqs), spos, qs, None if nq is None else dev(nq),
                               None if nk is None else dev(nk))
    torch.cuda.synchronize()
    return q.cpu().numpy(), kcd.cpu().numpy(), vcd.cpu().numpy(), k.cpu().numpy()


@pytest.mark.parametrize("case", META.get("rope", []), ids=lambda c: f"rope{c[0]}")
def test_rope_matches_reference_fixture(case):
    tid, nh, nkv, hd, clen, spos, ntok, qs, norm, _, _ = case
    xq, xk, xv, kc, vc, nq, nk = synth.rope_inputs(tid, nh, nkv, hd, clen, ntok, norm)
    gq, gk, gv, k_after = run_rope(xq, xk, xv, kc, vc, GOLD[f"rope_{tid}_freqs"], spos, qs, nq, nk)
    assert_attn_close(gq, GOLD[f"rope_{tid}_xq"])
    assert_attn_close(gk[:, spos:spos + ntok], GOLD[f"rope_{tid}_k"])
    assert np.array_equal(gv[:, spos:spos + ntok], xv)
    assert np.array_equal(gk[:, :spos], kc[:, :spos]) and np.array_equal(gk[:, spos + ntok:], kc[:, spos + ntok:])
    assert np.array_equal(k_after, xk)  # the keys are read, not changed


@pytest.mark.parametrize("nh,nkv,hd,clen,spos,ntok,qs,norm", [
    (16, 8, 256, 4096, 4000, 1, 1.0, True),     # 12B decode step
    (4, 1, 256, 512, 0, 512, 0.0625, True),     # 1B prefill chunk
    (8, 4, 128, 300, 37, 200, 0.088, False),
    (3, 3, 64, 100, 99, 1, 1.0, True)])
def test_rope_matches_oracle(nh, nkv, hd, clen, spos, ntok, qs, norm):
    xq, xk, xv, kc, vc, nq, nk = synth.rope_inputs(800 + ntok, nh, nkv, hd, clen, ntok, norm)
    pos = np.arange(spos, spos + ntok, dtype=np.float64)[:, None]
    inv = 10000.0 ** (-np.arange(0, hd, 2, dtype=np.float64) / hd)
    freqs = np.empty((ntok, hd), np.float32)
    freqs[:, 0::2] = np.cos(pos * inv)
    freqs[:, 1::2] = np.sin(pos * inv)
    got = run_rope(xq, xk, xv, kc, vc, freqs, spos, qs, nq, nk)
    want = O.qk_norm_rope_cache(xq, xk, xv, kc, vc, freqs, spos, qs, nq, nk)
    for g, w in zip(got[:3], want):
        assert_attn_close(g, w)


def test_rope_then_decode_attention_matches_oracle_chain():
    # QK norm + RoPE + cache write, then the decode attention over the cache
    nh, nkv, hd, clen, spos = 8, 4, 256, 2048, 2047
    xq, xk, xv, kc, vc, nq, nk = synth.rope_inputs(900, nh, nkv, hd, clen, 1, True)
    freqs = np.tile(np.float32([1.0, 0.0]), (1, hd // 2))  # position 0 angles: the identity rotation
    q, k, v = dev(xq), dev(xk), dev(xv)
    kcd, vcd = dev(kc), dev(vc)
    gcu.dev_qk_norm_rope_cache(q, k, v, kcd, vcd, dev(freqs), spos, 1.0, dev(nq), dev(nk))
    xo = torch.empty((nh, hd), device="cuda")
    gcu.dev_attention_decode(xo, q[:, 0, :].contiguous(), kcd, vcd, 0, clen, 1.0 / 16)
    torch.cuda.synchronize()
    oq, okc, ovc = O.qk_norm_rope_cache(xq, xk, xv, kc, vc, freqs, spos, 1.0, nq, nk)
    want = O.attention_decode(oq[:, 0, :], okc, ovc, 0, clen, np.float32(1.0 / 16))
    assert_attn_close(xo.cpu().numpy(), want)


@pytest.mark.parametrize("nh,nkv,hd,clen,spos,attlen,sc,norm", [
    (4, 1, 256, 1024, 0, 1024, 0.0, True),       # 1B global layer at position 1023 (split window)
    (4, 1, 256, 1024, 512, 512, 0.0, True),      # 1B sliding layer: window [512, 1023]
    (16, 8, 256, 4096, 3072, 1024, 50.0, True),  # 12B-like sliding layer with a score softcap
    (8, 4, 128, 300, 0, 37, 0.0, False),         # one CTA per kv head, no qk_norm
    (3, 3, 64, 100, 0, 1, 0.0, True)])           # the new position alone
def test_fused_rope_decode_equals_two_calls(nh, nkv, hd, clen, spos, attlen, sc, norm):
    # gcu_dev_attention_decode_rope: QK norm + RoPE + cache write inside the
    # attention launch; output and cache bit for bit those of the two calls
    xq, xk, xv, kc, vc, nq, nk = synth.rope_inputs(1000 + attlen, nh, nkv, hd, clen, 1, norm)
    pos = spos + attlen - 1
    inv = 10000.0 ** (-np.arange(0, hd, 2, dtype=np.float64) / hd)
    freqs = np.empty((1, hd), np.float32)
    freqs[0, 0::2] = np.cos(pos * inv)
    freqs[0, 1::2] = np.sin(pos * inv)
    asc = float(np.float32(1.0) / np.sqrt(np.float32(hd)))
    nqd = dev(nq) if norm else None
    nkd = dev(nk) if norm else None
    # two calls
    q1, k1, v1, kc1, vc1 = dev(xq), dev(xk), dev(xv), dev(kc), dev(vc)
    gcu.dev_qk_norm_rope_cache(q1, k1, v1, kc1, vc1, dev(freqs), pos, 1.0, nqd, nkd)
    xo1 = torch.empty((nh, hd), device="cuda")
    gcu.dev_attention_decode(xo1, q1[:, 0, :].contiguous(), kc1, vc1, spos, attlen, asc, sc)
    # one launch, twice (the cache row is rewritten with the same values)
    xq2, kc2, vc2 = dev(xq[:, 0, :]), dev(kc), dev(vc)
    xo2 = torch.full((nh, hd), float("nan"), device="cuda")
    for _ in range(2):
        gcu.dev_attention_decode_rope(xo2, xq2, dev(xk[:, 0, :]), dev(xv[:, 0, :]), kc2, vc2, dev(freqs[0]), spos,
                                      attlen, asc, sc, nq=nqd, nk=nkd)
    torch.cuda.synchronize()
    gcu.check_device()
    assert torch.equal(xo2.view(torch.int32), xo1.view(torch.int32))
    assert torch.equal(kc2.view(torch.int32), kc1.view(torch.int32))
    assert torch.equal(vc2.view(torch.int32), vc1.view(torch.int32))
    assert np.array_equal(xq2.cpu().numpy(), xq[:, 0, :])  # the projections are inputs only


# ---- size-independent properties at full size (no oracle needed)

def test_decode_full_window_is_linear_in_values():
    # Gemma-3-12B global layer (16 query heads over 8 kv heads, a 32768-position
    # window split over many CTAs and merged): the weights do not depend on V,
    # so scaling V by a power of two scales every output exactly
    nh, nkv, hd, clen = 16, 8, 256, 32768
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn((nh, hd), generator=g, device="cuda")
    kc = torch.randn((nkv, clen, hd), generator=g, device="cuda")
    vc = torch.randn((nkv, clen, hd), generator=g, device="cuda")
    a, b = torch.empty((nh, hd), device="cuda"), torch.empty((nh, hd), device="cuda")
    gcu.dev_attention_decode(a, q, kc, vc, 0, clen, 1.0 / 16)
    vc.mul_(4.0)
    gcu.dev_attention_decode(b, q, kc, vc, 0, clen, 1.0 / 16)
    torch.cuda.synchronize()
    assert torch.equal(b, a * 4.0)
    gcu.check_device()


def test_prefill_rows_equal_decode_over_their_windows():
    # a full Gemma-3-1B chunk (512 tokens, 4 heads over 1 kv head) with a
    # 128-position sliding window: sampled rows of the causal prefill equal
    # decode attention over the same window (queries pre-scaled, unit scale)
    nh, nkv, hd, ntok, slide = 4, 1, 256, 512, 128
    g = torch.Generator(device="cuda").manual_seed(6)
    xq = torch.randn((nh, ntok, hd), generator=g, device="cuda") * 0.0625
    kc = torch.randn((nkv, ntok, hd), generator=g, device="cuda")
    vc = torch.randn((nkv, ntok, hd), generator=g, device="cuda")
    pre = torch.empty((ntok, nh * hd), device="cuda")
    gcu.dev_attention_prefill(pre, xq, kc, vc, 0, slide)
    for i in (0, 1, 63, 64, 127, 128, 129, 300, 511):
        t0 = i + 1 - slide if i >= slide else 0
        dec = torch.empty((nh, hd), device="cuda")
        gcu.dev_attention_decode(dec, xq[:, i, :].contiguous(), kc, vc, t0, i + 1 - t0, 1.0)
        torch.cuda.synchronize()
        assert_attn_close(pre[i].view(nh, hd).cpu().numpy(), dec.cpu().numpy())
    gcu.check_device()
