"""A device-resident decode step (decode.Decoder) against gemma.c's own.

tests/golden/decode.npz holds what gemma.c's forward_text_decode computes for
positions 0..7 on small seeded W8A8 decoders (make_decode_golden.py): logits
and final hidden states per step, and its RoPE tables.  The GPU decoder runs
the same step as one chain of C-ABI calls (norm+quantize, multi-GEMV, QK
norm/RoPE/cache, attention, fused quantize+GEMV, residual, GeGLU+quantize,
lm_head), with the KV cache on the device across the 8 steps.

Each stage is checked exactly or to fp32 reassociation by its own tests; the
chain adds int8 rounding boundaries: an fp32 value a few ulps from a
quantization boundary can round to the neighbouring code, which moves that
product by one code step.  So the bound here is max |gpu - ref| <= 2e-3 of
the largest |ref| per step, and the median difference within 1e-5 of it
(the typical element agrees to fp32 rounding).  The last link is then checked
exactly: the logits equal the lm_head of the quantized final hidden state on
both sides, and the two quantizations are counted code by code (on these
fixtures no code flips, and the logits are bit-identical without a softcap).
"""
import json
import os

import numpy as np
import pytest

import synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import decode  # noqa: E402
import gcu  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "decode.npz"))
META = json.loads(str(GOLD["meta"]))


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    gcu.init(0)
    yield
    gcu.check_device()


def close(got, want):
    err = np.abs(got - want)
    scale = float(np.max(np.abs(want)))
    return float(err.max()) <= 2e-3 * scale and float(np.median(err)) <= 1e-5 * scale, float(err.max()) / scale


@pytest.mark.parametrize("name", list(META["cases"]))
def test_decode_steps_match_reference(name):
    cfg = META["cases"][name]
    layers, emb, fnorm = synth.decoder_model(cfg["tid"], cfg)
    npos = META["npos"]
    x0 = synth.normal(cfg["tid"] + 999, (npos, cfg["dim"]))
    dec = decode.Decoder(cfg, layers, emb, fnorm, clen=npos)
    for p in range(npos):
        dec.set_freqs(GOLD[f"{name}_slid"][p], GOLD[f"{name}_full"][p])
        dec.x.copy_(torch.from_numpy(x0[p][None]))
        dec.step(p)
        torch.cuda.synchronize()
        ok, rel = close(dec.logits.cpu().numpy()[0], GOLD[f"{name}_logits"][p])
        assert ok, f"logits at position {p}: max diff {rel:.3g} of the largest"
        ok, rel = close(dec.x.cpu().numpy()[0], GOLD[f"{name}_hid"][p])
        assert ok, f"hidden state at position {p}: max diff {rel:.3g} of the largest"
    gcu.check_device()


@pytest.mark.parametrize("name", list(META["cases"]))
def test_decode_logit_error_is_last_quantize_code_flips(name):
    # The logit bound above is a tolerance; this accounts for it at the last
    # link of the chain.  The fixture's hidden state is the final RMSNorm's
    # output, the input of the lm_head's quantize_act (gemma.c:4965-4966).
    # (1) the GPU's logits are exactly lm_head(quantize(GPU hidden)), (2) the
    # reference's are exactly lm_head(quantize(reference hidden)) -- so the
    # logit difference IS the difference of those two int8 inputs -- and (3)
    # the two quantizations differ only by codes flipped by one step at a
    # rounding boundary (counted per step) and a scale within fp32 rounding.
    import oracle as O
    cfg = META["cases"][name]
    layers, emb, fnorm = synth.decoder_model(cfg["tid"], cfg)
    npos = META["npos"]
    x0 = synth.normal(cfg["tid"] + 999, (npos, cfg["dim"]))
    dec = decode.Decoder(cfg, layers, emb, fnorm, clen=npos)
    cap = cfg["sc_log"]

    def lm_head(q, sc):
        y = O.gemv_int8(emb[0], emb[1], q, sc)
        # gemma.c:4971-4976: tanhf(logit / cap) * cap
        return (np.tanh(y / np.float32(cap)) * np.float32(cap)).astype(np.float32) if cap else y

    flips = []
    for p in range(npos):
        dec.set_freqs(GOLD[f"{name}_slid"][p], GOLD[f"{name}_full"][p])
        dec.x.copy_(torch.from_numpy(x0[p][None]))
        dec.step(p)
        torch.cuda.synchronize()
        hid_g, log_g = dec.x.cpu().numpy()[0], dec.logits.cpu().numpy()[0]
        hid_r, log_r = GOLD[f"{name}_hid"][p], GOLD[f"{name}_logits"][p]
        qg, sg = O.quantize_act(hid_g)
        qr, sr = O.quantize_act(hid_r)
        tol = 0.0 if not cap else 2e-6 * float(np.max(np.abs(log_r)))  # tanhf vs numpy's tanh
        assert np.max(np.abs(lm_head(qg, sg) - log_g)) <= tol, f"GPU lm_head at position {p}"
        assert np.max(np.abs(lm_head(qr, sr) - log_r)) <= tol, f"reference lm_head at position {p}"
        d = qg.astype(np.int32) - qr.astype(np.int32)
        assert np.max(np.abs(d)) <= 1, f"position {p}: a code moved by {np.max(np.abs(d))} steps"
        assert abs(float(sg) - float(sr)) <= 1e-5 * float(sr), f"position {p}: scales {sg} vs {sr}"
        flips.append(int(np.count_nonzero(d)))
        assert flips[-1] <= max(2, cfg["dim"] // 50), f"position {p}: {flips[-1]} codes flipped"
        if flips[-1] == 0 and sg == sr:  # the same int8 input: the same logits
            assert np.max(np.abs(log_g - log_r)) <= 2 * tol, f"position {p}: equal codes, different logits"
            if not cap:
                assert np.array_equal(log_g.view(np.uint32), log_r.view(np.uint32))
    print(f"{name}: codes flipped at the lm_head quantize per step: {flips}")


def test_decode_step_graph_replay_matches_eager():
    # the whole step is capturable: a CUDA graph replay gives the eager result bit for bit
    name = "gemma3"
    cfg = META["cases"][name]
    layers, emb, fnorm = synth.decoder_model(cfg["tid"], cfg)
    x0 = synth.normal(cfg["tid"] + 999, (2, cfg["dim"]))
    outs = []
    for use_graph in (False, True):
        dec = decode.Decoder(cfg, layers, emb, fnorm, clen=4)
        dec.set_freqs(GOLD[f"{name}_slid"][0], GOLD[f"{name}_full"][0])
        dec.x.copy_(torch.from_numpy(x0[0][None]))
        dec.step(0)  # position 0 eagerly (also warms the library)
        dec.set_freqs(GOLD[f"{name}_slid"][1], GOLD[f"{name}_full"][1])
        dec.x.copy_(torch.from_numpy(x0[1][None]))
        st = torch.cuda.Stream()
        torch.cuda.synchronize()
        if use_graph:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                dec.step(1, stream=st)
            g.replay()
        else:
            with torch.cuda.stream(st):
                dec.step(1, stream=st)
        torch.cuda.synchronize()
        outs.append(dec.logits.cpu().numpy().copy())
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))


def test_rope_tables_follow_rope_freqs():
    # the host tables (numpy float32) against the reference's own for the fixture positions
    cfg = META["cases"]["gemma3"]
    for p in range(META["npos"]):
        slid, full = decode.rope_tables(cfg["hdim"], cfg["theta_l"], cfg["theta_g"], p)
        assert np.max(np.abs(slid - GOLD["gemma3_slid"][p])) <= 2e-6
        assert np.max(np.abs(full - GOLD["gemma3_full"][p])) <= 2e-6


# ---- the residual / softcap kernels on their own

import oracle as O  # noqa: E402


def _d(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("m,dim", [(1, 1152), (3, 2560), (2, 96), (1, 4096)])
def test_rmsnorm_residual(m, dim):
    y, r = synth.normal(50 + dim, (m, dim)), synth.normal(51 + dim, (m, dim))
    w = synth.normal(52 + dim, (dim,), 0.1)
    x = torch.empty((m, dim), device="cuda")
    gcu.dev_rmsnorm_residual(x, _d(y), _d(r), None, 1e-6, m, dim)  # no post-norm: an exact add
    torch.cuda.synchronize()
    assert np.array_equal(x.cpu().numpy(), y + r)
    gcu.dev_rmsnorm_residual(x, _d(y), _d(r), _d(w), 1e-6, m, dim)
    torch.cuda.synchronize()
    y64 = y.astype(np.float64)
    want = r + y64 / np.sqrt((y64 ** 2).mean(axis=1, keepdims=True) + 1e-6) * (w + 1.0)
    assert np.max(np.abs(x.cpu().numpy() - want)) <= 1e-5 * np.max(np.abs(want))


@pytest.mark.parametrize("m,dim,post", [(1, 1152, True), (2, 2560, False), (1, 96, True)])
def test_residual_norm_quantize_equals_the_two_step_path(m, dim, post):
    y, r = synth.normal(60 + dim, (m, dim)), synth.normal(61 + dim, (m, dim))
    wp = synth.normal(62 + dim, (dim,), 0.1) if post else None
    wn = synth.normal(63 + dim, (dim,), 0.1)
    x1 = _d(r.copy())
    q = torch.empty((m, dim), dtype=torch.int8, device="cuda")
    s = torch.empty(m, device="cuda")
    gcu.dev_residual_norm_quantize(x1, q, s, _d(y), x1, None if wp is None else _d(wp), _d(wn), 1e-6, m, dim)
    x2 = _d(r.copy())
    gcu.dev_rmsnorm_residual(x2, _d(y), x2, None if wp is None else _d(wp), 1e-6, m, dim)
    torch.cuda.synchronize()
    xg = x1.cpu().numpy()
    assert np.array_equal(xg.view(np.uint32), x2.cpu().numpy().view(np.uint32))  # same residual update
    _, qo, so = O.rmsnorm_quantize(xg, wn, 1e-6)
    d = np.abs(q.cpu().numpy().astype(np.int32) - qo.astype(np.int32))
    assert d.max() <= 1 and (d != 0).sum() <= max(2, d.size // 1000)
    assert np.max(np.abs(s.cpu().numpy() - so)) <= 1e-6 * np.max(so)


def test_softcap():
    x = synth.normal(70, (5, 1000), 40.0)
    t = _d(x)
    gcu.dev_softcap(t, 30.0)
    torch.cuda.synchronize()
    want = np.tanh(x.astype(np.float64) / 30.0) * 30.0
    assert np.max(np.abs(t.cpu().numpy() - want)) <= 1e-5 * 30.0
    with pytest.raises(gcu.GcuError, match="zero cap"):
        gcu.dev_softcap(t, 0.0)


@pytest.mark.parametrize("name", list(META["cases"]))
def test_prefill_chunks_match_reference(name):
    # forward_text_chunk over chunks of 5 and 11 tokens, the KV cache carried
    # from the first chunk to the second
    cfg = META["cases"][name]
    layers, emb, fnorm = synth.decoder_model(cfg["tid"], cfg)
    chunks = META["chunks"]
    total = sum(chunks)
    xp = synth.normal(cfg["tid"] + 777, (total, cfg["dim"]))
    dec = decode.Decoder(cfg, layers, emb, fnorm, clen=total)
    spos = 0
    for c, n in enumerate(chunks):
        dec.set_prefill_freqs(GOLD[f"{name}_pslid"][spos:spos + n], GOLD[f"{name}_pfull"][spos:spos + n])
        dec.px[:n].copy_(torch.from_numpy(xp[spos:spos + n]))
        dec.prefill(spos, n)
        torch.cuda.synchronize()
        ok, rel = close(dec.logits.cpu().numpy()[0], GOLD[f"{name}_pre_logits"][c])
        assert ok, f"chunk {c} logits: max diff {rel:.3g} of the largest"
        ok, rel = close(dec.px[:n].cpu().numpy(), GOLD[f"{name}_pre_hid"][spos:spos + n])
        assert ok, f"chunk {c} hidden states: max diff {rel:.3g} of the largest"
        spos += n
    gcu.check_device()


def test_prefill_then_decode_continues_the_cache():
    # prefill 16 tokens, then decode position 16 on the same KV cache: the
    # reference decode of 17 positions gives the same last logits
    name = "gemma3"
    cfg = META["cases"][name]
    layers, emb, fnorm = synth.decoder_model(cfg["tid"], cfg)
    xp = synth.normal(cfg["tid"] + 777, (17, cfg["dim"]))
    dec = decode.Decoder(cfg, layers, emb, fnorm, clen=17)
    dec.set_prefill_freqs(GOLD[f"{name}_pslid"][:16], GOLD[f"{name}_pfull"][:16])
    dec.px[:16].copy_(torch.from_numpy(xp[:16]))
    dec.prefill(0, 16)
    slid, full = decode.rope_tables(cfg["hdim"], cfg["theta_l"], cfg["theta_g"], 16)
    dec.set_freqs(slid, full)
    dec.x.copy_(torch.from_numpy(xp[16][None]))
    dec.step(16)
    torch.cuda.synchronize()
    got = dec.logits.cpu().numpy()[0]
    dec2 = decode.Decoder(cfg, layers, emb, fnorm, clen=17)
    for p in range(17):
        s_, f_ = (GOLD[f"{name}_pslid"][p], GOLD[f"{name}_pfull"][p]) if p < 16 else (slid, full)
        dec2.set_freqs(s_, f_)
        dec2.x.copy_(torch.from_numpy(xp[p][None]))
        dec2.step(p)
    torch.cuda.synchronize()
    ok, rel = close(got, dec2.logits.cpu().numpy()[0])
    assert ok, f"prefill+decode vs decode only: {rel:.3g}"
