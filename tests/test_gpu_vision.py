"""GPU SigLIP head (k_vision.cu) against the reference and the oracle.

Patch embedding (gemma.c:4411-4466) and LayerNorm -> pool -> RMSNorm ->
quantize (gemma.c:4660-4705, 4714) through the C ABI, then the projection
through gcu_dev_gemm_int8.  fp32 stages agree to fp32 reassociation
(max |gpu - want| <= 1e-5 * max |want|); int8 codes agree except for rare
off-by-one codes at rounding boundaries; the projection on the GPU's own
codes is bit-exact against the oracle.
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
GOLD = np.load(os.path.join(HERE, "golden", "vision.npz"))
CASES = json.loads(str(GOLD["meta"]))["cases"]
TOL = 1e-5


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    gcu.init(0)
    yield
    gcu.check_device()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def assert_rows_close(got, want, tol=TOL):
    err = float(np.max(np.abs(got - want)))
    assert np.all(np.isfinite(got)) and err <= tol * float(np.max(np.abs(want))), err


def assert_codes_close(got, want):
    d = np.abs(got.astype(np.int32) - want.astype(np.int32))
    assert d.max() <= 1 and (d != 0).sum() <= max(2, got.size // 1000), (int(d.max()), int((d != 0).sum()))


def run_head(v):
    """GPU patch embed -> pool/quantize -> projection; returns every stage."""
    ppi = v["img_px"] // v["psize"]
    side = int(round(np.sqrt(v["img_tok"])))
    dim, tdim = v["dim"], v["tdim"]
    x = torch.empty((ppi * ppi, dim), device="cuda")
    gcu.dev_patch_embed(x, dev(v["img"]), dev(v["pe"]), dev(v["pe_b"]), dev(v["pos_q"]), dev(v["pos_s"]),
                        v["img_px"], v["psize"], dim)
    q = torch.empty((side * side, dim), dtype=torch.int8, device="cuda")
    s = torch.empty(side * side, device="cuda")
    pooled = torch.empty((side * side, dim), device="cuda")
    gcu.dev_vision_pool_quantize(q, s, x, dev(v["post_n"]), dev(v["post_nb"]), dev(v["norm"]), v["eps"], ppi, side,
                                 dim, out=pooled)
    torch.cuda.synchronize()
    qn, sn = q.cpu().numpy(), s.cpu().numpy()
    if dim % 16 == 0:  # the device GEMM reads 16-byte activation rows
        y = torch.empty((side * side, tdim), device="cuda")
        gcu.dev_gemm_int8(y, dev(v["proj_q"]), dev(v["proj_s"]), q, s, side * side, tdim, dim)
        torch.cuda.synchronize()
        y = y.cpu().numpy()
    else:  # the host entry point repacks other row lengths
        y = gcu.gemm_int8(v["proj_q"], v["proj_s"], qn, sn)
    return x.cpu().numpy(), pooled.cpu().numpy(), qn, sn, y


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"vision{c[0]}")
def test_head_matches_reference_fixture(case):
    tid = case[0]
    v = synth.vision_head_inputs(*case)
    x, pooled, q, s, y = run_head(v)
    assert_rows_close(pooled, GOLD[f"pooled_{tid}"])
    assert_codes_close(q, GOLD[f"q_{tid}"])
    assert_rows_close(s, GOLD[f"s_{tid}"])
    assert np.array_equal(y.view(np.uint32), O.gemm_int8(v["proj_q"], v["proj_s"], q, s).view(np.uint32))


def test_siglip_full_size_against_oracle():
    # SigLIP-So400m at 896 px: 64 x 64 patches of 14 px, dim 1152, pooled to
    # 16 x 16 = 256 tokens, projected to the 4B text width 2560
    v = synth.vision_head_inputs(700, 896, 14, 1152, 256, 2560)
    x, pooled, q, s, y = run_head(v)
    xo = O.patch_embed(v)
    assert_rows_close(x, xo)
    po, qo, so = O.vision_pool(x, v)  # pool the GPU's own patch rows: the stage alone
    assert_rows_close(pooled, po)
    assert_codes_close(q, qo)
    assert np.array_equal(y.view(np.uint32), O.gemm_int8(v["proj_q"], v["proj_s"], q, s).view(np.uint32))


def test_patch_embed_tails():
    # patches and channels that do not fill the 64 x 64 tiles
    v = synth.vision_head_inputs(710, 70, 7, 100, 4, 8)  # 10 x 10 patches, dim 100
    x = torch.empty((100, 100), device="cuda")
    gcu.dev_patch_embed(x, dev(v["img"]), dev(v["pe"]), dev(v["pe_b"]), dev(v["pos_q"]), dev(v["pos_s"]), 70, 7, 100)
    torch.cuda.synchronize()
    assert_rows_close(x.cpu().numpy(), O.patch_embed(v))


def test_rejections():
    v = synth.vision_head_inputs(720, 56, 14, 64, 16, 32)
    x = torch.empty((16, 64), device="cuda")
    args = [dev(v[k]) for k in ("img", "pe", "pe_b", "pos_q", "pos_s")]
    with pytest.raises(gcu.GcuError, match="patches"):
        gcu.dev_patch_embed(x, *args, 56, 15, 64)
    with pytest.raises(gcu.GcuError, match="patches"):
        gcu.dev_patch_embed(x, *args, 56, 28 + 4, 64)
    q = torch.empty((4, 64), dtype=torch.int8, device="cuda")
    s = torch.empty(4, device="cuda")
    norms = [dev(v[k]) for k in ("post_n", "post_nb", "norm")]
    with pytest.raises(gcu.GcuError, match="pool"):
        gcu.dev_vision_pool_quantize(q, s, x, *norms, 1e-6, 4, 3, 64)
    with pytest.raises(gcu.GcuError, match="multiple of 4"):
        gcu.dev_vision_pool_quantize(q, s, x, *norms, 1e-6, 4, 2, 62)
    gcu.check_device()
