"""gcu_dev_gemm_int8_noalloc: the GEMM entry point for callers that may not
allocate device memory while running (processes that fix all GPU memory at
start-up, or that cannot accept the device synchronisation an allocation may
cause).  Its split-K scratch is a fixed array inside libgcu.so, so the check
here is that it returns exactly what gcu_dev_gemm_int8 returns, on two calls
in a row (the second call finds the first call's leftovers in the shared
array), and that a plan needing more scratch than the array holds is refused
with a clear error.  Both entry points are also checked bit for bit against
the CPU oracle (the restatement of gemma.c's gemm_int8, pinned to the
compiled reference by the oracle tests), so a fault shared by the two GPU
paths cannot pass.  This file sorts last so a failure here never hides the
other GPU tests."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import gcu  # noqa: E402
import oracle  # noqa: E402  (the CPU checker)
import synth  # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    gcu.init(0)


def _operands(m, n, k, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    w, ws = synth.weight_torch(n, k, gen, "cuda")
    x = synth.activations_torch(m, k, gen, "cuda", outliers=True)
    q = torch.empty((m, k), dtype=torch.int8, device="cuda")
    s = torch.empty(m, dtype=torch.float32, device="cuda")
    gcu.dev_quantize_acts(q, s, x, m, k)
    return w, ws, q, s


@pytest.mark.parametrize("m,n,k", [(256, 1152, 6912),   # long K: split six ways through the array
                                   (384, 1000, 2304),   # K split, ragged N
                                   (512, 1536, 1152),   # no split: no scratch used
                                   (4, 4096, 2560)])    # m <= 8: streaming kernel
def test_noalloc_matches_allocating_entry_point(m, n, k):
    w, ws, q, s = _operands(m, n, k, seed=m + n + k)
    ref = torch.empty((m, n), dtype=torch.float32, device="cuda")
    gcu.dev_gemm_int8(ref, w, ws, q, s, m, n, k)
    want = oracle.gemm_int8(w.cpu().numpy(), ws.cpu().numpy(), q.cpu().numpy(), s.cpu().numpy())
    got = ref.cpu().numpy().view(np.uint32)
    assert np.array_equal(got, want.view(np.uint32)), f"{(got != want.view(np.uint32)).sum()} differ from the oracle"
    for _ in range(2):  # two calls in a row share the scratch array
        out = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        gcu.dev_gemm_int8_noalloc(out, w, ws, q, s, m, n, k)
        torch.cuda.synchronize()
        gcu.check_device()
        a = out.cpu().numpy().view(np.uint32)
        b = ref.cpu().numpy().view(np.uint32)
        assert np.array_equal(a, b), f"{(a != b).sum()} outputs differ"


def test_noalloc_rejects_plans_beyond_the_array():
    # M=512, N=1152, K=6912 in 128x128 tiles split four ways needs 9 MiB of
    # partials (the plan is forced: the planner's own pick may need less)
    m, n, k = 512, 1152, 6912
    w, ws, q, s = _operands(m, n, k, seed=5)
    out = torch.empty((m, n), dtype=torch.float32, device="cuda")
    with pytest.raises(gcu.GcuError, match="split-K needs"):
        gcu.dev_gemm_int8_noalloc_tuned(out, w, ws, q, s, m, n, k, 128, 4, 1)
    # the same plan within the array: 256 rows need 4.5 MiB
    m = 256
    w, ws, q, s = _operands(m, n, k, seed=6)
    ref = torch.empty((m, n), dtype=torch.float32, device="cuda")
    gcu.dev_gemm_int8(ref, w, ws, q, s, m, n, k)
    out = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    gcu.dev_gemm_int8_noalloc_tuned(out, w, ws, q, s, m, n, k, 128, 4, 1)
    torch.cuda.synchronize()
    gcu.check_device()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.cpu().numpy().view(np.uint32))
    want = oracle.gemm_int8(w.cpu().numpy(), ws.cpu().numpy(), q.cpu().numpy(), s.cpu().numpy())
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))
