"""Failure detection on the GPU, without a GPU fault.

Every device-side wait in libgcu.so is bounded: when its budget runs out the
kernel records a code in the device error word and returns, and the host's
next check reports "device-side wait gave up".  Here a wait runs on something
that never completes (an mbarrier nobody arrives on, a flag nobody sets) with
a 20 ms budget; the tests check that the wait ends near its budget, that the
host reads the code (through gcu_check_device and through an ordinary call's
own check), that reading clears it, and that the context keeps computing
bit-exact results afterwards.  Nothing here faults, traps or hangs a GPU.
"""
import numpy as np
import pytest

import oracle as O
import synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import gcu  # noqa: E402

BUDGET_US = 20000
SELFTEST_CODE = 8


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    gcu.init(0)
    gcu.check_device()
    yield
    gcu.check_device()


def _gemm_still_exact(m, n, k, seed):
    w, ws = synth.weight(seed, n, k)
    x = synth.activations(seed + 1, m, k)
    q, s = O.quantize_acts(x)
    got = gcu.gemm_int8(w, ws, q, s)
    want = O.gemm_int8(w, ws, q, s)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("mode", [0, 1], ids=["mbarrier", "flag"])
def test_wait_gives_up_and_host_reads_code(mode):
    waited = gcu.selftest_bounded_wait(mode, BUDGET_US)
    # the loop re-reads the timer between polls, so it ends just past the budget
    assert BUDGET_US * 1000 <= waited < BUDGET_US * 1000 + 50_000_000, waited
    with pytest.raises(gcu.GcuError, match=f"device-side wait gave up \\(code {SELFTEST_CODE}\\)"):
        gcu.check_device()
    gcu.check_device()  # reading the word cleared it
    _gemm_still_exact(256, 384, 1152, 11 + mode)  # tensor-core GEMM
    _gemm_still_exact(3, 1024, 640, 21 + mode)  # GEMV


def test_next_call_reports_code_then_recovers():
    gcu.selftest_bounded_wait(1, BUDGET_US)
    w, ws = synth.weight(31, 512, 1152)
    x = synth.activations(32, 64, 1152)
    q, s = O.quantize_acts(x)
    with pytest.raises(gcu.GcuError, match="device-side wait gave up"):
        gcu.gemm_int8(w, ws, q, s)
    got = gcu.gemm_int8(w, ws, q, s)
    assert np.array_equal(got.view(np.uint32), O.gemm_int8(w, ws, q, s).view(np.uint32))


def test_wait_runs_in_stream_order():
    # the wait is an ordinary launch on the caller's stream: later work on the
    # same stream runs after it and is unaffected
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        waited = gcu.selftest_bounded_wait(0, 2000, stream=st)
        a = torch.arange(1 << 20, device="cuda", dtype=torch.float32)
        b = (a * 2).sum().item()
    assert waited >= 2_000_000
    assert b == float((1 << 20) * ((1 << 20) - 1))
    with pytest.raises(gcu.GcuError, match="code 8"):
        gcu.check_device()


@pytest.mark.parametrize("mode,budget", [(2, 1000), (-1, 1000), (0, 0), (1, 2_000_000)])
def test_selftest_rejects_bad_arguments(mode, budget):
    with pytest.raises(gcu.GcuError, match="selftest_bounded_wait"):
        gcu.selftest_bounded_wait(mode, budget)
    gcu.check_device()  # nothing was launched
