"""GPU parity of the chain launch (gcu_gemm_chain_*, k_chain.cu).

A chain runs a list of quantize_acts -> gemm_int8 steps in one persistent
launch.  Every output -- int8 codes, fp32 scales, fp32 GEMM outputs -- must be
bit-identical to the step-by-step device calls (gcu_dev_quantize_acts +
gcu_dev_gemm_int8_multi), which are themselves pinned to the reference; the
oracle recomputes sampled rows as well.  Covered: the Gemma-3-1B prefill layer
of BASELINE configs[1] with the planner's tiles, every tile shape and K split
the chain runs (M and N tails, TMA-store and direct-store outputs, split-K with
every split resident and with more units than SMs), steps that read earlier
steps' outputs, chains longer than one launch, repeated launches and
CUDA-graph replay, and the argument checks.
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


def bits(t):
    return t.contiguous().view(torch.int32) if t.dtype == torch.float32 else t.contiguous()


def assert_same(got, want, what):
    g, w = bits(got), bits(want)
    bad = (g != w)
    if bool(bad.any()):
        idx = torch.nonzero(bad)[:3].tolist()
        raise AssertionError(f"{what}: {int(bad.sum())} of {bad.numel()} differ, first {idx}")


def make_step(gen, m, k, ns, x=None):
    if x is None:
        x = synth.activations_torch(m, k, gen, "cuda", outliers=True)
    q = torch.empty((m, k), dtype=torch.int8, device="cuda")
    s = torch.empty(m, dtype=torch.float32, device="cuda")
    jobs = []
    for n in ns:
        w, sc = synth.weight_torch(n, k, gen, "cuda")
        jobs.append((w, sc, torch.empty((m, n), dtype=torch.float32, device="cuda")))
    return [x, q, s, jobs]


def stepwise(steps):
    """The same steps as separate device calls into fresh outputs."""
    outs = []
    for x, q, s, jobs in steps:
        m, k = x.shape
        q2, s2 = torch.empty_like(q), torch.empty_like(s)
        gcu.dev_quantize_acts(q2, s2, x, m, k)
        ys = [torch.empty_like(o) for _, _, o in jobs]
        gcu.dev_gemm_int8_multi([(w, sc, y) for (w, sc, _), y in zip(jobs, ys)], q2, s2, m, k)
        outs.append((q2, s2, ys))
    torch.cuda.synchronize()
    gcu.check_device()
    return outs


def check_against(steps, ref, what=""):
    for i, ((x, q, s, jobs), (q2, s2, ys)) in enumerate(zip(steps, ref)):
        assert_same(q, q2, f"{what} step {i} codes")
        assert_same(s, s2, f"{what} step {i} scales")
        for j, ((_, _, o), y) in enumerate(zip(jobs, ys)):
            assert_same(o, y, f"{what} step {i} job {j}")


def check_oracle_rows(steps, nrows=6, seed=0):
    rng = np.random.default_rng(seed)
    for x, q, s, jobs in steps:
        m = x.shape[0]
        rows = np.sort(rng.choice(m, min(nrows, m), replace=False))
        xq, xs = O.quantize_acts(x[rows].cpu().numpy())
        assert np.array_equal(q[rows].cpu().numpy(), xq)
        assert np.array_equal(s[rows].cpu().numpy().view(np.uint32), xs.view(np.uint32))
        for w, sc, o in jobs:
            ref = O.gemm_int8(w.cpu().numpy(), sc.cpu().numpy(), xq, xs)
            assert np.array_equal(o[rows].cpu().numpy().view(np.uint32), ref.view(np.uint32))


LAYER_1B = [(1152, (1024, 256, 256)), (1024, (1152,)), (1152, (6912, 6912)), (6912, (1152,))]


def test_chain_prefill1b_layers():
    # two Gemma-3-1B prefill layers (M = 512) as one
    # chain of eight steps with the planner's tiles, launched twice
    gen = torch.Generator(device="cuda").manual_seed(21)
    steps = [make_step(gen, 512, k, ns) for _ in range(2) for k, ns in LAYER_1B]
    ch = gcu.GemmChain(steps)
    plan = ch.plan()
    assert len(plan) == 8 and all(bn in (64, 128, 192, 256) for bn, _, _ in plan)
    ref = stepwise(steps)
    for rep in range(2):
        for _, q, s, jobs in steps:
            q.fill_(0)
            s.fill_(0)
            for _, _, o in jobs:
                o.fill_(0)
        ch.run()
        torch.cuda.synchronize()
        gcu.check_device()
        check_against(steps, ref, f"launch {rep}")
    check_oracle_rows(steps[:4], nrows=4)
    ch.close()


def test_chain_longer_than_one_launch():
    # 26 layers of the 1B prefill (104 steps): several launches of at most
    # 22 steps each, sharing the hand-off counters
    gen = torch.Generator(device="cuda").manual_seed(3)
    steps = [make_step(gen, 512, k, ns) for _ in range(7) for k, ns in LAYER_1B[:2]]
    steps += [make_step(gen, 256, k, ns) for _ in range(6) for k, ns in LAYER_1B[2:]]
    ch = gcu.GemmChain(steps)
    for _ in range(2):
        ch.run()
    torch.cuda.synchronize()
    gcu.check_device()
    check_against(steps, stepwise(steps))
    ch.close()


def test_chain_steps_read_earlier_outputs():
    # step i's input is step i-1's output: the hand-offs order them
    gen = torch.Generator(device="cuda").manual_seed(5)
    m = 300
    s0 = make_step(gen, m, 1024, (2048,))
    s1 = make_step(gen, m, 2048, (1536,), x=s0[3][0][2])
    s2 = make_step(gen, m, 1536, (512, 768), x=s1[3][0][2])
    s3 = make_step(gen, m, 768, (1024,), x=s2[3][1][2])
    steps = [s0, s1, s2, s3]
    ch = gcu.GemmChain(steps)
    ch.run()
    torch.cuda.synchronize()
    gcu.check_device()
    # recompute step by step into fresh buffers, each step on the previous
    # step's fresh output
    ref = []
    xin = s0[0]
    for i, (x, q, s, jobs) in enumerate(steps):
        k = x.shape[1]
        q2, s2_ = torch.empty_like(q), torch.empty_like(s)
        gcu.dev_quantize_acts(q2, s2_, xin, m, k)
        ys = [torch.empty_like(o) for _, _, o in jobs]
        gcu.dev_gemm_int8_multi([(w, sc, y) for (w, sc, _), y in zip(jobs, ys)], q2, s2_, m, k)
        ref.append((q2, s2_, ys))
        xin = ys[1] if i == 2 else ys[0]
    torch.cuda.synchronize()
    check_against(steps, ref)
    check_oracle_rows(steps, nrows=5, seed=1)
    ch.close()


SHAPES = [(64, 1), (128, 1), (256, 1), (128, 2), (192, 2), (256, 2)]


@pytest.mark.parametrize("bn,mb", SHAPES)
@pytest.mark.parametrize("splits", [1, 3])
def test_chain_tile_shapes_and_splits(bn, mb, splits):
    # M tail (300 rows), N tails (1000 rows -> TMA-store output, 1001 -> direct
    # stores), a K that is not a multiple of the 128-byte stage (1168)
    gen = torch.Generator(device="cuda").manual_seed(bn * 10 + mb + splits)
    steps = [make_step(gen, 300, 1168, (1000, 1001)), make_step(gen, 300, 1152, (72,))]
    ch = gcu.GemmChain(steps, force=[(bn, mb, splits), (bn, mb, splits)])
    assert ch.plan()[0] == (bn, mb, splits)
    ch.run()
    torch.cuda.synchronize()
    gcu.check_device()
    check_against(steps, stepwise(steps))
    ch.close()


def test_chain_split_k_more_units_than_sms():
    # 1024 units over 148 CTAs: the last split of each tile reduces it
    gen = torch.Generator(device="cuda").manual_seed(8)
    steps = [make_step(gen, 1024, 4096, (2048,)), make_step(gen, 512, 6912, (1152,))]
    ch = gcu.GemmChain(steps, force=[(64, 1, 4), (128, 1, 4)])
    for _ in range(2):
        ch.run()
    torch.cuda.synchronize()
    gcu.check_device()
    check_against(steps, stepwise(steps))
    ch.close()


def test_chain_graph_replay_sees_new_inputs():
    gen = torch.Generator(device="cuda").manual_seed(13)
    steps = [make_step(gen, 512, k, ns) for k, ns in LAYER_1B]
    ch = gcu.GemmChain(steps)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        ch.run(st)
    st.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        ch.run(st)
    for rep in range(2):
        for x, _, _, _ in steps:
            x.copy_(synth.activations_torch(x.shape[0], x.shape[1], gen, "cuda", outliers=True))
        g.replay()
        torch.cuda.synchronize()
        gcu.check_device()
        check_against(steps, stepwise(steps), f"replay {rep}")
    del g
    ch.close()


def test_chain_rejects_bad_steps():
    gen = torch.Generator(device="cuda").manual_seed(2)
    with pytest.raises(gcu.GcuError, match="multiple of 16"):
        gcu.GemmChain([make_step(gen, 64, 40, (64,))])
    with pytest.raises(gcu.GcuError, match="weights"):
        gcu.GemmChain([make_step(gen, 64, 256, (64,) * 5)])
    with pytest.raises(gcu.GcuError, match="tile"):
        gcu.GemmChain([make_step(gen, 64, 256, (64,))], force=[(96, 1, 1)])
    with pytest.raises(gcu.GcuError, match="unknown handle"):
        gcu._check(gcu.lib().gcu_gemm_chain_run(987654, None), "run")
