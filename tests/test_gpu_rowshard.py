"""Row-sharded W8A8 GEMM/GEMV over 2 GPUs with NCCL (gcu_dev_gemm_int8_rowshard).

Each rank (one process per GPU) holds n/2 weight rows, computes its slice on
its own GPU and all-gathers over NVLink; every rank's full output must equal
the unsharded oracle bit for bit.  Needs >= 2 GPUs (skipped otherwise).
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "oracle"), os.path.join(root, "gemma.c_b200")]
    import torch.distributed as dist
    import gcu
    import oracle as O
    import shard
    import synth
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    bad = []
    try:
        gcu.init(rank)
        obj = [gcu.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        gcu.comm_init(rank, world, obj[0])
        if not gcu.comm_fused_allgather():  # NVLink peers: the fused path must be on
            bad.append("fused all-gather off")
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        # several calls in a row alternate the two halves of the symmetric
        # buffer; m <= 8 runs the fused GEMV + peer-store all-gather, m = 300
        # the tensor-core GEMM + NCCL all-gather
        for it, (m, n, k) in enumerate([(1, 8192, 2560), (4, 4096, 640), (1, 8192, 2560), (8, 2048, 1152),
                                        (300, 2048, 1152), (1, 262144, 640), (1, 8192, 2560)]):
            w, ws = synth.weight(700 + m + it, n, k) if n * k <= 8 << 20 else (
                np.random.default_rng(it).integers(-127, 128, (n, k), dtype=np.int8),
                np.random.default_rng(it + 1).random(n, dtype=np.float32) * 1e-3)
            xq, xs = O.quantize_acts(synth.activations(800 + m + it, m, k))
            sl = shard.row_slice(n, rank, world)
            y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
            work = torch.empty((m, n), dtype=torch.float32, device="cuda")
            gcu.dev_gemm_int8_rowshard(y, work, dev(w[sl]), dev(ws[sl]), dev(xq), dev(xs), m, n, k)
            torch.cuda.synchronize()
            ref = O.gemm_int8(w, ws, xq, xs)
            if not np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32)):
                bad.append(f"rowshard m={m} n={n} k={k}")
        # quantize + several row-sharded weights in one call: fused (one
        # launch, pushes to the peer) for m <= 8, else quantize + NCCL per job
        for it, (m, ns, k) in enumerate([(1, (4096, 4096), 1152), (4, (2048, 1024, 512), 640),
                                         (1, (4096, 4096), 1152), (12, (1024, 512), 640), (2, (8192,), 2560)]):
            x = synth.activations(900 + it, m, k, outliers=True)
            wts = [synth.weight(950 + 10 * it + j, n, k) for j, n in enumerate(ns)]
            qt = torch.empty((m, k), dtype=torch.int8, device="cuda")
            st = torch.empty(m, dtype=torch.float32, device="cuda")
            ys = [torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda") for n in ns]
            work = torch.empty((m, max(ns)), dtype=torch.float32, device="cuda")
            jobs = [(dev(w[shard.row_slice(n, rank, world)]), dev(sc[shard.row_slice(n, rank, world)]), y, n)
                    for (w, sc), y, n in zip(wts, ys, ns)]
            gcu.dev_quantize_gemm_int8_rowshard_multi(jobs, qt, st, dev(x), m, k, work=work)
            torch.cuda.synchronize()
            xq, xs = O.quantize_acts(x)
            if not (np.array_equal(qt.cpu().numpy(), xq) and
                    np.array_equal(st.cpu().numpy().view(np.uint32), xs.view(np.uint32))):
                bad.append(f"multi m={m} ns={ns}: codes or scales")
            for j, ((w, sc), y) in enumerate(zip(wts, ys)):
                ref = O.gemm_int8(w, sc, xq, xs)
                got = y.cpu().numpy()
                if not np.array_equal(got.view(np.uint32), ref.view(np.uint32)):
                    nbad = int((got.view(np.uint32) != ref.view(np.uint32)).sum())
                    bad.append(f"multi m={m} ns={ns} job {j}: {nbad} of {got.size} differ")
        gcu.check_device()
        gcu.comm_destroy()
    finally:
        dist.destroy_process_group()
    q.put((rank, bad))


def test_rowshard_two_gpus_matches_unsharded():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = dict(q.get(timeout=10) for _ in range(2))
    assert res == {0: [], 1: []}, res
