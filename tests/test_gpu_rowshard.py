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
    ok = True
    try:
        gcu.init(rank)
        obj = [gcu.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        gcu.comm_init(rank, world, obj[0])
        for m, n, k in [(1, 8192, 2560), (4, 4096, 640), (300, 2048, 1152)]:
            w, ws = synth.weight(700 + m, n, k)
            xq, xs = O.quantize_acts(synth.activations(800 + m, m, k))
            sl = shard.row_slice(n, rank, world)
            dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
            y = torch.empty((m, n), dtype=torch.float32, device="cuda")
            work = torch.empty((m, n), dtype=torch.float32, device="cuda")
            gcu.dev_gemm_int8_rowshard(y, work, dev(w[sl]), dev(ws[sl]), dev(xq), dev(xs), m, n, k)
            torch.cuda.synchronize()
            ref = O.gemm_int8(w, ws, xq, xs)
            ok = ok and bool(np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32)))
        gcu.check_device()
        gcu.comm_destroy()
    finally:
        dist.destroy_process_group()
    q.put((rank, ok))


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
    assert res == {0: True, 1: True}
