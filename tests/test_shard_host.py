"""Host logic of the row-sharded path on CPU ranks (gloo, world sizes 2 and 4).

Each rank computes its row slice of a W8A8 GEMM/GEMV with the oracle, the
slices are all-gathered over gloo in rank order, and the re-layout must give
the unsharded result bit for bit -- the convention gcu_dev_gemm_int8_rowshard
follows on the GPU with NCCL.
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, m, n, k, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "oracle"), os.path.join(root, "gemma.c_b200")]
    import oracle as O
    import shard
    import synth
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w, ws = synth.weight(41, n, k)
        xq, xs = O.quantize_acts(synth.activations(42, m, k))
        sl = shard.row_slice(n, rank, world)
        local = O.gemm_int8(w[sl], ws[sl], xq, xs)  # (m, n/world)
        bufs = [torch.empty(m * (n // world), dtype=torch.float32) for _ in range(world)]
        dist.all_gather(bufs, torch.from_numpy(np.ascontiguousarray(local).reshape(-1)))
        full = shard.relayout(torch.cat(bufs).numpy(), m, n, world)
        ref = O.gemm_int8(w, ws, xq, xs)
        q.put((rank, bool(np.array_equal(full.view(np.uint32), ref.view(np.uint32)))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("m,world", [(1, 2), (4, 2), (9, 2), (1, 4), (9, 4)])
def test_rowshard_gather_matches_unsharded(m, world):
    n, k = 96, 640
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, m, n, k, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    res = dict(q.get(timeout=10) for _ in range(world))
    assert res == {r: True for r in range(world)}


def test_row_slice_rejects_uneven():
    import shard
    with pytest.raises(ValueError):
        shard.row_slice(10, 0, 4)
    assert shard.row_slice(262144, 7, 8) == slice(229376, 262144)
