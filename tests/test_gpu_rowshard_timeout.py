"""A rank that skips a row-sharded call: the fused all-gather gives up, the
other rank learns of it, and nothing runs on out-of-step counters.

Two processes, one GPU each, NCCL with NVLS off; the fused all-gather uses
plain peer loads of CUDA-IPC mappings (no multicast objects).  Rank 1 leaves
one call out between steps, with none of its own work in flight: rank 0's
launch waits for rank 1's arrival, gives up after its bounded wait (device
code 6, DEV_TIMEOUT_PEER) and returns, leaving its context usable.  Rank 0
must then report the failure (gcu_check_device), refuse its next row-sharded
call, and -- after gcu_comm_destroy and gcu_comm_init on both ranks -- get
bit-exact results again.  Needs >= 2 GPUs (skipped otherwise).
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
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    bad = []
    m, n, k = 1, 8192, 2560
    w, ws = synth.weight(71, n, k)
    xq, xs = O.quantize_acts(synth.activations(72, m, k))
    ref = O.gemm_int8(w, ws, xq, xs)
    sl = shard.row_slice(n, rank, world)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    wl, wsl, xqd, xsd = dev(w[sl]), dev(ws[sl]), dev(xq), dev(xs)

    def call():
        y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        work = torch.empty((m, n), dtype=torch.float32, device="cuda")
        gcu.dev_gemm_int8_rowshard(y, work, wl, wsl, xqd, xsd, m, n, k)
        return y

    def init():
        obj = [gcu.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        gcu.comm_init(rank, world, obj[0])
        if not gcu.comm_fused_allgather():
            bad.append("fused all-gather off")

    try:
        gcu.init(rank)
        init()
        # step 1: both ranks, bit-exact
        y = call()
        torch.cuda.synchronize()
        if not np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32)):
            bad.append("step 1 differs")
        dist.barrier()
        # step 2: rank 1 leaves the call out (decided on the host, between steps)
        if rank == 0:
            call()
            torch.cuda.synchronize()  # the launch returns once its bounded wait gives up
            try:
                gcu.check_device()
                bad.append("no device-side error after the peer skipped the call")
            except gcu.GcuError as e:
                if "code 6" not in str(e):
                    bad.append(f"unexpected error: {e}")
            try:
                call()
                bad.append("row-sharded call not refused after the peer timeout")
            except gcu.GcuError as e:
                if "refused" not in str(e):
                    bad.append(f"unexpected refusal message: {e}")
        dist.barrier()
        # step 3: rebuild on both ranks, bit-exact again
        torch.cuda.synchronize()
        gcu.comm_destroy()
        init()
        y = call()
        torch.cuda.synchronize()
        if not np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32)):
            bad.append("step 3 (after re-init) differs")
        gcu.check_device()
        gcu.comm_destroy()
    except Exception as e:  # report, do not hang the other rank
        bad.append(f"exception: {e}")
    finally:
        dist.destroy_process_group()
    q.put((rank, bad))


def test_rowshard_peer_skips_a_call():
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
