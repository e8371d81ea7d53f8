"""Gemma's FFN block with the hidden dimension split over 2 GPUs
(gcu_dev_ffn_rowshard): bit for bit the unsharded block.

Each rank (one process per GPU, NCCL with NVLS off) first runs the block
unsharded on the full weights, then -- after gcu_comm_init -- on its slices:
rows [r*fl, (r+1)*fl) of up and gate, the same columns of down.  The row
maxima of h are all-reduced before quantizing, the down projection's int32
partial sums after, so both ranks must return exactly the unsharded output,
for the Gemma-3-12B FFN shape of BASELINE configs[4] (dim 3840, ffn 15360) at
a reduced token count and a 4B shape.  Needs >= 2 GPUs (skipped otherwise).
"""
import os
import socket

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
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "oracle"), os.path.join(root, "gemma.c_b200")]
    import torch.distributed as dist
    import gcu
    import synth
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    bad = []
    try:
        gcu.init(rank)
        cases = [(512, 3840, 15360), (300, 2560, 10240), (1024, 1152, 6912)]
        refs = []
        data = []
        for m, dim, ffn in cases:
            gen = torch.Generator(device="cuda").manual_seed(m + dim)  # the same weights on both ranks
            w1 = synth.weight_torch(ffn, dim, gen, "cuda")
            w2 = synth.weight_torch(ffn, dim, gen, "cuda")
            w3 = synth.weight_torch(dim, ffn, gen, "cuda")
            x = synth.activations_torch(m, dim, gen, "cuda", outliers=True)
            xq = torch.empty((m, dim), dtype=torch.int8, device="cuda")
            xs = torch.empty(m, device="cuda")
            gcu.dev_quantize_acts(xq, xs, x, m, dim)
            out = torch.empty((m, dim), device="cuda")
            gcu.dev_ffn_rowshard(out, xq, xs, m, dim, ffn, w1[0], w1[1], w2[0], w2[1], w3[0], w3[1])
            refs.append(out)
            data.append((m, dim, ffn, w1, w2, w3, xq, xs))
        torch.cuda.synchronize()
        obj = [gcu.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        gcu.comm_init(rank, world, obj[0])
        for (m, dim, ffn, w1, w2, w3, xq, xs), ref in zip(data, refs):
            fl = ffn // world
            r0, r1 = rank * fl, (rank + 1) * fl
            up = (w1[0][r0:r1].contiguous(), w1[1][r0:r1].contiguous())
            gate = (w2[0][r0:r1].contiguous(), w2[1][r0:r1].contiguous())
            down = w3[0][:, r0:r1]  # a strided view of the full weight: row stride ffn bytes
            out = torch.full((m, dim), float("nan"), device="cuda")
            for _ in range(2):  # twice: the scratch and the collectives are reused
                gcu.dev_ffn_rowshard(out, xq, xs, m, dim, ffn, up[0], up[1], gate[0], gate[1], down, w3[1],
                                     w_down_stride=ffn)
            torch.cuda.synchronize()
            if not torch.equal(out.view(torch.int32), ref.view(torch.int32)):
                nbad = int((out.view(torch.int32) != ref.view(torch.int32)).sum())
                bad.append(f"m={m} dim={dim} ffn={ffn}: {nbad} of {out.numel()} differ")
        gcu.check_device()
        gcu.comm_destroy()
    except Exception as e:
        bad.append(f"exception: {e}")
    finally:
        dist.destroy_process_group()
    q.put((rank, bad))


def test_ffn_two_gpus_equals_unsharded():
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
