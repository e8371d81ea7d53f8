#!/usr/bin/env python3
"""Benchmark of the W8A8 matmul hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload prefill1b|decode270m|lmhead4b|prefill4b|prefill12b|decode12b|
                                upload1b|upload4b]

Workloads (synthetic seeded data, no checkpoints):
  prefill1b   configs[1], the default: Gemma-3-1B-shaped prefill, M=512
              tokens, 26 layers.  One step = every layer's quantize_acts +
              Q/K/V, O, up/gate, down int8 GEMMs (gemma.c:5034-5391), inputs
              1% outlier channels x20.  Metric unit: int8 TOPS (2*M*N*K).
              At N>1 every rank runs its own replica (weak scaling).
  decode270m  configs[0]: Gemma-3-270m decode, batch 1: 18 layers of
              quantize_act + Q/K/V multi-GEMV, O, gate/up multi-GEMV, down,
              then the 262144-row lm_head GEMV.  Unit: HBM GB/s.
  lmhead4b    configs[2]: lm_head GEMV 262144 x 2560, batch 1, rows sharded
              over the ranks and all-gathered (strong scaling).
  prefill4b   configs[3]: SigLIP-So400m tower (27 layers, M=4096), the
              image projector (M=256) and the Gemma-3-4B text stack (34
              layers, M=2048).  Unit: int8 TOPS; N>1 runs replicas.
  prefill12b  configs[4] prefill: Gemma-3-12B, M=4096, 48 layers; at N>1 the
              FFN rows are sharded over the ranks and every FFN output is
              all-gathered (strong scaling).
  decode12b   configs[4] decode: Gemma-3-12B, batch 1, 48 layers + lm_head;
              at N>1 the lm_head rows, and at N>=4 the FFN rows too, are
              sharded (strong scaling).
  upload1b    not a BASELINE metric: gcu_register_model of a synthetic `-q`
  upload4b    model image (1B text / 4B text + SigLIP), GB/s of matmul
              weights into HBM against the measured PCIe copy rate.

`value` is measured with inputs resident in HBM, one CUDA graph replay per
step, CUDA events on the launching stream, max over ranks.  `e2e` is the same
metric through the host-pointer C ABI (gcu_quantize_acts / gcu_gemm_int8 /
gcu_gemv_int8 on pinned host buffers, copies inside the timed region).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "gemma.c_b200"))

METRIC = "W8A8 matmul: decode GEMV HBM GB/s, prefill GEMM int8 TOPS (% roofline)"


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------
PREFILL = {
    # name: (BASELINE configs index, title, stacks(synth) -> [(label, groups, M, layers)], FFN row-sharded)
    "prefill1b": (1, "Gemma-3-1B-shaped W8A8 prefill GEMM set",
                  lambda S: [("text", S.layer_groups(S.CONFIGS["1b"]), 512, 26)], False),
    "prefill4b": (3, "Gemma-3-4B-shaped W8A8 prefill with a SigLIP-So400m vision tower",
                  lambda S: [("vision", S.vision_layer_groups(S.CONFIGS["siglip"]), 4096, 27),
                             ("projector", S.projector_groups(S.CONFIGS["siglip"], S.CONFIGS["4b"]), 256, 1),
                             ("text", S.layer_groups(S.CONFIGS["4b"]), 2048, 34)], False),
    "prefill12b": (4, "Gemma-3-12B-shaped W8A8 prefill matmul set; each layer's FFN as one block (up/gate, "
                      "GeGLU, quantize, down) with its hidden dimension sharded over the GPUs",
                   lambda S: [("text", S.layer_groups(S.CONFIGS["12b"]), 4096, 48)], True),
}


def is_ffn(name):
    return name.startswith("w1") or name.startswith("w2") or name.startswith("w3")


class Prefill:
    """Prefill GEMM sets (configs[1], [3], [4]): stacks of identical layers,
    each layer the quantize_acts -> GEMM pairs of gemma.c (5034-5391 text,
    4497-4633 vision, 4714-4716 projector).  configs[4] runs each layer's FFN
    as one block (gcu_dev_ffn_rowshard: up/gate, GeGLU, quantize, down,
    gemma.c:5365-5391): unsharded on one GPU; at N > 1 its hidden dimension
    is split over the ranks (rows of up/gate, columns of down) and the ranks
    exchange row maxima and int32 partial sums, bit-exact; Q/K/V/O stay
    replicated."""

    def __init__(self, name="prefill1b", seed=0, fused=False, world=1, rank=0, layers=0, chain=False):
        import synth
        self.name = name
        self.index, self.title, stacks, shard = PREFILL[name]
        self.stacks = stacks(synth)
        if layers > 0:  # profiling captures of a small case: every stack cut to `layers` layers
            self.stacks = [(lb, g, m, min(nl, layers)) for lb, g, m, nl in self.stacks]
        self.fused, self.world, self.rank = fused, world, rank
        self.shard = shard and world > 1
        self.ffn_block = name == "prefill12b"
        self.chain = chain and not self.shard and not self.ffn_block
        self._chain = None
        self.needs_comm = self.shard
        self.m = self.stacks[-1][2]
        self.layers = sum(st[3] for st in self.stacks)
        self.ops = sum(synth.groups_ops(g, m) * nl for _, g, m, nl in self.stacks)
        self.seed = seed
        # single-stack workloads keep the flat view the host path uses
        self.groups = self.stacks[-1][1]

    def config(self):
        c = {"workload": f"{self.name} (configs[{self.index}]): {self.title}",
             "stacks": [{"stack": lb, "tokens_m": m, "layers": nl,
                         "gemms": [[n, k] for k, jobs in g for _, n in jobs]} for lb, g, m, nl in self.stacks],
             "calls_per_layer": ("quantize_acts->GEMM pairs, each one launch" if self.fused else
                                 "quantize_acts + one GEMM launch per group") +
                                " (weights sharing an input as one multi-weight launch)",
             "inputs": "1% outlier channels x20; per-layer weights+activations exceed L2 (no flush)"}
        if self.name == "prefill1b":
            c.update(tokens_m=self.m, layers=self.layers, d_model=self.groups[0][0], ffn=self.groups[3][0])
        if self.chain:
            c["calls_per_layer"] = "every quantize_acts -> GEMM pair of the step in chain launches (<= 22 pairs each)"
        if self.ffn_block:
            c["calls_per_layer"] = ("quantize_acts + one GEMM launch for Q/K/V and O; the FFN as one block "
                                    "(gcu_dev_ffn_rowshard)")
        if self.shard:
            c["sharding"] = (f"FFN hidden dimension over {self.world} GPUs (row maxima and int32 partial "
                             "sums all-reduced); Q/K/V/O replicated (counted once in value)")
        return c

    def build(self, device):
        import torch
        import synth
        gen = torch.Generator(device=device).manual_seed(1234 + self.seed)
        wgen = torch.Generator(device=device).manual_seed(4321)  # identical weights on every rank
        self.L, self.out, self.work = [], [], []
        for _, groups, m, nl in self.stacks:
            stack = []
            for _ in range(nl):
                layer = []
                for k, jobs in groups:
                    if self.ffn_block and jobs[0][0] == "w3_down":
                        continue  # part of the FFN block built with up/gate
                    if self.ffn_block and jobs[0][0] == "w1_up":
                        layer.append(self._ffn_record(synth, gen, wgen, device, m, k, jobs[0][1]))
                        continue
                    x = synth.activations_torch(m, k, gen, device, outliers=True)
                    q = torch.empty((m, k), dtype=torch.int8, device=device)
                    s = torch.empty(m, dtype=torch.float32, device=device)
                    sh = self.shard and all(is_ffn(nm) for nm, _ in jobs)
                    ws = []
                    for _, n in jobs:
                        if sh:
                            nl_rows = n // self.world
                            w, sc = synth.weight_torch(n, k, wgen, device)
                            r0 = self.rank * nl_rows
                            w, sc = w[r0:r0 + nl_rows].contiguous(), sc[r0:r0 + nl_rows].contiguous()
                        else:
                            w, sc = synth.weight_torch(n, k, gen, device)
                        ws.append((w, sc))
                    layer.append({"x": x, "q": q, "s": s, "k": k, "w": ws, "shard": sh,
                                  "n": [n for _, n in jobs]})
                stack.append(layer)
            self.L.append(stack)
            # output buffers (fp32) per group, shared by the stack's layers
            self.out.append([[torch.empty((m, n), dtype=torch.float32, device=device) for _, n in jobs]
                             for _, jobs in groups if not (self.ffn_block and jobs[0][0] == "w3_down")])
            self.work.append([[torch.empty((m, n), dtype=torch.float32, device=device) for _, n in jobs]
                              if self.shard and not self.ffn_block and all(is_ffn(nm) for nm, _ in jobs) else None
                              for _, jobs in groups if not (self.ffn_block and jobs[0][0] == "w3_down")])

    def _ffn_record(self, synth, gen, wgen, device, m, d, f):
        """One layer's FFN block: its input, the up/gate rows and the down
        columns this rank holds (all of them on one GPU)."""
        import torch
        x = synth.activations_torch(m, d, gen, device, outliers=True)
        src = wgen if self.shard else gen  # identical weights on every rank
        w1, s1 = synth.weight_torch(f, d, src, device)
        w2, s2 = synth.weight_torch(f, d, src, device)
        w3, s3 = synth.weight_torch(d, f, src, device)
        if self.shard:
            fl = f // self.world
            r0 = self.rank * fl
            w1, s1 = w1[r0:r0 + fl].contiguous(), s1[r0:r0 + fl].contiguous()
            w2, s2 = w2[r0:r0 + fl].contiguous(), s2[r0:r0 + fl].contiguous()
            w3 = w3[:, r0:r0 + fl].contiguous()
        return {"ffn": True, "x": x, "k": d, "f": f,
                "q": torch.empty((m, d), dtype=torch.int8, device=device),
                "s": torch.empty(m, dtype=torch.float32, device=device),
                "w1": (w1, s1), "w2": (w2, s2), "w3": (w3, s3),
                "out": torch.empty((m, d), dtype=torch.float32, device=device), "shard": False}

    @property
    def kinds(self):
        if self.chain:
            return ("chain",)
        if self.ffn_block:
            return ("quant", "gemm", "ffn")
        if self.shard:
            return ("quant", "gemm", "gemm_allgather")
        return ("qgemm",) if self.fused else ("quant", "gemm")

    def step(self, gcu, stream=None, want=None):
        """Enqueue one step.  `want(kind, bytes, ops)` filters the launches
        (and accounts their algorithmic work) for per-kernel timing."""
        if self.chain:
            # every quantize_acts -> GEMM pair of the step through the chain launch
            # (gcu_gemm_chain_*): built on the first (eager) step, outside any capture
            if self._chain is None:
                steps = []
                for si, (_, _, m, _) in enumerate(self.stacks):
                    for layer in self.L[si]:
                        for gi, g in enumerate(layer):
                            steps.append([g["x"], g["q"], g["s"],
                                          [(w, sc, o) for (w, sc), o in zip(g["w"], self.out[si][gi])]])
                self._chain = gcu.GemmChain(steps)
            nb = ops = 0
            for si, (_, groups, m, nl) in enumerate(self.stacks):
                for k, jobs in groups:
                    ns = sum(n for _, n in jobs)
                    nb += nl * (5 * m * k + 4 * m + ns * k + 4 * ns + m * k + 4 * m + 4 * m * ns)
                    ops += nl * 2 * m * ns * k
            if want is None or want("chain", nb, ops):
                self._chain.run(stream)
            return
        for si, (_, _, m, _) in enumerate(self.stacks):
            for layer in self.L[si]:
                for gi, g in enumerate(layer):
                    k = g["k"]
                    if g.get("ffn"):
                        f, (w1, s1), (w2, s2), (w3, s3) = g["f"], g["w1"], g["w2"], g["w3"]
                        if want is None or want("quant", 5 * m * k + 4 * m, 0):
                            gcu.dev_quantize_acts(g["q"], g["s"], g["x"], m, k, stream=stream)
                        fl = w1.shape[0]
                        # this rank's weights, the block's activations (up, gate, h in fp32, its
                        # codes) and output; ops of up, gate and down over this rank's slice
                        fb = 3 * (fl * k + 4 * fl) + m * k + 4 * m + 3 * 4 * m * fl + m * fl + 4 * m * k
                        if want is None or want("ffn", fb, 3 * 2 * m * fl * k):
                            gcu.dev_ffn_rowshard(g["out"], g["q"], g["s"], m, k, f, w1, s1, w2, s2, w3, s3,
                                                 stream=stream)
                        continue
                    outs = self.out[si][gi]
                    if g["shard"]:
                        if want is None or want("quant", 5 * m * k + 4 * m, 0):
                            gcu.dev_quantize_acts(g["q"], g["s"], g["x"], m, k, stream=stream)
                        for (w, sc), o, wk in zip(g["w"], outs, self.work[si][gi]):
                            nl, n = w.shape[0], o.shape[1]
                            if want is None or want("gemm_allgather", nl * k + 4 * nl + m * k + 4 * m + 4 * m * n,
                                                    2 * m * nl * k):
                                gcu.dev_gemm_int8_rowshard(o, wk, w, sc, g["q"], g["s"], m, n, k, stream=stream)
                        continue
                    nsum = sum(w.shape[0] for w, _ in g["w"])
                    jobs = [(w, sc, o) for (w, sc), o in zip(g["w"], outs)]
                    if self.fused:
                        qb = 5 * m * k + 4 * m
                        gb = nsum * k + 4 * nsum + m * k + 4 * m + 4 * m * nsum
                        if want is None or want("qgemm", qb + gb, 2 * m * nsum * k):
                            gcu.dev_quantize_gemm_int8_multi(jobs, g["q"], g["s"], g["x"], m, k, stream=stream)
                        continue
                    if want is None or want("quant", 5 * m * k + 4 * m, 0):
                        gcu.dev_quantize_acts(g["q"], g["s"], g["x"], m, k, stream=stream)
                    if want is not None and not want("gemm", nsum * k + 4 * nsum + m * k + 4 * m + 4 * m * nsum,
                                                     2 * m * nsum * k):
                        continue
                    if len(jobs) == 1:
                        w, sc, o = jobs[0]
                        gcu.dev_gemm_int8(o, w, sc, g["q"], g["s"], m, w.shape[0], k, stream=stream)
                    else:
                        gcu.dev_gemm_int8_multi(jobs, g["q"], g["s"], m, k, stream=stream)

    @property
    def launches_per_step(self):
        if self.chain:
            npairs = sum(nl * len(groups) for _, groups, _, nl in self.stacks)
            return -(-npairs // 22)
        n = 0
        for si, (_, groups, _, nl) in enumerate(self.stacks):
            for k, jobs in groups:
                if self.ffn_block and jobs[0][0] == "w3_down":
                    continue
                if self.ffn_block and jobs[0][0] == "w1_up":
                    # quantize; up/gate GEMM, GeGLU(+quantize), down GEMM; sharded: the two
                    # all-reduces, the separate quantize and the dequant
                    n += nl * (1 + (3 if not self.shard else 7))
                    continue
                sh = self.shard and all(is_ffn(nm) for nm, _ in jobs)
                n += nl * ((1 + len(jobs)) if sh else (1 if self.fused else 2))
        return n

    # ---- end to end through the host-pointer ABI --------------------------
    def build_host(self):
        import torch
        self.H = []
        for layer in self.L[-1]:
            hl = []
            for g in layer:
                x = torch.empty(g["x"].shape, dtype=torch.float32, pin_memory=True)
                x.copy_(g["x"].cpu())
                ws = []
                for w, sc in g["w"]:
                    ws.append((w.cpu().numpy(), sc.cpu().numpy()))
                hl.append({"x": x.numpy(), "k": g["k"], "w": ws,
                           "q": torch.empty((self.m, g["k"]), dtype=torch.int8, pin_memory=True).numpy(),
                           "s": torch.empty(self.m, dtype=torch.float32, pin_memory=True).numpy()})
            self.H.append(hl)
        self.Hout = [[torch.empty((self.m, n), dtype=torch.float32, pin_memory=True).numpy() for _, n in jobs]
                     for _, jobs in self.groups]
        self.h2d = self.d2h = 0
        for hl in self.H:
            for gi, g in enumerate(hl):
                mk = self.m * g["k"]
                self.h2d += 4 * mk + (mk + 4 * self.m) * len(g["w"])
                self.d2h += mk + 4 * self.m + sum(4 * self.m * w.shape[0] for w, _ in g["w"])
        return self.H

    def register_host(self, gcu):
        for hl in self.H:
            for g in hl:
                for w, s in g["w"]:
                    gcu.register_weight(w, s)

    def unregister_host(self, gcu):
        for hl in self.H:
            for g in hl:
                for w, _ in g["w"]:
                    gcu.unregister_weight(w)

    def step_host(self, gcu, rec=None):
        """One step through the host-pointer ABI in gemma.c's call order.
        rec(kind, seconds, h2d_bytes, d2h_bytes), when given, times each call."""
        lib = gcu.lib()
        m = self.m
        clock = time.perf_counter
        for hl in self.H:
            for gi, g in enumerate(hl):
                k = g["k"]
                t0 = clock()
                rc = lib.gcu_quantize_acts(g["q"].ctypes.data, g["s"].ctypes.data, g["x"].ctypes.data, 0, m, k)
                if rc:
                    raise RuntimeError(lib.gcu_last_error().decode())
                if rec:
                    rec(f"quantize_acts {m}x{k}", clock() - t0, 4 * m * k, m * k + 4 * m)
                for (w, s), o in zip(g["w"], self.Hout[gi]):
                    t0 = clock()
                    rc = lib.gcu_gemm_int8(o.ctypes.data, 0, w.ctypes.data, 0, s.ctypes.data, g["q"].ctypes.data,
                                           0, g["s"].ctypes.data, m, w.shape[0], k)
                    if rc:
                        raise RuntimeError(lib.gcu_last_error().decode())
                    if rec:
                        rec(f"gemm_int8 {m}x{w.shape[0]}x{k}", clock() - t0, m * k + 4 * m, 4 * m * w.shape[0])

    def host_call_breakdown(self, gcu):
        """Per call kind of one (untimed) host step: calls, average us, bytes
        each way per call and the bytes/second the call achieved."""
        acc = {}

        def rec(kind, dt, h2d, d2h):
            a = acc.setdefault(kind, [0, 0.0, h2d, d2h])
            a[0] += 1
            a[1] += dt
        self.step_host(gcu, rec)
        return {kind: {"calls": n, "avg_us": round(t / n * 1e6, 1), "h2d_mb": round(h / 1e6, 3),
                       "d2h_mb": round(d / 1e6, 3), "gbs": round((h + d) * n / t / 1e9, 1)}
                for kind, (n, t, h, d) in acc.items()}

    # ---- CPU reference ---------------------------------------------------------
    def cpu_sample(self, R, layers):
        """Time `layers` layers of every stack with the reference's own
        quantize_acts + gemm_int8 (OpenMP over all threads), in gemma.c's
        call pattern: a text layer's Q/K/V as per-(head, 128-token) tasks
        (gemma.c:5037-5091, head size 256), every other weight one
        gemm_int8 call with omp = true."""
        import numpy as np
        import synth
        data = []
        ops = 0
        for si, (_, groups, m, _) in enumerate(self.stacks):
            for li in range(layers):
                layer = []
                for gi, (k, jobs) in enumerate(groups):
                    x = synth.activations(9000 + 100 * si + 10 * li + gi, m, k, outliers=True)
                    ws = [synth.weight(9500 + 100 * si + 10 * li + 3 * gi + j, n, k) for j, (_, n) in enumerate(jobs)]
                    outs = [np.empty((m, n), np.float32) for _, n in jobs]
                    layer.append((x, ws, outs))
                data.append(layer)
            ops += synth.groups_ops(groups, m) * layers

        head_tasks = [label == "text" and hasattr(R.lib, "ref_qkv_head_tasks")
                      for label, _, _, _ in self.stacks for _ in range(layers)]
        qkv_outs = {}

        def run():
            for li, layer in enumerate(data):
                for gi, (x, ws, outs) in enumerate(layer):
                    q, s = R.quantize_acts(x)
                    if gi == 0 and head_tasks[li] and len(ws) == 3:
                        (wq, sq), (wk, sk), (wv, sv) = ws
                        key = (li, q.shape[0])
                        qkv_outs[key] = R.qkv_head_tasks(wq, sq, wk, sk, wv, sv, q, s, 256, qkv_outs.get(key))
                        continue
                    for (w, sc), o in zip(ws, outs):
                        R.gemm_int8(w, sc, q, s, dst=o)
        return ops, run


# The decode FFN rows are sharded from this many GPUs on: below it the
# per-layer all-gathers cost more than the smaller FFN slices save.
FFN_SHARD_MIN_GPUS = 4

DECODE = {
    # name: (configs index, model, rows sharded at N > 1)
    "decode270m": (0, "270m", False),
    "decode12b": (4, "12b", True),
}


class Decode:
    """Decode, batch 1 (configs[0], and configs[4]'s decode half): every
    layer's quantize_act -> Q/K/V, O, gate/up, down GEMVs, then the
    262144-row lm_head.  Sharded workloads split the lm_head rows over the
    ranks, and from FFN_SHARD_MIN_GPUS ranks on the FFN rows too, with the
    all-gather fused into the GEMV when the peers are mapped
    (gcu_dev_gemm_int8_rowshard); Q/K/V/O stay replicated.  (At 2 GPUs the
    per-layer FFN all-gathers cost more than the halved FFN slices save:
    12B step 2.69 ms with them against 2.565 ms on one GPU.)"""

    def __init__(self, name="decode270m", seed=0, fused=True, world=1, rank=0, layers=0):
        import synth
        self.name = name
        self.index, cfg, shard = DECODE[name]
        self.fused = fused
        self.world, self.rank = world, rank
        self.shard = shard and world > 1
        self.shard_ffn = self.shard and world >= FFN_SHARD_MIN_GPUS
        self.needs_comm = self.shard
        self.cfg = synth.CONFIGS[cfg]
        self.groups = synth.layer_groups(self.cfg)
        self.layers = min(self.cfg["layers"], layers) if layers > 0 else self.cfg["layers"]
        self.bytes = (synth.layer_weight_bytes(self.cfg) * self.layers +
                      self.cfg["vocab"] * (self.cfg["dim"] + 4))
        self.seed = seed

    def config(self):
        import gcu
        c = {"workload": f"{self.name} (configs[{self.index}]): Gemma-3-{self.name[6:]} W8A8 decode, batch 1, "
                         f"{self.layers} layers + lm_head",
             "vocab": self.cfg["vocab"], "d_model": self.cfg["dim"],
             "inputs": f"{self.bytes / 1e6:.0f} MB of weights per token > L2 (no flush)",
             "calls": "quantize_act->gemv pairs fused into one launch each" if self.fused else
                      "quantize_act and gemv_int8(_multi) as separate launches"}
        if self.shard:
            ag = "fused into the GEMV (NVLink peer loads)" if gcu.comm_fused_allgather() else "NCCL"
            rows = "FFN and lm_head rows" if self.shard_ffn else "lm_head rows (FFN replicated below 4 GPUs)"
            c["sharding"] = (f"{rows} over {self.world} GPUs, all-gather {ag}; "
                             "Q/K/V/O replicated (counted once in value)")
        return c

    def build(self, device):
        import torch
        import synth
        gen = torch.Generator(device=device).manual_seed(99 + self.seed)
        wgen = torch.Generator(device=device).manual_seed(4321)

        def weight(n, k, sharded):
            if not sharded:
                return synth.weight_torch(n, k, gen, device)
            nl = n // self.world
            w, sc = synth.weight_torch(n, k, wgen, device)
            r0 = self.rank * nl
            return w[r0:r0 + nl].contiguous(), sc[r0:r0 + nl].contiguous()

        self.L = []
        for _ in range(self.layers):
            layer = []
            for k, jobs in self.groups:
                sh = self.shard_ffn and all(is_ffn(nm) for nm, _ in jobs)
                layer.append({"x": synth.activations_torch(1, k, gen, device),
                              "q": torch.empty(k, dtype=torch.int8, device=device),
                              "s": torch.empty(1, dtype=torch.float32, device=device), "k": k, "shard": sh,
                              "w": [weight(n, k, sh) for _, n in jobs],
                              "o": [torch.empty(n, dtype=torch.float32, device=device) for _, n in jobs],
                              "work": [torch.empty(n, dtype=torch.float32, device=device) for _, n in jobs]
                              if sh else None})
            self.L.append(layer)
        d = self.cfg["dim"]
        self.head = {"x": synth.activations_torch(1, d, gen, device), "q": torch.empty(d, dtype=torch.int8, device=device),
                     "s": torch.empty(1, dtype=torch.float32, device=device),
                     "w": weight(self.cfg["vocab"], d, self.shard),
                     "o": torch.empty(self.cfg["vocab"], dtype=torch.float32, device=device),
                     "work": torch.empty(self.cfg["vocab"], dtype=torch.float32, device=device)}

    @property
    def kinds(self):
        base = ("qgemv",) if self.fused else ("quant", "gemv")
        if self.shard:
            return base + ("qgemv_allgather",)
        return base

    def _sharded(self, gcu, x, q, s, k, ws, outs, works, stream, want):
        # quantize + every sharded weight of the group + their all-gathers:
        # one launch when the peers are mapped
        nl = sum(w.shape[0] for w, _ in ws)
        n = sum(o.shape[0] for o in outs)
        if want is None or want("qgemv_allgather", nl * (k + 8) + 6 * k + 8 + 4 * n, 2 * nl * k):
            gcu.dev_quantize_gemm_int8_rowshard_multi([(w, sc, o, o.shape[0]) for (w, sc), o in zip(ws, outs)],
                                                      q, s, x, 1, k, work=works[0], stream=stream)

    def step(self, gcu, stream=None, want=None):
        h = self.head
        d = self.cfg["dim"]
        n = self.cfg["vocab"]
        if self.fused or self.shard:
            for layer in self.L:
                for g in layer:
                    k = g["k"]
                    if g["shard"]:
                        self._sharded(gcu, g["x"], g["q"], g["s"], k, g["w"], g["o"], g["work"], stream, want)
                        continue
                    nsum = sum(w.shape[0] for w, _ in g["w"])
                    if self.fused:
                        if want is None or want("qgemv", nsum * (k + 8) + 6 * k + 8, 2 * nsum * k):
                            gcu.dev_quantize_gemm_int8_multi([(w, sc, o) for (w, sc), o in zip(g["w"], g["o"])],
                                                             g["q"], g["s"], g["x"], 1, k, stream=stream)
                        continue
                    if want is None or want("quant", 5 * k + 4, 0):
                        gcu.dev_quantize_acts(g["q"], g["s"], g["x"], 1, k, stream=stream)
                    if want is None or want("gemv", nsum * (k + 8) + k + 4, 2 * nsum * k):
                        gcu.dev_gemv_int8_multi([(w, sc, o) for (w, sc), o in zip(g["w"], g["o"])], g["q"],
                                                g["s"], k, stream=stream)
            if self.shard:
                self._sharded(gcu, h["x"], h["q"], h["s"], d, [h["w"]], [h["o"]], [h["work"]], stream, want)
            elif want is None or want("qgemv", n * (d + 8) + 6 * d + 8, 2 * n * d):
                gcu.dev_quantize_gemm_int8_multi([(h["w"][0], h["w"][1], h["o"])], h["q"], h["s"], h["x"], 1, d,
                                                 stream=stream)
            return
        for layer in self.L:
            for g in layer:
                k = g["k"]
                if want is None or want("quant", 5 * k + 4, 0):
                    gcu.dev_quantize_acts(g["q"], g["s"], g["x"], 1, k, stream=stream)
                nsum = sum(w.shape[0] for w, _ in g["w"])
                if want is None or want("gemv", nsum * (k + 8) + k + 4, 2 * nsum * k):
                    gcu.dev_gemv_int8_multi([(w, sc, o) for (w, sc), o in zip(g["w"], g["o"])], g["q"], g["s"],
                                            k, stream=stream)
        if want is None or want("quant", 5 * d + 4, 0):
            gcu.dev_quantize_acts(h["q"], h["s"], h["x"], 1, d, stream=stream)
        if want is None or want("gemv", n * (d + 8) + d + 4, 2 * n * d):
            gcu.dev_gemv_int8(h["o"], h["w"][0], h["w"][1], h["q"], h["s"], n, d, stream=stream)

    @property
    def launches_per_step(self):
        if not self.shard:
            return (self.layers * len(self.groups) + 1) * (1 if self.fused else 2)
        n = 1  # lm_head: one fused quantize + sharded GEMV
        for k, jobs in self.groups:
            if self.shard_ffn and all(is_ffn(nm) for nm, _ in jobs):
                n += self.layers
            else:
                n += self.layers * (1 if self.fused else 2)
        return n


class LmHead:
    """lm_head GEMV 262144 x 2560, rows sharded over ranks."""
    name = "lmhead4b"

    def __init__(self, world, rank, vocab=262144, dim=2560, batch=1):
        self.world, self.rank = world, rank
        self.needs_comm = world > 1
        self.n, self.k, self.b = vocab, dim, batch
        self.bytes = vocab * (dim + 4) + batch * (dim + 4) + 4 * batch * vocab

    def config(self):
        import gcu
        ag = "all-gather fused into the GEMV (NVLink peer loads)" if (self.world > 1 and gcu.comm_fused_allgather()) else \
            "NCCL all-gather"
        return {"workload": f"lmhead4b (configs[2]): lm_head GEMV {self.n} x {self.k}, batch {self.b}, "
                            f"rows sharded over {self.world} GPU(s) + {ag}",
                "inputs": "672 MB of weights > L2 (no flush)"}

    def build(self, device):
        import torch
        import synth
        gen = torch.Generator(device=device).manual_seed(7 + self.rank)
        nl = self.n // self.world
        self.w, self.ws = synth.weight_torch(nl, self.k, gen, device)
        x = synth.activations_torch(self.b, self.k, torch.Generator(device=device).manual_seed(5), device)
        self.q = torch.empty((self.b, self.k), dtype=torch.int8, device=device)
        self.s = torch.empty(self.b, dtype=torch.float32, device=device)
        self.x = x
        self.y = torch.empty((self.b, self.n), dtype=torch.float32, device=device)
        self.work = torch.empty((self.b, self.n), dtype=torch.float32, device=device)

    @property
    def kinds(self):
        return ("quant", "gemv") if self.world == 1 else ("quant", "gemv_allgather")

    def step(self, gcu, stream=None, want=None):
        if want is None or want("quant", 5 * self.b * self.k + 4 * self.b, 0):
            gcu.dev_quantize_acts(self.q, self.s, self.x, self.b, self.k, stream=stream)
        if self.world == 1:
            if want is None or want("gemv", self.bytes, 2 * self.b * self.n * self.k):
                gcu.dev_gemm_int8(self.y, self.w, self.ws, self.q, self.s, self.b, self.n, self.k, stream=stream)
        elif want is None or want("gemv_allgather", self.bytes // self.world + 4 * self.b * self.n,
                                  2 * self.b * (self.n // self.world) * self.k):
            gcu.dev_gemm_int8_rowshard(self.y, self.work, self.w, self.ws, self.q, self.s, self.b, self.n,
                                       self.k, stream=stream)

    launches_per_step = property(lambda self: 2)
    fused = False


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def make_workload(name, args, world, rank, batch=1):
    if name in PREFILL:
        return Prefill(name, seed=rank, fused=args.fused, world=world, rank=rank, layers=args.layers,
                       chain=getattr(args, "chain", False))
    if name in DECODE:
        return Decode(name, seed=rank, fused=not args.unfused, world=world, rank=rank, layers=args.layers)
    return LmHead(world, rank, batch=batch)


def time_workload(wl, gcu, stream, args, world):
    """Eager warm-up, CUDA-graph capture where the step holds no NCCL call,
    `warmup` untimed steps, then `steps` timed steps between CUDA events on
    the launching stream.  Returns (ms per step, max over ranks; graph)."""
    import torch
    with torch.cuda.stream(stream):
        wl.step(gcu)  # allocates the split-K workspace before capture
    stream.synchronize()
    gcu.check_device()
    # a sharded step is graph-captured only when every all-gather is the fused
    # peer-load GEMV (no NCCL call inside the step): sharded decode with the
    # peers mapped, never sharded prefill (m > 8 all-gathers through NCCL)
    use_graph = not wl.needs_comm or (not isinstance(wl, Prefill) and gcu.comm_fused_allgather())
    graph = None
    if use_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            wl.step(gcu)
    torch.cuda.synchronize()

    def one():
        if graph is not None:
            graph.replay()
        else:
            with torch.cuda.stream(stream):
                wl.step(gcu)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            one()
    torch.cuda.synchronize()
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            one()
        e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    gcu.check_device()
    return ms, graph


def class_profile(wl, gcu, stream, steps):
    """Per-kernel-class durations: the step's launches of one kernel class
    only (same inputs, same order), captured as a CUDA graph and replayed
    `steps` times between CUDA events on the launching stream; the average
    launch duration includes the graph's inter-kernel gap."""
    import torch
    prof = {}
    for kind in wl.kinds:
        acc = {"launches": 0, "bytes": 0, "ops": 0}

        def want(k, nbytes, ops, kind=kind, acc=acc):
            if k != kind:
                return False
            acc["launches"] += 1
            acc["bytes"] += nbytes
            acc["ops"] += ops
            return True

        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            wl.step(gcu, want=want)
        with torch.cuda.stream(stream):
            for _ in range(2):
                g.replay()
            k0 = torch.cuda.Event(enable_timing=True)
            k1 = torch.cuda.Event(enable_timing=True)
            k0.record(stream)
            for _ in range(steps):
                g.replay()
            k1.record(stream)
        torch.cuda.synchronize()
        prof[kind] = {"launches": acc["launches"] * steps, "ms": k0.elapsed_time(k1),
                      "bytes": acc["bytes"] * steps, "ops": acc["ops"] * steps}
        del g
    return prof


def roofline_of(prof, peaks, traffic_file=None, kind=None):
    """Roofline of the dominant kernel class (or of `kind`) from class_profile
    numbers: algorithmic bytes (ops) per launch over the average launch."""
    int8_peak = 2.0 * peaks["bf16_tflops"]
    dom = kind or max(prof, key=lambda k: prof[k]["ms"])
    d = prof[dom]
    t = d["ms"] * 1e-3
    t_hbm = d["bytes"] / (peaks["hbm_gbs"] * 1e9)
    t_tc = d["ops"] / (int8_peak * 1e12) if d["ops"] else 0.0
    if t_tc > t_hbm:
        roof = {"bound": "tensor", "achieved": d["ops"] / t / 1e12, "peak": int8_peak, "unit": "TOPS",
                "peak_src": f"2 x {peaks['src']} bf16 dense"}
    else:
        roof = {"bound": "hbm", "achieved": d["bytes"] / t / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "peak_src": f"{peaks['src']} copy bandwidth"}
    roof.update(frac=roof["achieved"] / roof["peak"], kernel=dom, launches=d["launches"],
                avg_launch_us=d["ms"] * 1e3 / d["launches"],
                bytes_per_launch=d["bytes"] / d["launches"], ops_per_launch=d["ops"] / d["launches"],
                roofline_time_frac=max(t_hbm, t_tc) / t, traffic=None)
    if traffic_file and os.path.exists(traffic_file):
        # ncu dram__bytes_read.sum + dram__bytes_write.sum per launch of this
        # class, from a capture of the same build (profiles/); the fp32
        # outputs usually leave L2 after the kernel ends, so the in-kernel
        # write counter can read ~0 and the figure is then reads-only, to be
        # set against the algorithmic READ bytes recorded beside it
        rec = json.load(open(traffic_file)).get("kernels", {}).get(dom)
        if rec is not None:
            roof["traffic"] = rec["read_bytes"] + rec["write_bytes"]
            roof["traffic_detail"] = rec
    kernels = {k: {"launches": v["launches"], "share": v["ms"] / sum(x["ms"] for x in prof.values()),
                   "avg_us": v["ms"] * 1e3 / v["launches"]} for k, v in prof.items()}
    return roof, kernels


def run_ours(args):
    import torch
    world, rank, local = dist_setup(args)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    import gcu
    gcu.init(local)
    peaks = load_peaks()
    wl = make_workload(args.workload, args, world, rank)
    comm_on = False
    if wl.needs_comm or (args.workload == "prefill1b" and world > 1 and not args.no_decode):
        comm_init(gcu, rank, world)
        comm_on = True
    wl.build(device)
    torch.cuda.synchronize()

    stream = torch.cuda.Stream(device)
    barrier(world)
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.3)
    ms, graph = time_workload(wl, gcu, stream, args, world)
    clk = clocks.stop()
    prof = class_profile(wl, gcu, stream, args.steps) if graph is not None else {}

    out = {"metric": METRIC, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": ms, "higher_is_better": True, "vs_baseline": None, "data": "synthetic",
           "impl": "ours"}
    # replicas: every rank runs the whole workload (weak scaling, value sums
    # them); sharded: the ranks share one workload (strong scaling)
    copies = 1 if wl.needs_comm else world
    par = (f"row-shard x{world}" if wl.needs_comm else f"replicas x{world}") if world > 1 else "single GPU"
    if isinstance(wl, Prefill):
        out.update(value=wl.ops * copies / (ms * 1e-3) / 1e12, unit="int8 TOPS",
                   dtype="int8 (int32 accum, fp32 out)", scaling="strong" if wl.needs_comm else "weak")
        cfg = wl.config()
        cfg.update(parallelism=par)
    elif isinstance(wl, Decode):
        out.update(value=wl.bytes * copies / (ms * 1e-3) / 1e9, unit="GB/s", dtype="int8 (int32 accum, fp32 out)",
                   scaling="strong" if wl.needs_comm else "weak")
        cfg = wl.config()
        cfg.update(parallelism=par)
    else:
        out.update(value=wl.bytes / (ms * 1e-3) / 1e9, unit="GB/s", dtype="int8 (int32 accum, fp32 out)",
                   scaling="strong")
        cfg = wl.config()
        cfg.update(parallelism=f"row-shard x{world}" if world > 1 else "single GPU")
    if args.layers > 0:
        cfg["reduced"] = f"--layers {args.layers}: a profiling case, not the benchmark workload"
    out["config"] = cfg
    out["clocks"] = clk
    out["gpu_launches"] = wl.launches_per_step * args.steps

    # roofline of the dominant kernel
    if prof:
        out["roofline"], out["kernels"] = roofline_of(
            prof, peaks, os.path.join(ROOT, "profiles", f"traffic_{wl.name}.json"))

    # end to end through the host-pointer ABI
    if isinstance(wl, Prefill) and wl.name == "prefill1b" and not args.no_e2e:
        wl.build_host()
        wl.register_host(gcu)
        wl.step_host(gcu)  # warm-up
        torch.cuda.synchronize()
        barrier(world)
        esteps = max(1, min(args.steps, 3))
        t0 = time.perf_counter()
        for _ in range(esteps):
            wl.step_host(gcu)
        t1 = time.perf_counter()
        e_ms = (t1 - t0) * 1e3 / esteps
        e_ms = max_over_ranks(e_ms, world)
        out["e2e"] = {"value": wl.ops * world / (e_ms * 1e-3) / 1e12, "unit": "int8 TOPS", "ms_per_step": e_ms,
                      "h2d_bytes_per_step": wl.h2d, "d2h_bytes_per_step": wl.d2h,
                      "path": "gcu_quantize_acts + gcu_gemm_int8 host-pointer ABI, registered weights, "
                              "pinned host activations, wall clock around synchronous calls",
                      "calls": wl.host_call_breakdown(gcu)}
        wl.unregister_host(gcu)

    # CPU baseline on rank 0 at N=1 (bounded sample)
    if world == 1 and not args.no_cpu and isinstance(wl, Prefill) and wl.name == "prefill1b":
        out["cpu_baseline"] = cpu_baseline(wl, args.cpu_seconds)

    if graph is not None:
        del graph
    # the decode half of the metric (configs[2] and configs[0] at N=1; the
    # row-sharded lm_head and 12B decode at N>1), each with its roofline
    if args.workload == "prefill1b" and not args.no_decode and args.layers == 0:
        del wl
        torch.cuda.empty_cache()
        out["decode"] = decode_records(args, gcu, world, rank, device, stream, peaks)
        out["ffn12b"] = ffn_record(args, gcu, world, rank, device, stream)
    if comm_on:
        gcu.comm_destroy()
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def comm_init(gcu, rank, world):
    import torch.distributed as dist
    uid = gcu.comm_unique_id() if rank == 0 else None
    obj = [uid]
    dist.broadcast_object_list(obj, src=0)
    gcu.comm_init(rank, world, obj[0])


def decode_records(args, gcu, world, rank, device, stream, peaks):
    """The decode-GEMV half of BASELINE's metric, in HBM GB/s with its
    roofline.  N=1: configs[2]'s lm_head GEMV 262144 x 2560 at batch 1 and
    8, and configs[0]'s Gemma-3-270m decode step, each beside the reference's
    own gemv_int8 / gemv_int8_multi (gemma.c:2765-2837) on the host cores.
    N>1: the row-sharded lm_head and the 12B decode step with
    FFN and lm_head rows sharded, with the share of the step
    spent in the launches that carry the all-gather."""
    import torch
    rec = {}
    if world == 1:
        cases = [("lmhead4b_b1", "lmhead4b", 1), ("lmhead4b_b8", "lmhead4b", 8), ("decode270m", "decode270m", 1)]
    else:
        cases = [("lmhead4b_b1", "lmhead4b", 1), ("decode12b", "decode12b", 1)]
    for key, name, batch in cases:
        wl = make_workload(name, args, world, rank, batch=batch)
        wl.build(device)
        torch.cuda.synchronize()
        ms, graph = time_workload(wl, gcu, stream, args, world)
        prof = class_profile(wl, gcu, stream, args.steps) if graph is not None else {}
        r = {"workload": wl.config()["workload"], "unit": "GB/s", "ms_per_step": ms,
             "value": wl.bytes / (ms * 1e-3) / 1e9 * (1 if wl.needs_comm else world),
             "scaling": "strong" if wl.needs_comm else "weak"}
        if prof:
            gemv_kind = max((k for k in wl.kinds if "gemv" in k), key=lambda k: prof[k]["ms"])
            tf = os.path.join(ROOT, "profiles", f"traffic_{name}.json") if batch == 1 and world == 1 else None
            r["roofline"], r["kernels"] = roofline_of(prof, peaks, tf, kind=gemv_kind)
            if world > 1:
                ag = {k: v for k, v in prof.items() if "allgather" in k}
                tot = sum(v["ms"] for v in prof.values())
                r["allgather_launch_share"] = sum(v["ms"] for v in ag.values()) / tot if tot else None
                for k, v in ag.items():
                    # time over the HBM floor of the rank's own rows: the
                    # cross-rank hand-off and the NVLink pull of the others'
                    floor_us = v["bytes"] / v["launches"] / (peaks["hbm_gbs"] * 1e9) * 1e6
                    r.setdefault("allgather_overhead_us_per_launch", {})[k] = \
                        v["ms"] * 1e3 / v["launches"] - floor_us
        if world == 1 and rank == 0 and not args.no_cpu:
            r["cpu_baseline"] = decode_cpu_baseline(wl, args.cpu_seconds / 4)
        rec[key] = r
        del graph, wl, prof
        torch.cuda.empty_cache()
    return rec


def ffn_record(args, gcu, world, rank, device, stream, layers=4):
    """The Gemma-3-12B FFN block of configs[4] (M = 4096 tokens, dim 3840,
    ffn 15360) through gcu_dev_ffn_rowshard over `layers` layers: unsharded at
    N = 1; at N > 1 the hidden dimension split over the ranks, with the row
    maxima and the int32 partial sums all-reduced (bit-exact, strong scaling:
    the same total work at every N).  A block-level record (the full 48-layer
    prefill12b step is `--workload prefill12b`)."""
    import torch
    import synth
    m, d, f = 4096, 3840, 15360
    fl = f // world
    r0 = rank * fl
    wgen = torch.Generator(device=device).manual_seed(4321)
    L = []
    for _ in range(layers):
        x = synth.activations_torch(m, d, wgen, device, outliers=True)
        q = torch.empty((m, d), dtype=torch.int8, device=device)
        s = torch.empty(m, dtype=torch.float32, device=device)
        gcu.dev_quantize_acts(q, s, x, m, d)
        del x
        w1, s1 = synth.weight_torch(f, d, wgen, device)
        w2, s2 = synth.weight_torch(f, d, wgen, device)
        w3, s3 = synth.weight_torch(d, f, wgen, device)
        L.append((q, s, w1[r0:r0 + fl].contiguous(), s1[r0:r0 + fl].contiguous(), w2[r0:r0 + fl].contiguous(),
                  s2[r0:r0 + fl].contiguous(), w3[:, r0:r0 + fl].contiguous(), s3,
                  torch.empty((m, d), dtype=torch.float32, device=device)))
        del w1, w2, w3
    torch.cuda.synchronize()

    def step():
        for q, s, w1, s1, w2, s2, w3, s3, out in L:
            gcu.dev_ffn_rowshard(out, q, s, m, d, f, w1, s1, w2, s2, w3, s3, stream=stream)

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            step()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(1, min(args.steps, 10))
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            step()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / reps / layers, world)
    gcu.check_device()
    ops = 3 * 2 * m * f * d
    rec = {"workload": "Gemma-3-12B FFN block (configs[4]): M=4096, dim 3840, ffn 15360; up/gate, GeGLU, "
                       "quantize, down per layer",
           "sharding": ("hidden dimension over %d GPUs: row maxima and int32 partial sums all-reduced (exact)"
                        % world) if world > 1 else "single GPU, unsharded",
           "unit": "int8 TOPS", "ms_per_layer": ms, "value": ops / (ms * 1e-3) / 1e12, "layers_timed": layers,
           "scaling": "strong"}
    del L
    torch.cuda.empty_cache()
    return rec


def decode_cpu_baseline(wl, seconds):
    """The reference's own GEMV code on the host cores (all threads) over the
    same weights: gemv_int8 (batch 1) or gemm_int8 (batch 8) for the
    lm_head; for a decode step, per layer quantize_act + gemv_int8_multi for
    Q/K/V and gate/up, gemv_int8 for O and down, then the lm_head, as
    forward_text_decode issues them (gemma.c:4768-4966)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    threads = os.cpu_count() or 1
    variant = oracle.ref_variant()
    if variant is None:
        return {"value": None, "unit": "GB/s", "cores": threads, "kind": "reference",
                "sample": "reference build not runnable on this host"}
    R = oracle.Ref(variant, threads=threads)
    if isinstance(wl, LmHead):
        w, ws = wl.w.cpu().numpy(), wl.ws.cpu().numpy()
        x = wl.x.cpu().numpy()
        q, s = R.quantize_acts(x)
        out = np.empty((wl.b, w.shape[0]), np.float32)
        if wl.b == 1:
            def run():
                qq, ss = R.quantize_act(x[0])
                R.gemv_int8(w, ws, qq, ss, dst=out[0])
            what = "gemma.c quantize_act + gemv_int8 (gemma.c:2765-2788)"
        else:
            def run():
                R.quantize_acts(x)
                R.gemm_int8(w, ws, q, s, dst=out)
            what = "gemma.c quantize_acts + gemm_int8 at m = 8 (gemma.c:3937-4054)"
        nbytes = wl.bytes
    else:
        layers = [[(g["x"].cpu().numpy()[0], [(w.cpu().numpy(), sc.cpu().numpy()) for w, sc in g["w"]])
                   for g in layer] for layer in wl.L]
        hw, hs = wl.head["w"][0].cpu().numpy(), wl.head["w"][1].cpu().numpy()
        hx = wl.head["x"].cpu().numpy()[0]
        outs = [[[np.empty(w.shape[0], np.float32) for w, _ in ws] for _, ws in layer] for layer in layers]
        hout = np.empty(hw.shape[0], np.float32)

        def run():
            for layer, lo in zip(layers, outs):
                for (x, ws), o in zip(layer, lo):
                    q, s = R.quantize_act(x)
                    if len(ws) > 1:
                        R.gemv_int8_multi([w for w, _ in ws], [sc for _, sc in ws], q, s, outs=o)
                    else:
                        R.gemv_int8(ws[0][0], ws[0][1], q, s, dst=o[0])
            q, s = R.quantize_act(hx)
            R.gemv_int8(hw, hs, q, s, dst=hout)
        what = ("gemma.c per layer quantize_act + gemv_int8_multi (Q/K/V, gate/up) / gemv_int8 (O, down), "
                "then the lm_head (gemma.c:4768-4966)")
        nbytes = wl.bytes
    run()  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        run()
        n += 1
        if time.perf_counter() - t0 > seconds or n >= 20:
            break
    dt = (time.perf_counter() - t0) / n
    return {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "reference",
            "sample": f"{what}, {n} reps of the whole step, {oracle.ref_build_desc(variant)}; {R.isa} kernels",
            "ms_per_step": dt * 1e3}


def cpu_baseline(wl, seconds):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    threads = os.cpu_count() or 1
    variant = oracle.ref_variant()
    if variant is not None:
        R = oracle.Ref(variant, threads=threads)
        kind = "reference"
        desc = f"gemma.c quantize_acts+gemm_int8 ({oracle.ref_build_desc(variant)}; {R.isa} kernels)"
    else:
        return {"value": None, "unit": "int8 TOPS", "cores": threads, "kind": "reference",
                "sample": "reference build not runnable on this host"}
    ops, run = wl.cpu_sample(R, 1)
    run()  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        run()
        n += 1
        if time.perf_counter() - t0 > seconds or n >= 50:
            break
    dt = (time.perf_counter() - t0) / n
    return {"value": ops / dt / 1e12, "unit": "int8 TOPS", "cores": threads, "kind": kind,
            "sample": f"1 of {wl.layers} layers of the same step (M={wl.m}), {n} reps, {desc}",
            "ms_per_layer": dt * 1e3}


# ---------------------------------------------------------------------------
# model upload (gcu_register_model): a `-q` model image -> one HBM arena
# ---------------------------------------------------------------------------
UPLOAD = {"upload1b": ("Gemma-3-1B text decoder", "TEXT_1B", None),
          "upload4b": ("Gemma-3-4B text decoder + SigLIP tower", "TEXT_4B", "VISION_SIGLIP")}


def run_upload(args):
    """One step = gcu_register_model of a synthetic `-q` image (timed on the
    host clock around the synchronous call: parse, arena allocation, packed
    pinned copies, registry insert), then gcu_unregister_arena (untimed).
    Two sources: the image resident in process memory, and a FRESH mmap of
    the same file in the page cache every step (gemma.c's mmap path,
    gemma.c:1946-2043: each step pays the page faults).  Beside them: the
    per-weight gcu_register_weight loop, a plain pinned cudaMemcpy (the
    PCIe roofline) and the reference's own read_gemma_model of the file."""
    import mmap
    import tempfile

    import numpy as np
    import torch

    import binfmt
    import gcu
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    gcu.init(0)
    torch.cuda.set_device(0)
    title, tkey, vkey = UPLOAD[args.workload]
    text, vision = getattr(binfmt, tkey), (getattr(binfmt, vkey) if vkey else None)
    buf, _ = binfmt.image(text, vision, seed=1, fast=True)
    recs = gcu.bin_qtensors(buf)
    wbytes = sum(r["rows"] * r["k"] + 4 * r["rows"] for r in recs)

    arenas = []

    def step_resident():
        arenas.append(gcu.register_model(buf))

    def drop():
        while arenas:
            gcu.unregister_arena(arenas.pop())

    for _ in range(args.warmup):
        step_resident()
        drop()
    ts = []
    clocks = Clocks(0)
    clocks.start()
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step_resident()
        ts.append(time.perf_counter() - t0)
        drop()
    clk = clocks.stop()
    t_res = statistics.median(ts)

    # fresh mapping of the page-cached file per step
    tmpdir = tempfile.mkdtemp(prefix="gcu_upload_")
    path = os.path.join(tmpdir, "model.bin")
    buf.tofile(path)
    ts = []
    for i in range(args.warmup + args.steps):
        with open(path, "rb") as f:
            mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        img = np.frombuffer(mm, np.uint8)
        t0 = time.perf_counter()
        a = gcu.register_model(img)
        t1 = time.perf_counter()
        gcu.unregister_arena(a)
        del img
        mm.close()
        if i >= args.warmup:
            ts.append(t1 - t0)
    t_mmap = statistics.median(ts)

    # per-weight registration (one cudaMalloc + two pageable copies each)
    def per_weight():
        views = [binfmt.qtensor_arrays(buf, r) for r in recs]
        for q, s in views:
            gcu.lib().gcu_register_weight(q.ctypes.data, s.ctypes.data, q.shape[0], q.shape[1])
        for q, _ in views:
            gcu.lib().gcu_unregister_weight(q.ctypes.data)
    per_weight()
    ts = []
    for _ in range(max(1, min(args.steps, 3))):
        views = [binfmt.qtensor_arrays(buf, r) for r in recs]
        t0 = time.perf_counter()
        for q, s in views:
            gcu.lib().gcu_register_weight(q.ctypes.data, s.ctypes.data, q.shape[0], q.shape[1])
        ts.append(time.perf_counter() - t0)
        for q, _ in views:
            gcu.lib().gcu_unregister_weight(q.ctypes.data)
    t_pw = statistics.median(ts)

    # PCIe roofline: one pinned 256 MB host->device copy, CUDA events
    hb = torch.empty(256 << 20, dtype=torch.uint8, pin_memory=True)
    db = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(3):
        db.copy_(hb, non_blocking=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        db.copy_(hb, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    pcie = 5 * hb.numel() / (e0.elapsed_time(e1) * 1e-3) / 1e9
    del hb, db

    ref = None
    if not args.no_cpu:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle
        variant = oracle.ref_variant()
        lib = oracle.ref(variant) if variant else None
        if lib is not None and hasattr(lib, "ref_read_model_seconds"):
            R = oracle.Ref(variant, threads=1)
            R.read_model_seconds(path)
            tr = statistics.median(R.read_model_seconds(path) for _ in range(3))
            ref = {"value": wbytes / tr / 1e9, "unit": "GB/s", "cores": 1, "kind": "reference",
                   "sample": f"gemma.c read_gemma_model of the same {buf.nbytes / 1e9:.2f} GB file (page cache warm), "
                             f"host memory only, median of 3",
                   "seconds": tr}
    os.unlink(path)
    os.rmdir(tmpdir)

    v = wbytes / t_mmap / 1e9
    out = {"metric": "model registration: matmul weights of a -q model image -> HBM (GB/s)",
           "value": v, "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": t_mmap * 1e3, "higher_is_better": True, "scaling": "none", "vs_baseline": None,
           "dtype": "u8 (int8 weights + fp32 scales, byte copy)", "data": "synthetic", "impl": "ours",
           "config": {"workload": f"{args.workload}: {title}, {len(recs)} QTensors, {wbytes / 1e9:.3f} GB of "
                                  f"weights in a {buf.nbytes / 1e9:.3f} GB image",
                      "source": "fresh mmap of the page-cached file per step (value); resident buffer "
                                "(resident_gbs)",
                      "timing": "host clock around the synchronous gcu_register_model, median of steps"},
           "resident_gbs": wbytes / t_res / 1e9,
           "per_weight_gbs": wbytes / t_pw / 1e9,
           "roofline": {"bound": "pcie", "achieved": v, "peak": pcie, "unit": "GB/s", "frac": v / pcie,
                        "peak_src": "pinned 256 MB cudaMemcpy host->device measured in this run",
                        "resident_frac": wbytes / t_res / 1e9 / pcie, "traffic": None},
           "clocks": clk, "gpu_launches": 0,
           "copy_engine": "no kernels: cudaMemcpyAsync of 8 MB packed pinned slots"}
    if ref is not None:
        out["cpu_baseline"] = ref
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------------------
# attention (gcu_dev_attention_decode / _prefill), the fp32 layer around the
# matmuls: Gemma 3's pattern of 5 sliding-window layers then 1 global layer
# ---------------------------------------------------------------------------
ATTN = {
    "attn_decode12b": dict(title="Gemma-3-12B decode attention at position 32767, 48 layers "
                                 "(40 sliding-window 1024, 8 global)", kind="decode", n_heads=16, nkv=8, hd=256,
                           layers=48, pos=32767, slide=1024),
    "attn_prefill1b": dict(title="Gemma-3-1B prefill attention, M=512 tokens from position 0, 26 layers "
                                 "(sliding window 512 / global)", kind="prefill", n_heads=4, nkv=1, hd=256,
                           layers=26, ntok=512, spos=0, slide=512),
}


def _attn_layers(c):
    """Per layer: (global, spos, attlen or ntok, slide).  Layer l is global
    when (l + 1) % 6 == 0 (Gemma 3's 5:1 pattern)."""
    out = []
    for l in range(c["layers"]):
        glob = (l + 1) % 6 == 0
        if c["kind"] == "decode":
            pos = c["pos"]
            spos = 0 if glob or pos < c["slide"] else pos + 1 - c["slide"]
            out.append((glob, spos, pos + 1 - spos, 0 if glob else c["slide"]))
        else:
            out.append((glob, c["spos"], c["ntok"], 0 if glob else c["slide"]))
    return out


def run_attention(args):
    """Decode: one step = every layer's attention of one token at `pos` (K/V
    windows streamed from HBM; roofline: measured HBM copy bandwidth).
    Prefill: one step = every layer's causal attention of an M-token chunk
    (roofline: the fp32 FMA peak derived from the SM count and clock).
    Inputs resident in HBM, each layer its own cache, one CUDA graph replay
    per step, CUDA events on the launching stream."""
    import numpy as np
    import torch

    import gcu
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    gcu.init(0)
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    peaks = load_peaks()
    c = ATTN[args.workload]
    nh, nkv, hd = c["n_heads"], c["nkv"], c["hd"]
    lay = _attn_layers(c)
    if args.layers > 0:  # profiling captures of a small case
        lay = lay[:args.layers]
    gen = torch.Generator(device=dev).manual_seed(5)
    clen = c["pos"] + 1 if c["kind"] == "decode" else c["spos"] + c["ntok"]
    bufs = []
    for glob, spos, n, slide in lay:
        kc = torch.randn((nkv, clen, hd), generator=gen, device=dev)
        vc = torch.randn((nkv, clen, hd), generator=gen, device=dev)
        if c["kind"] == "decode":
            xq = torch.randn((nh, hd), generator=gen, device=dev)
            xo = torch.empty((nh, hd), device=dev)
        else:
            xq = torch.randn((nh, n, hd), generator=gen, device=dev) / hd ** 0.5
            xo = torch.empty((n, nh * hd), device=dev)
        bufs.append((xq, kc, vc, xo))
    asc = 1.0 / hd ** 0.5
    stream = torch.cuda.Stream(dev)

    def step():
        for (glob, spos, n, slide), (xq, kc, vc, xo) in zip(lay, bufs):
            if c["kind"] == "decode":
                gcu.dev_attention_decode(xo, xq, kc, vc, spos, n, asc, stream=stream)
            else:
                gcu.dev_attention_prefill(xo, xq, kc, vc, spos, slide, stream=stream)

    with torch.cuda.stream(stream):
        step()
    stream.synchronize()
    gcu.check_device()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    torch.cuda.synchronize()
    clocks = Clocks(0)
    clocks.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    clk = clocks.stop()
    gcu.check_device()

    if c["kind"] == "decode":
        kv = sum(2 * nkv * n * hd * 4 for _, _, n, _ in lay)
        nbytes = kv + len(lay) * 2 * nh * hd * 4
        value = nbytes / (ms * 1e-3) / 1e9
        splits = [1 if n <= 64 else None for _, _, n, _ in lay]
        roof = {"bound": "hbm", "achieved": value, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": value / peaks["hbm_gbs"], "peak_src": f"{peaks['src']} copy bandwidth",
                "bytes_per_step": nbytes, "traffic": None}
        unit, metric = "GB/s", "decode attention: K/V window bytes streamed from HBM per second"
        launches = sum(1 if s == 1 else 2 for s in splits)
    else:
        flops = 0
        for _, spos, n, slide in lay:
            vis = 0
            for i in range(n):
                pos = spos + i
                t0 = pos + 1 - slide if slide and pos >= slide else 0
                vis += pos - t0 + 1
            flops += 4 * nh * hd * vis  # q.k and p.v, 2 flops per multiply-add
        value = flops / (ms * 1e-3) / 1e12
        mhz = clk.get("sm_max_mhz") or 1965.0
        peak = 148 * 128 * 2 * mhz * 1e6 / 1e12
        roof = {"bound": "fp32", "achieved": value, "peak": peak, "unit": "TFLOP/s", "frac": value / peak,
                "peak_src": "derived fp32 FMA peak: 148 SMs x 128 lanes x 2 flops x max SM clock",
                "flops_per_step": flops, "note": "a chunk of one 64-key tile keeps its scores between the max and "
                "weight passes; a longer chunk scores its keys twice (up to 1.5x the counted flops)",
                "traffic": None}
        unit, metric = "TFLOP/s", "prefill attention: causal fp32 flops per second"
        launches = len(lay)
    out = {"metric": metric, "value": value, "unit": unit, "n_gpus": 1, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "none",
           "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "ours",
           "config": {"workload": f"{args.workload}: {c['title']}", "heads": nh, "kv_heads": nkv, "head_dim": hd,
                      "inputs": "each layer its own K/V cache in HBM (no L2 reuse across layers)",
                      **({"reduced": f"--layers {args.layers}: a profiling case, not the benchmark workload"}
                         if args.layers > 0 else {})},
           "roofline": roof, "clocks": clk, "gpu_launches": launches * args.steps,
           "e2e": None, "e2e_note": "attention has no host-pointer entry point: it runs between device-resident "
                                  "matmuls"}
    if not args.no_cpu:
        out["cpu_baseline"] = _attn_cpu_baseline(c, lay)
    del graph
    print(json.dumps(out), flush=True)


def _attn_cpu_baseline(c, lay):
    """gemma.c's own attention (oracle/_ref build, all host threads) on one
    period of the layer pattern (5 sliding + 1 global), scaled to the step."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    variant = oracle.ref_variant()
    lib = oracle.ref(variant) if variant else None
    threads = os.cpu_count() or 1
    if lib is None or not hasattr(lib, "ref_attention_decode"):
        return {"value": None, "cores": threads, "kind": "reference", "sample": "reference build not available"}
    R = oracle.Ref(variant, threads=threads)
    nh, nkv, hd = c["n_heads"], c["nkv"], c["hd"]
    rng = np.random.default_rng(0)
    period = lay[:6]
    clen = max(spos + n for _, spos, n, _ in period)
    kc = rng.standard_normal((nkv, clen, hd), dtype=np.float32)
    vc = rng.standard_normal((nkv, clen, hd), dtype=np.float32)
    t = 0.0
    for _, spos, n, slide in period:
        if c["kind"] == "decode":
            xq = rng.standard_normal((nh, hd), dtype=np.float32)
            R.attention_decode(xq, kc, vc, spos, n, np.float32(1 / hd ** 0.5))
            t0 = time.perf_counter()
            R.attention_decode(xq, kc, vc, spos, n, np.float32(1 / hd ** 0.5))
        else:
            xq = rng.standard_normal((nh, n, hd), dtype=np.float32) / np.float32(hd ** 0.5)
            R.attention_prefill(xq, kc, vc, spos, slide)
            t0 = time.perf_counter()
            R.attention_prefill(xq, kc, vc, spos, slide)
        t += time.perf_counter() - t0
    scale = len(lay) / len(period)
    step_s = t * scale
    return {"ms_per_step": step_s * 1e3, "cores": threads, "kind": "reference",
            "sample": f"one period of the layer pattern (6 layers, gemma.c's attention, {variant}/{R.isa}), "
                      f"scaled x{scale:.1f} to the step",
            "speedup_note": "GPU step time vs this CPU step time"}


# ---------------------------------------------------------------------------
# device-resident decode step (decode.Decoder): every layer of a Gemma 3
# text decoder plus the lm_head for one token, activations and KV cache in HBM
# ---------------------------------------------------------------------------
DECODE_STEP = {
    "decode_step1b": dict(title="Gemma-3-1B decode step at position 1023 (26 layers + lm_head)", nl=26, n_heads=4,
                          nkv=1, hdim=256, dim=1152, mlp_dim=6912, nvocab=262144, q_scale=256, slide=512, pos=1023),
    "decode_step4b": dict(title="Gemma-3-4B decode step at position 1023 (34 layers + lm_head)", nl=34, n_heads=8,
                          nkv=4, hdim=256, dim=2560, mlp_dim=10240, nvocab=262144, q_scale=256, slide=1024, pos=1023),
    "prefill_chunk1b": dict(title="Gemma-3-1B prefill of a 512-token chunk from position 0 (26 layers + last-token "
                                  "lm_head)", nl=26, n_heads=4, nkv=1, hdim=256, dim=1152, mlp_dim=6912,
                            nvocab=262144, q_scale=256, slide=512, pos=0, ntok=512),
}


def run_decode_step(args):
    """One step = decode.Decoder.step: per layer RMSNorm+quantize, Q/K/V
    multi-GEMV, QK norm/RoPE/cache write, attention over the window, fused
    quantize+O GEMV, post-norm residual, pre-FFN norm+quantize, gate/up
    multi-GEMV, GeGLU+quantize, down GEMV, post-norm residual; then the final
    norm and the 262144-row lm_head.  Weights and a KV cache of `pos`
    positions resident in HBM, one CUDA graph replay per step, CUDA events.
    Roofline: HBM bytes the step must read (all weights + the K/V windows)
    over the measured copy bandwidth."""
    import numpy as np
    import torch

    import decode
    import gcu
    import synth
    if int(os.environ.get("RANK", "0")) != 0:
        return
    gcu.init(0)
    torch.cuda.set_device(0)
    peaks = load_peaks()
    spec = DECODE_STEP[args.workload]
    nl = spec["nl"] if args.layers <= 0 else min(spec["nl"], args.layers)
    cfg = dict(spec, nl=nl, swa=[(l + 1) % 6 != 0 for l in range(nl)], qk_norm=True, mlp_pre=True, mlp_pst=True,
               theta_l=10000.0, theta_g=1000000.0, eps=1e-6, sc_att=0.0, sc_log=0.0)
    pos = cfg["pos"]
    dim, mlp, hd = cfg["dim"], cfg["mlp_dim"], cfg["hdim"]
    q_sz, kv_sz = cfg["n_heads"] * hd, cfg["nkv"] * hd
    gen = torch.Generator(device="cuda").manual_seed(11)
    wt = lambda n, k: synth.weight_torch(n, k, gen, "cuda")
    nv = lambda n: torch.randn(n, generator=gen, device="cuda") * 0.1
    layers = [{"wq": wt(q_sz, dim), "wk": wt(kv_sz, dim), "wv": wt(kv_sz, dim), "wo": wt(dim, q_sz),
               "w1": wt(mlp, dim), "w2": wt(mlp, dim), "w3": wt(dim, mlp), "n1": nv(dim), "n2": nv(dim),
               "n3": nv(dim), "n4": nv(dim), "nq": nv(hd), "nk": nv(hd)} for _ in range(nl)]
    emb = wt(cfg["nvocab"], dim)
    fnorm = nv(dim)
    ntok = cfg.get("ntok", 0)
    prefill = ntok > 0
    dec = decode.Decoder(cfg, layers, emb, fnorm, clen=pos + max(ntok, 1))
    stream = torch.cuda.Stream()
    if prefill:
        tabs = [decode.rope_tables(hd, cfg["theta_l"], cfg["theta_g"], pos + t) for t in range(ntok)]
        dec.set_prefill_freqs(np.stack([t[0] for t in tabs]), np.stack([t[1] for t in tabs]))
        dec.px[:ntok].normal_(generator=gen)
        run = lambda: dec.prefill(pos, ntok, stream=stream)
    else:
        dec.kv.normal_(generator=gen)  # positions 0 .. pos-1 as if decoded before
        slid, full = decode.rope_tables(hd, cfg["theta_l"], cfg["theta_g"], pos)
        dec.set_freqs(slid, full)
        dec.x.normal_(generator=gen)
        run = lambda: dec.step(pos, stream=stream)
    with torch.cuda.stream(stream):
        run()  # eager: allocates the split scratch
    stream.synchronize()
    gcu.check_device()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        run()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            g.replay()
    torch.cuda.synchronize()
    clocks = Clocks(0)
    clocks.start()
    time.sleep(0.2)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    clk = clocks.stop()
    gcu.check_device()
    wbytes = sum(t[0].numel() + 4 * t[1].numel() for lay in dec.L for k, t in lay.items()
                 if isinstance(t, tuple)) + emb[0].numel() + 4 * emb[1].numel()
    kvbytes = 0
    for l in range(nl):
        n = min(pos + 1, cfg["slide"]) if cfg["swa"][l] else pos + 1
        kvbytes += 2 * kv_sz * n * 4
    nbytes = wbytes + kvbytes
    ach = nbytes / (ms * 1e-3) / 1e9
    if prefill:
        ops = ntok * sum(2 * t[0].numel() for lay in dec.L for t in lay.values() if isinstance(t, tuple))
        ach_t = ops / (ms * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": ach_t, "peak": 2.0 * peaks["bf16_tflops"], "unit": "TOPS",
                "frac": ach_t / (2.0 * peaks["bf16_tflops"]), "peak_src": f"2 x {peaks['src']} bf16 dense",
                "int8_ops_per_step": ops, "note": "layer matmuls only; attention and norms are fp32", "traffic": None}
    else:
        roof = {"bound": "hbm", "achieved": ach, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": ach / peaks["hbm_gbs"], "peak_src": f"{peaks['src']} copy bandwidth",
                "bytes_per_step": nbytes, "weight_bytes": wbytes, "kv_bytes": kvbytes, "traffic": None}
    out = {"metric": ("device-resident prefill: tokens per second (all layers, last-token lm_head)" if prefill else
                      "device-resident decode: tokens per second (all layers + lm_head, batch 1)"),
           "value": (ntok if prefill else 1) * 1e3 / ms, "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
           "warmup": args.warmup,
           "ms_per_step": ms, "higher_is_better": True, "scaling": "none", "vs_baseline": None,
           "dtype": "int8 matmuls (int32 accum), fp32 norms/attention", "data": "synthetic", "impl": "ours",
           "config": {"workload": f"{args.workload}: {cfg['title']}", "layers": nl, "kv_cache_positions": pos + 1,
                      "layer_pattern": "5 sliding-window layers then 1 global",
                      **({"reduced": f"--layers {args.layers}: a profiling case, not the benchmark workload"}
                         if args.layers > 0 else {})},
           "roofline": roof,
           "clocks": clk, "gpu_launches": dec.launches_per_step(prefill) * args.steps, "e2e": None,
           "e2e_note": "device-resident by design: the step reads no host memory"}
    if not args.no_cpu and args.layers <= 0 and args.workload in ("decode_step1b", "prefill_chunk1b"):
        out["cpu_baseline"] = _decode_cpu_baseline(cfg, dec, emb, fnorm)
    del g
    print(json.dumps(out), flush=True)


def _decode_cpu_baseline(cfg, dec, emb, fnorm):
    """gemma.c's forward_text_decode on the same weights (copied to the host),
    positions 0..15, all host threads: seconds per token."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    variant = oracle.ref_variant()
    lib = oracle.ref(variant) if variant else None
    threads = os.cpu_count() or 1
    if lib is None or not hasattr(lib, "ref_decode_steps"):
        return {"value": None, "cores": threads, "kind": "reference", "sample": "reference build not available"}
    R = oracle.Ref(variant, threads=threads)
    host = lambda t: t.cpu().numpy()
    layers = []
    for w in dec.L:
        lay = {k: (host(w[k][0]), host(w[k][1])) for k in ("wq", "wk", "wv", "wo", "w1", "w2", "w3")}
        lay.update({k: host(w[k]) for k in ("n1", "n2", "n3", "n4", "nq", "nk")})
        layers.append(lay)
    e = (host(emb[0]), host(emb[1]))
    ntok = cfg.get("ntok", 0)
    if ntok:
        x0 = np.random.default_rng(0).standard_normal((ntok, cfg["dim"]), dtype=np.float32)
        R.prefill_chunks(cfg, layers, e, host(fnorm), x0[:16], [16])  # warm-up (pages the weights in)
        t0 = time.perf_counter()
        R.prefill_chunks(cfg, layers, e, host(fnorm), x0, [ntok])
        dt = time.perf_counter() - t0
        return {"value": ntok / dt, "unit": "tokens/s", "cores": threads, "kind": "reference",
                "ms_per_step": dt * 1e3,
                "sample": f"gemma.c forward_text_chunk of the same {ntok} tokens on the same weights, "
                          f"{variant}/{R.isa}"}
    x0 = np.random.default_rng(0).standard_normal((16, cfg["dim"]), dtype=np.float32)
    R.decode_steps(cfg, layers, e, host(fnorm), x0[:2])  # warm-up (pages the weights in)
    t0 = time.perf_counter()
    R.decode_steps(cfg, layers, e, host(fnorm), x0)
    dt = (time.perf_counter() - t0) / len(x0)
    return {"value": 1.0 / dt, "unit": "tokens/s", "cores": threads, "kind": "reference", "ms_per_step": dt * 1e3,
            "sample": f"gemma.c forward_text_decode on the same weights, positions 0..15, {variant}/{R.isa}"}


# ---------------------------------------------------------------------------
# SigLIP head (gcu_dev_patch_embed, gcu_dev_vision_pool_quantize, then the
# projection gcu_dev_gemm_int8): one 896 px image of Gemma-3-4B
# ---------------------------------------------------------------------------
def run_siglip_head(args):
    """One step = patch embedding of an (896, 896, 3) image (4096 patches of
    14 px -> 1152, the int8 position embedding added), LayerNorm -> 4x4
    average pool -> RMSNorm -> quantize (256 tokens), and the int8 projection
    to the 4B text width 2560.  Inputs resident in HBM, one CUDA graph replay
    per step, CUDA events; roofline of the dominant kernel (patch embedding,
    fp32 FMA-bound) against the fp32 FMA peak derived from SMs and clock."""
    import numpy as np
    import torch

    import gcu
    import synth
    if int(os.environ.get("RANK", "0")) != 0:
        return
    gcu.init(0)
    torch.cuda.set_device(0)
    v = synth.vision_head_inputs(700, 896, 14, 1152, 256, 2560)
    ppi, side, dim, tdim = 64, 16, 1152, 2560
    d = {k: torch.from_numpy(np.ascontiguousarray(v[k])).cuda() for k in
         ("img", "pe", "pe_b", "pos_q", "pos_s", "post_n", "post_nb", "norm", "proj_q", "proj_s")}
    x = torch.empty((ppi * ppi, dim), device="cuda")
    q = torch.empty((side * side, dim), dtype=torch.int8, device="cuda")
    sc = torch.empty(side * side, device="cuda")
    y = torch.empty((side * side, tdim), device="cuda")
    stream = torch.cuda.Stream()

    def step(which=("pe", "pool", "proj")):
        if "pe" in which:
            gcu.dev_patch_embed(x, d["img"], d["pe"], d["pe_b"], d["pos_q"], d["pos_s"], 896, 14, dim, stream=stream)
        if "pool" in which:
            gcu.dev_vision_pool_quantize(q, sc, x, d["post_n"], d["post_nb"], d["norm"], v["eps"], ppi, side, dim,
                                         stream=stream)
        if "proj" in which:
            gcu.dev_gemm_int8(y, d["proj_q"], d["proj_s"], q, sc, side * side, tdim, dim, stream=stream)

    def timed(which):
        with torch.cuda.stream(stream):
            step(which)
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step(which)
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.steps):
                g.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        del g
        return e0.elapsed_time(e1) / args.steps

    clocks = Clocks(0)
    clocks.start()
    ms = timed(("pe", "pool", "proj"))
    parts = {k: timed((k,)) for k in ("pe", "pool", "proj")}
    clk = clocks.stop()
    gcu.check_device()
    pe_flops = 2 * ppi * ppi * dim * 3 * 14 * 14
    mhz = clk.get("sm_max_mhz") or 1965.0
    peak = 148 * 128 * 2 * mhz * 1e6 / 1e12
    ach = pe_flops / (parts["pe"] * 1e-3) / 1e12
    out = {"metric": "SigLIP head: images per second (patch embedding, pool, int8 projection)",
           "value": 1e3 / ms, "unit": "images/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": ms, "higher_is_better": True, "scaling": "none", "vs_baseline": None,
           "dtype": "f32 (patch embedding, norms), int8 (projection)", "data": "synthetic", "impl": "ours",
           "config": {"workload": "siglip_head: Gemma-3-4B vision head, 896 px image, 4096 patches -> 256 tokens -> "
                                  "2560", "inputs": "seeded image and weights resident in HBM"},
           "stage_ms": parts,
           "roofline": {"bound": "fp32", "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
                        "kernel": "k_patch_embed", "flops_per_launch": pe_flops,
                        "peak_src": "derived fp32 FMA peak: 148 SMs x 128 lanes x 2 flops x max SM clock",
                        "traffic": None},
           "clocks": clk, "gpu_launches": 3 * args.steps, "e2e": None,
           "e2e_note": "no host-pointer entry point: the head runs between device-resident tower layers"}
    if not args.no_cpu:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle
        variant = oracle.ref_variant()
        lib = oracle.ref(variant) if variant else None
        if lib is not None and hasattr(lib, "ref_vision_head"):
            R = oracle.Ref(variant, threads=os.cpu_count() or 1)
            R.vision_head(v)
            t0 = time.perf_counter()
            R.vision_head(v)
            t = time.perf_counter() - t0
            out["cpu_baseline"] = {"value": 1.0 / t, "unit": "images/s", "cores": R.threads, "kind": "reference",
                                   "sample": f"gemma.c forward_vision on an encoder with no layers (the same head), "
                                             f"{variant}/{R.isa}", "ms_per_step": t * 1e3}
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------------------
# reference arm: the reference's own CPU implementation of the path
# ---------------------------------------------------------------------------
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    variant = oracle.ref_variant()
    if variant is None:
        print(json.dumps({"impl": "reference", "unavailable": "no runnable build of gemma.c's matmul functions "
                          "for this host CPU in oracle/_ref"}))
        return
    threads = os.cpu_count() or 1
    R = oracle.Ref(variant, threads=threads)
    wl = Prefill()
    ops, run = wl.cpu_sample(R, 1)
    for _ in range(args.warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run()
    dt = (time.perf_counter() - t0) / args.steps
    v = ops / dt / 1e12
    out = {"metric": METRIC, "value": v, "unit": "int8 TOPS", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "int8 (int32 accum, fp32 out)", "data": "synthetic", "impl": "reference",
           "config": dict(wl.config(), parallelism=("single GPU" if world == 1 else f"replicas x{world}")),
           "reference_calls": "per layer gemma.c quantize_acts x4; Q/K/V as per-(head, 128-token) gemm_int8 "
                              "tasks (gemma.c:5037-5091); O, up, gate, down one gemm_int8 each (omp)",
           "cpu_baseline": {"value": v, "unit": "int8 TOPS", "cores": threads, "kind": "reference",
                            "sample": f"1 layer (M=512) of gemma.c quantize_acts+gemm_int8 per step, "
                                      f"{oracle.ref_build_desc(variant)}; {R.isa} kernels"},
           "e2e": {"value": v, "unit": "int8 TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="prefill1b",
                    choices=list(PREFILL) + list(DECODE) + ["lmhead4b"] + list(UPLOAD) + list(ATTN) +
                    ["siglip_head"] + list(DECODE_STEP))
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--chain", action="store_true",
                    help="prefill workloads: the step's quantize_acts -> GEMM pairs as chain launches "
                         "(gcu_gemm_chain_*, at most 22 pairs per launch)")
    ap.add_argument("--unfused", action="store_true",
                    help="decode: quantize and GEMV as separate launches (the reference's call split)")
    ap.add_argument("--fused", action="store_true",
                    help="prefill: issue each quantize+GEMM pair through gcu_dev_quantize_gemm_int8_multi")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-decode", action="store_true",
                    help="default workload: skip the decode-GEMV sub-records")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--layers", type=int, default=0,
                    help="cut every stack to this many layers (small cases for ncu captures; the line "
                         "then describes a reduced workload and is not a benchmark value)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload in DECODE_STEP:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the decode-step line carries the reference's "
                              "forward_text_decode timing as its cpu_baseline"}))
        else:
            run_decode_step(args)
    elif args.workload == "siglip_head":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the SigLIP-head line carries the reference's "
                              "forward_vision timing as its cpu_baseline"}))
        else:
            run_siglip_head(args)
    elif args.workload in ATTN:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the attention lines carry the reference's "
                              "attention timing as their cpu_baseline"}))
        else:
            run_attention(args)
    elif args.workload in UPLOAD:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the model-upload line carries the reference's "
                              "read_gemma_model timing as its cpu_baseline"}))
        else:
            run_upload(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
