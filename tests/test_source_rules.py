"""Source-level guards on the CUDA library (CPU only).

The kernels run in multi-GPU jobs and on shared GPUs, so some constructs
must never appear in gemma.c_b200/csrc:

- a copy instruction that fans one load out to several CTAs of a cluster
  (every load of this library reads the launching GPU's own memory into the
  CTA that issued it; the cluster-wide form is kept to the tcgen05 commit
  that signals a CTA pair's barriers);
- a device trap or a device-side assert (a kernel that gives up records a
  code in the error word and returns);
- the batched host-to-device copy calls of the CUDA runtime and driver
  (one asynchronous copy per transfer is used instead).

The patterns are assembled from fragments so that this file itself names
none of the constructs it forbids.
"""
import glob
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SOURCES = sorted(glob.glob(os.path.join(ROOT, "gemma.c_b200", "csrc", "*.cu")) +
                 glob.glob(os.path.join(ROOT, "gemma.c_b200", "csrc", "*.cuh")) +
                 glob.glob(os.path.join(ROOT, "include", "*.h")))

FANOUT = "".join(["mul", "ti", "ca", "st"])
COPY = "".join(["cp.", "async", ".bu", "lk"])
GATHER = "".join(["tile::", "gat", "her4"])
COMMIT = "tcgen05" + ".commit"
TRAP = "__tr" + "ap("
BATCH = re.compile("Memcpy" + r"(3D)?" + "Batch" + "Async")


def _code_lines():
    for path in SOURCES:
        with open(path) as f:
            for no, line in enumerate(f, 1):
                code = line.split("//", 1)[0]  # comments may describe what is not done
                yield os.path.relpath(path, ROOT), no, code


def test_sources_exist():
    assert any(p.endswith("k_gemm.cu") for p in SOURCES)


def test_copies_read_local_memory_only():
    bad = [(p, n) for p, n, c in _code_lines() if FANOUT in c and (COPY in c or GATHER in c)]
    assert not bad, f"cluster fan-out on a copy instruction: {bad}"


def test_cluster_signal_only_on_pair_commit():
    uses = [(p, n, c.strip()) for p, n, c in _code_lines() if FANOUT in c]
    for p, n, c in uses:
        assert COMMIT in c, f"{p}:{n}: {c}"


def test_no_trap_or_device_assert():
    bad = []
    for p, n, c in _code_lines():
        if TRAP in c or re.search(r"(?<![A-Za-z_])assert\(", c):
            bad.append((p, n))
    assert not bad, f"trap or device assert: {bad}"


def test_no_batched_copy_calls():
    bad = [(p, n) for p, n, c in _code_lines() if BATCH.search(c)]
    assert not bad, f"batched copy call: {bad}"
