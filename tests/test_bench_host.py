"""Host logic of bench.py's extra workloads (no GPU): Gemma 3's layer
pattern for the attention lines and the flop count their roofline uses."""
import bench


def test_decode_layer_pattern():
    lay = bench._attn_layers(bench.ATTN["attn_decode12b"])
    assert len(lay) == 48
    glob = [i for i, (g, _, _, _) in enumerate(lay) if g]
    assert glob == [5, 11, 17, 23, 29, 35, 41, 47]  # every sixth layer is global
    for g, spos, n, slide in lay:
        if g:
            assert (spos, n, slide) == (0, 32768, 0)
        else:  # sliding window of 1024 ending at position 32767
            assert (spos, n, slide) == (32767 + 1 - 1024, 1024, 1024)


def test_prefill_flop_count():
    c = dict(bench.ATTN["attn_prefill1b"], layers=2, ntok=40, spos=30, slide=16)
    for _, spos, n, slide in bench._attn_layers(c):
        vis = 0
        for i in range(n):
            pos = spos + i
            t0 = pos + 1 - slide if slide and pos >= slide else 0
            vis += pos - t0 + 1
        brute = sum(min(spos + i + 1, slide if slide else 10 ** 9) for i in range(n))
        assert vis == brute


def test_reference_arm_prints_the_contract_line():
    # the reference arm runs gemma.c's own functions on host cores: no GPU
    import json
    import os
    import subprocess
    import sys

    import oracle as O
    if O.ref() is None:
        import pytest
        pytest.skip("reference build not available")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, os.path.join(root, "bench.py"), "--impl", "reference", "--steps", "3",
                          "--warmup", "3"], capture_output=True, text=True, timeout=300, cwd=root)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["steps"] == 3 and line["value"] > 0
    assert line["e2e"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["cpu_baseline"]["kind"] in ("reference", "port") and line["cpu_baseline"]["cores"] >= 1
    assert line["config"]["workload"].startswith("prefill1b")
