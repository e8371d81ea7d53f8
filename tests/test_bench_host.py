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
