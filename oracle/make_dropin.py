#!/usr/bin/env python3
"""Write gemma.c with the CUDA drop-in applied (test infrastructure).

    python oracle/make_dropin.py <reference gemma.c> <out.c>

The output is the reference's own gemma.c with the patch INTEGRATION.md
describes, applied mechanically so that a test can build the reference's
forward passes on top of libgcu.so:

* gemma.c's five hot-path definitions -- quantize_act / quantize_acts
  (gemma.c:2586-2674), gemv_int8_row / gemv_int8 (2754-2788), gemv_int8_multi
  (2812-2837) and gemm_int8 (3937-4054) -- are wrapped in
  ``#ifndef GEMMA_CUDA``, and the drop-in header gemma_gcu.h takes their place
  after GemvJob (2795-2800), which it needs;
* the model hooks (gemma_gcu_model.h) are included after GemmaModel
  (1882-1890); setup_gemma_model (6867) registers the model's matmul weights
  once it is read or mapped, and cleanup_gemma_model (6909) releases them.

Every anchor line is checked against the text the patch expects, so a
different gemma.c is refused instead of patched wrongly.  The output is a
build product (oracle/_ref, git-ignored); it is never committed.
"""
import sys

# (first line, last line) of each wrapped block, 1-based inclusive, with the
# text each block's key line must hold
BLOCKS = [
    (2586, 2674, 2590, "static floatx quantize_act(int8_t *dst, const floatx *vec, int dim,"),
    (2754, 2788, 2770, "static void gemv_int8(floatx *RESTRICT dst, const int8_t *RESTRICT mat,"),
    (2812, 2837, 2818, "static void gemv_int8_multi(const GemvJob *jobs, int njobs,"),
    (3937, 4054, 3943, "static int gemm_int8(floatx *RESTRICT dst, int dstr, const int8_t *RESTRICT mat,"),
]
DROPIN_AFTER = 2837          # gemma_gcu.h goes where gemv_int8_multi was
GEMVJOB_LINE = (2800, "} GemvJob;")
MODEL_TYPE_END = (1890, "} GemmaModel;")
SETUP = (6867, "int setup_gemma_model(")
SETUP_LOADED = "  if (*model == NULL)"
CLEANUP = (6909, "void cleanup_gemma_model(GemmaModel *model, TextBuffer *tb, VisionBuffer *vb,")


def expect(lines, no, text):
    got = lines[no - 1].rstrip("\n")
    if got.strip() != text.strip():
        raise SystemExit(f"gemma.c:{no}: expected {text!r}, found {got!r}; not the gemma.c this patch is for")


def patch(src: str) -> str:
    lines = src.splitlines(keepends=True)
    for first, last, key, text in BLOCKS:
        expect(lines, key, text)
        if lines[last - 1].rstrip() != "}":
            raise SystemExit(f"gemma.c:{last}: expected the closing brace of the block starting at {first}")
    expect(lines, *GEMVJOB_LINE)
    expect(lines, *MODEL_TYPE_END)
    expect(lines, *SETUP)
    expect(lines, *CLEANUP)
    starts = {b[0]: b for b in BLOCKS}
    ends = {b[1] for b in BLOCKS}
    out = []
    in_setup = False
    for no, line in enumerate(lines, 1):
        if no in starts:
            out.append("#ifndef GEMMA_CUDA /* CUDA drop-in: gemma_gcu.h defines this instead */\n")
        out.append(line)
        if no in ends:
            out.append("#endif /* GEMMA_CUDA */\n")
        if no == DROPIN_AFTER:
            out.append("#if defined(GEMMA_CUDA)\n#include \"gemma_gcu.h\"\n#endif\n")
        if no == MODEL_TYPE_END[0]:
            out.append("#if defined(GEMMA_CUDA)\n#include \"gemma_gcu_model.h\"\n#endif\n")
        if no == SETUP[0]:
            in_setup = True
        if in_setup and line.rstrip("\n") == SETUP_LOADED:
            nxt = lines[no].strip()
            if nxt != "return 1;":
                raise SystemExit(f"gemma.c:{no + 1}: expected 'return 1;' after the load check")
        if in_setup and no > SETUP[0] and lines[no - 2].rstrip("\n") == SETUP_LOADED:
            # the line just written is the load check's `return 1;`
            out.append("#if defined(GEMMA_CUDA)\n"
                       "  if (gcu_setup_gemma_model(*model, allow_mm))\n"
                       "    return 1;\n"
                       "#endif\n")
            in_setup = False
        if no == CLEANUP[0] + 1:  # the signature's second line
            out.append("#if defined(GEMMA_CUDA)\n  gcu_release_gemma_model();\n#endif\n")
    if in_setup:
        raise SystemExit("setup_gemma_model: load check not found")
    return "".join(out)


def main():
    if len(sys.argv) != 3:
        raise SystemExit(__doc__)
    with open(sys.argv[1]) as f:
        src = f.read()
    out = patch(src)
    with open(sys.argv[2], "w") as f:
        f.write(out)


if __name__ == "__main__":
    main()
