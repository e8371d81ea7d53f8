"""Synthetic `-q` models and token streams for the drop-in tests: gemma.c's
own model path (setup_gemma_model -> forward_gemma_image / _prefill /
_decode -> cleanup_gemma_model) run by the reference build and by the build
whose hot path is the CUDA drop-in (oracle/_ref/libgemma_dropin.so)."""
import ctypes
import os

import numpy as np

import binfmt

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref")

# small Gemma-3-style decoders: GQA, QK norm, pre/post FFN norms, sliding
# layers; the second one carries a SigLIP tower so the vision projections
# (gemma.c:4497-4717) run too
CASES = {
    "text": dict(text=dict(nl=3, n_heads=4, nkv=2, hdim=64, dim=256, mlp_dim=768, nvocab=2048, qk_norm=True,
                           mlp_pre=True, mlp_pst=True, slide=96, swa=[True, False, True]),
                 vision=None, prompt=300, chunk=128, decode=4, seed=11),
    "vision": dict(text=dict(nl=2, n_heads=2, nkv=1, hdim=128, dim=256, mlp_dim=512, nvocab=1024, qk_norm=True,
                             mlp_pre=True, mlp_pst=True, slide=64, img_tok=4, swa=[True, False]),
                   vision=dict(nl=2, n_heads=4, mlp_dim=384, dim=128, img_px=56, psize=14),
                   prompt=40, chunk=64, decode=3, seed=12),
}


def write_model(tmpdir, name):
    c = CASES[name]
    buf, _ = binfmt.image(c["text"], c["vision"], seed=c["seed"])
    path = os.path.join(str(tmpdir), f"dropin_{name}.bin")
    buf.tofile(path)
    return path


def tokens(name):
    c = CASES[name]
    rng = np.random.default_rng(c["seed"])
    return rng.integers(0, c["text"]["nvocab"], size=c["prompt"] + c["decode"]).astype(np.int32)


def image(name):
    c = CASES[name]
    if c["vision"] is None:
        return None
    px = c["vision"]["img_px"]
    rng = np.random.default_rng(c["seed"] + 1)
    return (rng.random((px, px, 3), dtype=np.float32) * 2 - 1).astype(np.float32)


def load(which):
    """'native' (the reference's own code) or 'dropin' (its hot path on the GPU)."""
    name = {"native": "libgemma_ref_native.so", "dropin": "libgemma_dropin.so"}[which]
    path = os.path.join(REF, name)
    if not os.path.exists(path):
        return None
    lib = ctypes.CDLL(path)
    lib.ref_dropin.restype = ctypes.c_int
    lib.ref_setup.restype = None
    lib.ref_setup()
    f32p = ctypes.POINTER(ctypes.c_float)
    lib.ref_model_run.restype = ctypes.c_int
    lib.ref_model_run.argtypes = [ctypes.c_char_p] + [ctypes.c_int] * 4 + [f32p, ctypes.POINTER(ctypes.c_int)] + \
        [ctypes.c_int] * 2 + [f32p] + [ctypes.c_int] * 2
    lib.ref_model_registered_bytes.restype = ctypes.c_longlong
    lib.ref_model_registered_bytes.argtypes = [ctypes.c_char_p] + [ctypes.c_int] * 4
    return lib


def run(lib, path, name, mmap_on, threads=8):
    """(1 + decode) x nvocab logits of the prompt and each decode step."""
    c = CASES[name]
    nv = c["text"]["nvocab"]
    tok = tokens(name)
    img = image(name)
    out = np.zeros((1 + c["decode"], nv), np.float32)
    f32p = ctypes.POINTER(ctypes.c_float)
    rc = lib.ref_model_run(path.encode(), int(mmap_on), 1, 1024, c["chunk"],
                           img.ctypes.data_as(f32p) if img is not None else None,
                           tok.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), c["prompt"], c["decode"],
                           out.ctypes.data_as(f32p), nv, threads)
    if rc:
        raise RuntimeError(f"gemma.c's model path failed ({name}, mmap={mmap_on})")
    return out
