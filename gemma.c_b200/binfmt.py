"""binfmt.py -- gemma.c's W8A8 model file layout, written from a config.

Synthetic model images for the loader's tests and benchmark (no real `.bin`
can be downloaded here).  The layout is the one export.py writes
(export.py:255-560) and gemma.c reads (check_head gemma.c:1915-1940,
read_text_config 770-865, read_vision_config 723-738, read_tokenizer
905-990, mmap_text_decoder 1470-1560, mmap_vision_encoder 1765-1875):

    "GEMA" "f32" 'Q'
    text config   >BBB HHHHHH II fffff   nl n_heads nkv | hdim dim mlp_dim
                                         q_scale slide img_tok | max_seq
                                         nvocab | theta_l theta_g eps
                                         sc_att sc_log
    u8 n, n bytes                        sliding-window layers, MSB first
    u8 flags                             8 multimodal, 4 qk_norm,
                                         2 mlp_pre, 1 mlp_post
    [vision config >BB HHHH f]           nl n_heads | mlp_dim dim img_px
                                         psize | eps
    nvocab (+1 if multimodal) pascal strings, >I nmerge, 2*nmerge strings
    tensors, little-endian, back to back; a QTensor is int8 [rows][k]
    followed by f32 [rows]

`layout()` lists every tensor with its offset; `image()` fills a uint8 buffer
(values seeded per tensor, or a cheap repeating pattern for large images).
"""
from __future__ import annotations

import struct

import numpy as np

QT_KINDS = ("lm_head", "wq", "wk", "wv", "wo", "w1", "w2", "w3",
            "vwq", "vwk", "vwv", "vwo", "vw1", "vw2", "vproj")

# text / vision configs of the BASELINE models (dims as gemma.c reads them)
TEXT_1B = dict(nl=26, n_heads=4, nkv=1, hdim=256, dim=1152, mlp_dim=6912, nvocab=262144,
               qk_norm=True, mlp_pre=True, mlp_pst=True)
TEXT_4B = dict(nl=34, n_heads=8, nkv=4, hdim=256, dim=2560, mlp_dim=10240, nvocab=262144,
               qk_norm=True, mlp_pre=True, mlp_pst=True)
VISION_SIGLIP = dict(nl=27, n_heads=16, mlp_dim=4304, dim=1152, img_px=896, psize=14)


def _header(text: dict, vision: dict | None, vocab: list[bytes], merges: list[tuple[bytes, bytes]]) -> bytes:
    nl = text["nl"]
    out = bytearray(b"GEMAf32Q")
    out += struct.pack(">BBB HHHHHH II fffff", nl, text["n_heads"], text["nkv"], text["hdim"], text["dim"],
                       text["mlp_dim"], text.get("q_scale", text["hdim"]), text.get("slide", 512),
                       text.get("img_tok", 256 if vision else 0), text.get("max_seq", 32768), text["nvocab"],
                       10000.0, 1000000.0, 1e-6, 0.0, 0.0)
    swa = text.get("swa", [(i % 6) != 5 for i in range(nl)])
    bits = bytearray((nl + 7) // 8)
    for i, on in enumerate(swa):
        if on:
            bits[i // 8] |= 1 << (7 - i % 8)
    out += bytes([len(bits)]) + bits
    out += bytes([(8 if vision else 0) | (4 if text.get("qk_norm") else 0) | (2 if text.get("mlp_pre") else 0)
                  | (1 if text.get("mlp_pst") else 0)])
    if vision:
        out += struct.pack(">BB HHHH f", vision["nl"], vision["n_heads"], vision["mlp_dim"], vision["dim"],
                           vision["img_px"], vision["psize"], 1e-6)
    assert len(vocab) == text["nvocab"] + (1 if vision else 0)
    for s in vocab:
        out += bytes([len(s)]) + s
    out += struct.pack(">I", len(merges))
    for a, b in merges:
        out += bytes([len(a)]) + a + bytes([len(b)]) + b
    return bytes(out)


def default_tokenizer(nvocab: int, multimodal: bool, seed: int = 0):
    """Distinct token strings of varying length (so tensors start at odd
    offsets), the special tokens gemma.c looks up, and a few merges."""
    rng = np.random.default_rng(seed)
    special = [b"<pad>", b"<eos>", b"<bos>", b"<unk>", b"<start_of_turn>", b"<end_of_turn>",
               b"<start_of_image>", b"<end_of_image>"]
    vocab = special[:min(len(special), nvocab)]
    lens = rng.integers(1, 12, size=max(nvocab - len(vocab), 0))
    vocab += [b"t%d_" % i + b"x" * int(n) for i, n in enumerate(lens)]
    if multimodal:
        vocab.append(b"<image_soft_token>")
    merges = [(b"t%d" % i, b"_x") for i in range(int(rng.integers(3, 17)))]
    return vocab, merges


def layout(text: dict, vision: dict | None, header_len: int):
    """Every tensor of the file after the header, in file order:
    (name, kind or None, layer, offset, rows, k) for QTensors (k = 0 and
    rows = float count for plain float tensors)."""
    recs = []
    off = header_len

    def qt(name, kind, layer, rows, k):
        nonlocal off
        recs.append((name, kind, layer, off, rows, k))
        off += rows * k + 4 * rows

    def fl(name, n, layer=-1):
        nonlocal off
        recs.append((name, None, layer, off, n, 0))
        off += 4 * n

    d, m = text["dim"], text["mlp_dim"]
    q_sz, kv_sz = text["n_heads"] * text["hdim"], text["nkv"] * text["hdim"]
    qt("emb", "lm_head", -1, text["nvocab"], d)
    for l in range(text["nl"]):
        qt("wq", "wq", l, q_sz, d)
        qt("wk", "wk", l, kv_sz, d)
        qt("wv", "wv", l, kv_sz, d)
        qt("wo", "wo", l, d, q_sz)
        if text.get("qk_norm"):
            fl("nq", text["hdim"], l)
            fl("nk", text["hdim"], l)
        qt("w1", "w1", l, m, d)
        qt("w2", "w2", l, m, d)
        qt("w3", "w3", l, d, m)
        fl("n1", d, l)
        fl("n2", d, l)
        if text.get("mlp_pre"):
            fl("n3", d, l)
        if text.get("mlp_pst"):
            fl("n4", d, l)
    fl("fnorm", d)
    text_end = off
    if vision:
        vd, vm, p = vision["dim"], vision["mlp_dim"], vision["psize"]
        side = vision["img_px"] // p
        fl("pe", vd * 3 * p * p)
        fl("pe_b", vd)
        qt("pos_emb", None, -1, side * side, vd)
        for l in range(vision["nl"]):
            fl("n1", vd, l)
            fl("n1_b", vd, l)
            for nm in ("wq", "wk", "wv", "wo"):
                qt(nm, "v" + nm, l, vd, vd)
            for nm in ("bq", "bk", "bv", "bo", "n2", "n2_b"):
                fl(nm, vd, l)
            qt("w1", "vw1", l, vm, vd)
            qt("w2", "vw2", l, vd, vm)
            fl("b1", vm, l)
            fl("b2", vd, l)
        fl("post_n", vd)
        fl("post_nb", vd)
        fl("norm", vd)
        qt("proj", "vproj", -1, d, vd)
    return recs, text_end, off


def expected_qtensors(text: dict, vision: dict | None, header_len: int, allow_mm: bool = True):
    """The records gcu_bin_qtensors should return, from this module's own layout."""
    recs, _, _ = layout(text, vision, header_len)
    out = []
    for name, kind, layer, off, rows, k in recs:
        if kind is None or (kind.startswith("v") and not (vision and allow_mm)):
            continue
        out.append({"kind": kind, "layer": layer, "rows": rows, "k": k, "q_off": off, "s_off": off + rows * k})
    return out


def image(text: dict, vision: dict | None = None, seed: int = 0, fast: bool = False, pad: int = 0):
    """(uint8 image, header length).  `fast` fills tensors with a repeating
    seeded block instead of drawing every value (for multi-GB images)."""
    vocab, merges = default_tokenizer(text["nvocab"] if text["nvocab"] < 4096 else 0, bool(vision), seed)
    if text["nvocab"] >= 4096:  # large vocabularies: short generated strings
        vocab = [b"v%d" % i for i in range(text["nvocab"])] + ([b"<image_soft_token>"] if vision else [])
    hdr = _header(text, vision, vocab, merges)
    recs, _, end = layout(text, vision, len(hdr))
    buf = np.zeros(end + pad, np.uint8)
    buf[:len(hdr)] = np.frombuffer(hdr, np.uint8)
    block = None
    if fast:
        rng = np.random.default_rng(seed)
        block = rng.integers(-127, 128, size=1 << 20, dtype=np.int8).view(np.uint8)
    for i, (name, kind, layer, off, rows, k) in enumerate(recs):
        rng = np.random.default_rng((seed << 20) + i)
        if k:
            n = rows * k
            if fast:
                _tile_fill(buf, off, n, block)
            else:
                buf[off:off + n] = rng.integers(-127, 128, size=n, dtype=np.int8).view(np.uint8)
            sc = (rng.random(rows, dtype=np.float32) * 1e-3 + 1e-4).astype("<f4")
            buf[off + n:off + n + 4 * rows] = sc.view(np.uint8)
        else:
            vals = (rng.standard_normal(rows, dtype=np.float32) * 0.1).astype("<f4")
            buf[off:off + 4 * rows] = vals.view(np.uint8)
    return buf, len(hdr)


def _tile_fill(buf, off, n, block):
    for s in range(0, n, block.size):
        e = min(n, s + block.size)
        buf[off + s:off + e] = block[:e - s]


def qtensor_arrays(buf: np.ndarray, rec: dict):
    """(int8 [rows][k], f32 [rows]) views of one record into the image."""
    q = buf[rec["q_off"]:rec["q_off"] + rec["rows"] * rec["k"]].view(np.int8).reshape(rec["rows"], rec["k"])
    s = buf[rec["s_off"]:rec["s_off"] + 4 * rec["rows"]].view(np.float32)
    return q, s
