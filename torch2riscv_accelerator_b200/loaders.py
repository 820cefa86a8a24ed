"""Model files of the reference, read (and written) for this runtime.

* llama2.c legacy checkpoints (`llm/checkpoint.py:33-59`): a header of seven
  int32 (dim, hidden, layers, heads, kv_heads, vocab, seq_len; a negative vocab
  means a separate classifier follows), then fp32 tensors in the run.c order
  (tok, rms_att, wq, wk, wv, wo, rms_ffn, w1, w2, w3, rms_final, the unused
  RoPE frequencies of seq_len * head_size floats, [wcls]), linear weights
  (out, in). `load_llama2c` returns (ModelConfig, fp32 tensors in the
  reference's naming); `weights.from_fp32` quantizes them.

* The device format `.w8a8` (`llm/export_w8a8.py:1-33, 102-168`): a 64-byte
  header (magic "W8A8LLM\\0", u32 version 1, D, dim, hidden, layers, heads,
  kv_heads, vocab, seq_len, n_entries, layer_base, layer_stride), a table of
  32-byte entries (name[16], u32 offset, bytes, per_layer, reserved), then the
  tensors, each 64-byte aligned; the layers share one layout at a fixed
  stride. Linear weights are stored as the overlay's B tiles (tile t = the
  output rows [tD, (t+1)D) transposed, in x D); the reader turns them back into
  row-major int8 [out, in], this GPU's layout. Per layer "kvp" holds the
  static KV scales (s_k, s_v, ...). `read_w8a8` returns (ModelConfig,
  QuantWeights-like, kv_scales [layers, 2]); `write_w8a8` writes the same
  format from quantized weights (the file a `.w8a8` consumer of the reference
  reads).

The byte layout is the reference's by necessity (a drop-in reads the files its
tools write); the code is this repository's own.
"""
import struct

import numpy as np

from . import config as C

F = np.float32
MAGIC = b"W8A8LLM\0"
VERSION = 1
_HDR = struct.Struct("<8s12I")
_ENT = struct.Struct("<16s4I")
_ALIGN = 64
_LAYER_ORDER = ("rms_att", "rms_ffn", "wqkv", "s_wqkv", "wo", "s_wo", "w13", "s_w13", "w2", "s_w2", "kvp")
_GLOBAL_ORDER = ("emb_q", "emb_s", "rms_final", "wcls", "s_wcls", "rope_cos", "rope_sin")
_INT8 = {"emb_q", "wcls", "wqkv", "wo", "w13", "w2"}


def _llama2c_config(name, dim, hidden, layers, heads, kv_heads, vocab, seq_len):
    """A llama2.c model: theta 1e4, eps 1e-5, NORM attention, interleaved RoPE."""
    return C.ModelConfig(name, dim, hidden, layers, heads, kv_heads, dim // heads, vocab, seq_len, theta=10000.0,
                         eps=1e-5, tied=False, attn="norm", rope="llama2c")


# ------------------------------------------------------------ llama2.c .bin
def load_llama2c(path, name="llama2c"):
    """(ModelConfig, {name: fp32 array}) of a legacy llama2.c checkpoint."""
    raw = np.fromfile(path, dtype=np.float32)
    if raw.size < 7:
        raise ValueError(f"{path}: too short for a llama2.c header")
    dim, hidden, layers, heads, kv_heads, vocab, seq = struct.unpack("<7i", raw[:7].tobytes())
    if min(dim, hidden, layers, heads, kv_heads, seq) <= 0 or vocab == 0 or dim % heads:
        raise ValueError(f"{path}: not a llama2.c header ({dim}, {hidden}, {layers}, {heads}, {kv_heads}, {vocab})")
    shared, vocab = vocab > 0, abs(vocab)
    hs = dim // heads
    kv = kv_heads * hs
    order = [("tok", (vocab, dim)), ("rms_att", (layers, dim)), ("wq", (layers, dim, dim)),
             ("wk", (layers, kv, dim)), ("wv", (layers, kv, dim)), ("wo", (layers, dim, dim)),
             ("rms_ffn", (layers, dim)), ("w1", (layers, hidden, dim)), ("w2", (layers, dim, hidden)),
             ("w3", (layers, hidden, dim)), ("rms_final", (dim,)), ("freq", (seq * hs,))]
    if not shared:
        order.append(("wcls", (vocab, dim)))
    w, off = {}, 7
    for n, shape in order:
        cnt = int(np.prod(shape))
        if off + cnt > raw.size:
            raise ValueError(f"{path}: ends inside {n}")
        w[n] = raw[off:off + cnt].reshape(shape)
        off += cnt
    if off != raw.size:
        raise ValueError(f"{path}: {raw.size} floats, {off} expected")
    del w["freq"]
    if shared:
        w["wcls"] = w["tok"]
    return _llama2c_config(name, dim, hidden, layers, heads, kv_heads, vocab, seq), w


def write_llama2c(path, cfg, w):
    """Write fp32 tensors (the reference's naming) as a legacy llama2.c file;
    the classifier is shared when w["wcls"] is w["tok"]."""
    shared = w.get("wcls") is None or w["wcls"] is w["tok"]
    hs = cfg.dim // cfg.heads
    parts = [np.frombuffer(struct.pack("<7i", cfg.dim, cfg.hidden, cfg.layers, cfg.heads, cfg.kv_heads,
                                       cfg.vocab if shared else -cfg.vocab, cfg.seq_len), F)]
    for n in ("tok", "rms_att", "wq", "wk", "wv", "wo", "rms_ffn", "w1", "w2", "w3", "rms_final"):
        parts.append(np.asarray(w[n], F).ravel())
    parts.append(np.zeros(cfg.seq_len * hs, F))                     # RoPE frequencies: unused by readers
    if not shared:
        parts.append(np.asarray(w["wcls"], F).ravel())
    np.concatenate(parts).tofile(path)


# ------------------------------------------------------------------ .w8a8
def _unpack_b(tiles):
    """Overlay B tiles (out/D, in, D) -> row-major int8 [out, in]."""
    nt, inp, d = tiles.shape
    return np.ascontiguousarray(tiles.transpose(0, 2, 1).reshape(nt * d, inp))


def _pack_b(q, d):
    """Row-major int8 [out, in] -> overlay B tiles (out/D, in, D)."""
    out, inp = q.shape
    if out % d or inp % d:
        raise ValueError(f"a {out} x {inp} linear is not a multiple of D = {d}")
    return np.ascontiguousarray(q.reshape(out // d, d, inp).transpose(0, 2, 1))


class W8A8Model:
    """The contents of a .w8a8 file in this runtime's layout (QuantWeights-like:
    emb_q/emb_s, cls_q/cls_s, rms_final, cos/sin, layers[l] dicts)."""


def read_w8a8(path_or_bytes, name="w8a8"):
    """(ModelConfig, W8A8Model, kv_scales [layers, 2]) of a .w8a8 file."""
    raw = (np.fromfile(path_or_bytes, np.uint8) if isinstance(path_or_bytes, str)
           else np.frombuffer(path_or_bytes, np.uint8))
    if raw.size < _HDR.size:
        raise ValueError("too short for a w8a8 header")
    h = _HDR.unpack(raw[:_HDR.size].tobytes())
    if h[0] != MAGIC or h[1] != VERSION:
        raise ValueError("not a w8a8 version 1 file")
    d, dim, hidden, layers, heads, kv_heads, vocab, seq, n, base, stride = h[2:]
    cfg = _llama2c_config(name, dim, hidden, layers, heads, kv_heads, vocab, seq)
    ents = {}
    for i in range(n):
        nm, off, nb, per, _ = _ENT.unpack(raw[64 + i * _ENT.size:64 + (i + 1) * _ENT.size].tobytes())
        ents[nm.rstrip(b"\0").decode()] = (off, nb, bool(per))

    def get(nm, layer=None):
        off, nb, per = ents[nm]
        if per:
            off = base + layer * stride + off
        if off + nb > raw.size:
            raise ValueError(f"{nm} runs past the end of the file")
        return raw[off:off + nb].view(np.int8 if nm in _INT8 else F)

    m = W8A8Model()
    hs, kv = dim // heads, kv_heads * (dim // heads)
    m.emb_q = get("emb_q").reshape(vocab, dim).copy()
    m.emb_s = get("emb_s").copy()
    m.cls_q = _unpack_b(get("wcls").reshape(vocab // d, dim, d))
    m.cls_s = get("s_wcls").copy()
    m.rms_final = get("rms_final").copy()
    m.cos = get("rope_cos").reshape(seq, dim)[:, :hs].copy()      # the same for every head
    m.sin = get("rope_sin").reshape(seq, dim)[:, :hs].copy()
    m.layers, kvs = [], []
    for l in range(layers):
        t = {"rms_att": get("rms_att", l).copy(), "rms_ffn": get("rms_ffn", l).copy()}
        t["wqkv"] = _unpack_b(get("wqkv", l).reshape(-1, dim, d))
        t["s_wqkv"] = get("s_wqkv", l).copy()
        t["wo"] = _unpack_b(get("wo", l).reshape(dim // d, dim, d))
        t["s_wo"] = get("s_wo", l).copy()
        w13 = _unpack_b(get("w13", l).reshape(2 * hidden // d, dim, d))
        s13 = get("s_w13", l)
        t["w1"], t["w3"] = w13[:hidden].copy(), w13[hidden:].copy()
        t["s_w1"], t["s_w3"] = s13[:hidden].copy(), s13[hidden:].copy()
        t["w2"] = _unpack_b(get("w2", l).reshape(dim // d, hidden, d))
        t["s_w2"] = get("s_w2", l).copy()
        if t["wqkv"].shape[0] != dim + 2 * kv:
            raise ValueError(f"layer {l}: wqkv has {t['wqkv'].shape[0]} rows, {dim + 2 * kv} expected")
        kvs.append(get("kvp", l)[:2].copy())
        m.layers.append(t)
    return cfg, m, np.stack(kvs).astype(F)


def write_w8a8(path, cfg, qw, kv_scales, d=16):
    """Write quantized weights (QuantWeights-like, llama2.c-style dense model)
    as a .w8a8 file with D = d; returns its size in bytes."""
    if cfg.moe or cfg.qk_norm:
        raise ValueError(".w8a8 holds llama2.c-style dense models only")
    hs = cfg.dim // cfg.heads
    g = {"emb_q": qw.emb_q, "emb_s": qw.emb_s, "rms_final": qw.rms_final,
         "wcls": _pack_b(np.asarray(qw.cls_q, np.int8), d), "s_wcls": qw.cls_s}
    cos_full = np.tile(np.asarray(qw.cos, F), (1, cfg.heads))         # (seq, dim): the head's table per head
    sin_full = np.tile(np.asarray(qw.sin, F), (1, cfg.heads))
    g["rope_cos"], g["rope_sin"] = cos_full, sin_full
    per = []
    for l, t in enumerate(qw.layers):
        s_k, s_v = F(kv_scales[l][0]), F(kv_scales[l][1])
        kvp = np.array([s_k, s_v, F(1.0 / s_k), F(1.0 / s_v), F(float(s_k) / np.sqrt(hs)), F(float(s_v) / 127.0),
                        0, 0], F)
        per.append({"rms_att": t["rms_att"], "rms_ffn": t["rms_ffn"],
                    "wqkv": _pack_b(np.asarray(t["wqkv"], np.int8), d), "s_wqkv": t["s_wqkv"],
                    "wo": _pack_b(np.asarray(t["wo"], np.int8), d), "s_wo": t["s_wo"],
                    "w13": _pack_b(np.concatenate([t["w1"], t["w3"]]).astype(np.int8), d),
                    "s_w13": np.concatenate([t["s_w1"], t["s_w3"]]),
                    "w2": _pack_b(np.asarray(t["w2"], np.int8), d), "s_w2": t["s_w2"], "kvp": kvp})
    a = lambda x: -(-x // _ALIGN) * _ALIGN
    as_bytes = lambda x: np.ascontiguousarray(x, np.int8 if x.dtype == np.int8 else F).tobytes()
    n_ent = len(_GLOBAL_ORDER) + len(_LAYER_ORDER)
    off = a(64 + _ENT.size * n_ent)
    ents, blobs = [], []
    for nm in _GLOBAL_ORDER:
        b = as_bytes(np.asarray(g[nm]))
        ents.append((nm, off, len(b), 0))
        blobs.append((off, b))
        off = a(off + len(b))
    base, rel = off, 0
    rels = {}
    for nm in _LAYER_ORDER:
        nb = len(as_bytes(np.asarray(per[0][nm])))
        ents.append((nm, rel, nb, 1))
        rels[nm] = rel
        rel = a(rel + nb)
    stride = rel
    buf = np.zeros(base + stride * cfg.layers, np.uint8)
    head = _HDR.pack(MAGIC, VERSION, d, cfg.dim, cfg.hidden, cfg.layers, cfg.heads, cfg.kv_heads, cfg.vocab,
                     cfg.seq_len, n_ent, base, stride)
    buf[:len(head)] = np.frombuffer(head, np.uint8)
    for i, (nm, o, nb, pl) in enumerate(ents):
        e = _ENT.pack(nm.encode().ljust(16, b"\0"), o, nb, pl, 0)
        buf[64 + i * _ENT.size:64 + (i + 1) * _ENT.size] = np.frombuffer(e, np.uint8)
    for o, b in blobs:
        buf[o:o + len(b)] = np.frombuffer(b, np.uint8)
    for l in range(cfg.layers):
        for nm in _LAYER_ORDER:
            b = as_bytes(np.asarray(per[l][nm]))
            o = base + l * stride + rels[nm]
            buf[o:o + len(b)] = np.frombuffer(b, np.uint8)
    buf.tofile(path)
    return buf.size
