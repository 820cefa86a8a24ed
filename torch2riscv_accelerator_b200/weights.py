"""Host-side model preparation (offline, NumPy): synthetic fp32 weights,
per-output-channel int8 quantization, RoPE tables and the per-layer KV
constants. This is the model-format step of the reference
(`llm/export_w8a8.py:75-99` device_tensors, `llm/ref_model.py:142-148`
quantize_rows, `compiler/frontend/qhf.py:254-300` QModel.__init__); the GPU
layout it produces is in `model.py`.

Weights are N(0, 0.02) float32 drawn per tensor from
`np.random.default_rng(SeedSequence([seed, tensor, layer]))`, so any layer
can be regenerated alone.
"""
import numpy as np

F = np.float32

_TENSOR_IDS = {"tok": 1, "wq": 2, "wk": 3, "wv": 4, "wo": 5, "w1": 6, "w3": 7, "w2": 8, "wcls": 9,
               "rms_att": 10, "rms_ffn": 11, "rms_final": 12, "q_norm": 13, "k_norm": 14,
               "router": 15, "e_gate": 16, "e_up": 17, "e_down": 18}


def _rng(seed, name, layer):
    return np.random.default_rng(np.random.SeedSequence([seed, _TENSOR_IDS[name], layer + 1]))


def gen_tensor(cfg, seed, name, layer=-1, gains="ones", std=0.02):
    """One fp32 tensor of the synthetic model, in PyTorch (out, in) orientation."""
    c = cfg
    shapes = {"tok": (c.vocab, c.dim), "wcls": (c.vocab, c.dim), "wq": (c.q_dim, c.dim), "wk": (c.kv_dim, c.dim),
              "wv": (c.kv_dim, c.dim), "wo": (c.dim, c.q_dim), "w1": (c.hidden, c.dim), "w3": (c.hidden, c.dim),
              "w2": (c.dim, c.hidden), "rms_att": (c.dim,), "rms_ffn": (c.dim,), "rms_final": (c.dim,),
              "q_norm": (c.head_dim,), "k_norm": (c.head_dim,), "router": (c.experts, c.dim),
              "e_gate": (c.experts, c.expert_hidden, c.dim), "e_up": (c.experts, c.expert_hidden, c.dim),
              "e_down": (c.experts, c.dim, c.expert_hidden)}
    shape = shapes[name]
    r = _rng(seed, name, layer)
    if name in ("rms_att", "rms_ffn", "rms_final", "q_norm", "k_norm"):
        if gains == "ones":
            return np.ones(shape, F)
        return (F(1) + F(0.1) * r.standard_normal(shape, dtype=F)).astype(F)
    return (r.standard_normal(shape, dtype=F) * F(std)).astype(F)


def quantize_rows(wt):
    """Symmetric int8 per output row: s = amax/127 (s = 1 for an all-zero
    row, `hf_generic._quantize_rows` :558-565), q = RNE(w/s) clipped to +-127
    (`llm/ref_model.py:136-148`)."""
    wt = np.asarray(wt, F)
    s = (np.abs(wt).max(axis=-1) / F(127)).astype(F)
    s = np.where(s == 0, F(1), s).astype(F)
    with np.errstate(divide="ignore", invalid="ignore"):
        y = np.rint(wt / s[..., None])
    q = np.clip(np.nan_to_num(y, nan=0.0, posinf=127, neginf=-127), -127, 127).astype(np.int8)
    return q, s


def rope_tables(cfg):
    """(cos, sin) float32 [seq_len, head_dim], each value repeated for both
    elements of its rotation pair (`llm/export_w8a8.py:84-86`).
    "llama2c": `llm/ref_model.py:34-41` (float32 arithmetic);
    "hf": `compiler/frontend/qhf.py:183-189` (float64, rounded once)."""
    hs = cfg.head_dim
    if cfg.rope == "llama2c":
        hd = (np.arange(0, hs, 2) % hs).astype(F)
        freq = F(1.0) / np.power(F(cfg.theta), hd / F(hs))
        val = np.arange(cfg.seq_len, dtype=F)[:, None] * freq[None, :]
        cos, sin = np.cos(val).astype(F), np.sin(val).astype(F)
    else:
        freq = 1.0 / np.power(cfg.theta, np.arange(0, hs, 2, dtype=np.float64) / hs)
        val = np.arange(cfg.seq_len, dtype=np.float64)[:, None] * freq[None, :]
        cos, sin = np.cos(val).astype(F), np.sin(val).astype(F)
    return np.repeat(cos, 2, axis=1).astype(F), np.repeat(sin, 2, axis=1).astype(F)


def kv_consts(s_k, s_v, head_dim):
    """(inv_sk, inv_sv, a_k, a_v) computed as the reference does on the host
    (`llm/export_w8a8.py:68-72`, `llm/ref_model.py:228-231`)."""
    s_k, s_v = F(s_k), F(s_v)
    return (F(1.0 / s_k), F(1.0 / s_v), F(float(s_k) / np.sqrt(head_dim)), F(float(s_v) / 127.0))


class QuantWeights:
    """The quantized model on the host: int8 rows + fp32 scales per linear layer
    (q|k|v rows fused as wqkv, w1|w3 as w13, `llm/export_w8a8.py:90-93`),
    fp32 gains, the int8 embedding (shared with a tied classifier)."""

    def __init__(self, cfg, seed=0, gains="ones", layers=None, with_cls=True):
        cfg.validate()
        self.cfg, self.seed = cfg, seed
        g = lambda n, l=-1: gen_tensor(cfg, seed, n, l, gains)
        self.emb_q, self.emb_s = quantize_rows(g("tok"))
        if with_cls:
            self.cls_q, self.cls_s = (self.emb_q, self.emb_s) if cfg.tied else quantize_rows(g("wcls"))
        self.rms_final = g("rms_final")
        self.layers = []
        for l in range(cfg.layers if layers is None else layers):
            t = {"rms_att": g("rms_att", l), "rms_ffn": g("rms_ffn", l)}
            t["wqkv"], t["s_wqkv"] = quantize_rows(np.concatenate([g("wq", l), g("wk", l), g("wv", l)]))
            t["wo"], t["s_wo"] = quantize_rows(g("wo", l))
            if cfg.qk_norm:
                t["q_norm"], t["k_norm"] = g("q_norm", l), g("k_norm", l)
            if cfg.moe:
                t["router"], t["s_router"] = quantize_rows(g("router", l))
                for n in ("e_gate", "e_up", "e_down"):
                    t[n], t["s_" + n] = quantize_rows(g(n, l))
            else:
                t["w1"], t["s_w1"] = quantize_rows(g("w1", l))
                t["w3"], t["s_w3"] = quantize_rows(g("w3", l))
                t["w2"], t["s_w2"] = quantize_rows(g("w2", l))
            self.layers.append(t)
        self.cos, self.sin = rope_tables(cfg)
