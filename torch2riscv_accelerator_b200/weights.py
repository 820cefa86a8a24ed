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


def layer_kv_consts(kv_l, head_dim):
    """A layer's KV constants from its scales: [2] (per layer) or [2, kv_dim]
    (per cache channel, `calibrate_kv(channel=...)`; a part whose row holds a
    single value is per layer), as `hf_generic.SaCache` (:153-187) computes them:
    ((inv_sk, inv_sv, a_k, a_v) scalars, per-channel arrays or None). K per
    channel: k_scale = s_k (folded into q), inv_sk_ch = F(1) / s_k, a_k =
    F(1 / sqrt(head_dim)); V per channel: inv_sv_ch = F(1) / s_v, a_v_ch =
    s_v * F(1/127)."""
    kv_l = np.asarray(kv_l, F)
    if kv_l.ndim == 1:
        return kv_consts(kv_l[0], kv_l[1], head_dim), None
    inv_sk, inv_sv, a_k, a_v = kv_consts(kv_l[0, 0], kv_l[1, 0], head_dim)
    ch = {}
    if not np.all(kv_l[0] == kv_l[0, 0]):
        ch["k_scale"], ch["inv_sk_ch"] = kv_l[0].copy(), (F(1.0) / kv_l[0]).astype(F)
        a_k = F(1.0 / np.sqrt(head_dim))
    if not np.all(kv_l[1] == kv_l[1, 0]):
        ch["inv_sv_ch"], ch["a_v_ch"] = (F(1.0) / kv_l[1]).astype(F), (kv_l[1] * F(1.0 / 127.0)).astype(F)
    return (inv_sk, inv_sv, a_k, a_v), (ch or None)


class QuantWeights:
    """The quantized model on the host: int8 rows + fp32 scales per linear layer
    (q|k|v rows fused as wqkv, w1|w3 as w13, `llm/export_w8a8.py:90-93`),
    fp32 gains, the int8 embedding (shared with a tied classifier)."""

    def __init__(self, cfg, seed=0, gains="ones", layers=None, with_cls=True, calib_tokens=None, kv_channel=""):
        """calib_tokens: token ids of an fp32 calibration run; the static KV
        scales it gives are in self.kv_scales (`compiler/frontend/qhf.py:245-251`
        calibrate_kv: max|k|, max|v| per layer after RoPE / QK-norm, / 127);
        kv_channel "k" / "v" / "kv": those parts per cache channel
        (`compiler/frontend/hf_generic.py:466-491`), kv_scales [layers, 2, kv_dim]."""
        cfg.validate()
        self.cfg, self.seed = cfg, seed
        g = lambda n, l=-1: gen_tensor(cfg, seed, n, l, gains)
        tok = g("tok")
        self.emb_q, self.emb_s = quantize_rows(tok)
        if with_cls:
            self.cls_q, self.cls_s = (self.emb_q, self.emb_s) if cfg.tied else quantize_rows(g("wcls"))
        self.rms_final = g("rms_final")
        self.cos, self.sin = rope_tables(cfg)
        cal = None if calib_tokens is None else tok[np.asarray(calib_tokens)].astype(F)
        del tok
        L = cfg.layers if layers is None else layers
        amax = np.zeros((L, 2, cfg.kv_dim), F)
        self.layers = []
        for l in range(L):
            t = {"rms_att": g("rms_att", l), "rms_ffn": g("rms_ffn", l)}
            f32 = {n: g(n, l) for n in ("wq", "wk", "wv", "wo")}
            t["wqkv"], t["s_wqkv"] = quantize_rows(np.concatenate([f32["wq"], f32["wk"], f32["wv"]]))
            t["wo"], t["s_wo"] = quantize_rows(f32["wo"])
            if cfg.qk_norm:
                t["q_norm"], t["k_norm"] = g("q_norm", l), g("k_norm", l)
            if cfg.moe:
                t["router"], t["s_router"] = quantize_rows(g("router", l))
                for n in ("e_gate", "e_up", "e_down"):
                    f32[n] = g(n, l)
                    t[n], t["s_" + n] = quantize_rows(f32[n])
                f32["router"] = g("router", l)
            else:
                for n in ("w1", "w3", "w2"):
                    f32[n] = g(n, l)
                    t[n], t["s_" + n] = quantize_rows(f32[n])
            if cal is not None:
                cal, amax[l, 0], amax[l, 1] = calibrate_layer(cfg, cal, t, f32, self.cos, self.sin)
            self.layers.append(t)
        self.kv_amax = amax if cal is not None else None
        self.kv_scales = kv_scales_of(amax, kv_channel) if cal is not None else None


def kv_scales_of(amax, channel=""):
    """Static KV scales from the calibration maxima amax [layers, 2, kv_dim]
    (`hf_generic.calibrate_kv` :466-491): max / 127 per layer ([layers, 2]), or
    with channel "k" / "v" / "kv" those parts per cache channel and the others'
    rows the layer's single value ([layers, 2, kv_dim]); at least 1e-8."""
    amax = np.asarray(amax, F)
    if not channel:
        return (np.maximum(amax.max(-1), F(1e-8)) / F(127.0)).astype(F)
    out = np.repeat(amax.max(-1, keepdims=True), amax.shape[-1], -1)
    for j, part in enumerate("kv"):
        if part in channel:
            out[:, j] = amax[:, j]
    return (np.maximum(out, F(1e-8)) / F(127.0)).astype(F)


def calibrate_kv(cfg, w, tokens, channel=""):
    """KV scales from fp32 runs of the model w (fp32 tensors in the
    reference's naming, `llm/checkpoint.py:33-59`) over `tokens` (one sequence,
    or a list of sequences each from position 0): the maxima of |k|, |v| per
    cache channel as they are written (after QK-norm and RoPE) over all runs,
    then kv_scales_of (`hf_generic.calibrate_kv`)."""
    runs = [tokens] if np.ndim(tokens[0]) == 0 else list(tokens)
    cos, sin = rope_tables(cfg)
    amax = np.zeros((cfg.layers, 2, cfg.kv_dim), F)
    names = ("wq", "wk", "wv", "wo") + (("router", "e_gate", "e_up", "e_down") if cfg.moe else ("w1", "w3", "w2"))
    for run in runs:
        x = w["tok"][np.asarray(run)].astype(F)
        for l in range(cfg.layers):
            t = {"rms_att": w["rms_att"][l], "rms_ffn": w["rms_ffn"][l]}
            if cfg.qk_norm:
                t["q_norm"], t["k_norm"] = w["q_norm"][l], w["k_norm"][l]
            x, k, v = calibrate_layer(cfg, x, t, {n: w[n][l] for n in names}, cos, sin)
            amax[l, 0], amax[l, 1] = np.maximum(amax[l, 0], k), np.maximum(amax[l, 1], v)
    return kv_scales_of(amax, channel)


def fp32_forward(cfg, w, tokens, last_only=False):
    """The fp32 model's logits at every position of `tokens` (from position 0,
    causal): the reference's Fp32Model (`llm/ref_model.py`, `qhf.py:210-242`)
    in NumPy float32, for quality evaluation. w: fp32 tensors in the
    reference's naming (plus router / e_gate / e_up / e_down for MoE)."""
    cos, sin = rope_tables(cfg)
    x = w["tok"][np.asarray(tokens)].astype(F)
    for l in range(cfg.layers):
        t = {"rms_att": w["rms_att"][l], "rms_ffn": w["rms_ffn"][l]}
        if cfg.qk_norm:
            t["q_norm"], t["k_norm"] = w["q_norm"][l], w["k_norm"][l]
        names = ("wq", "wk", "wv", "wo") + (("router", "e_gate", "e_up", "e_down") if cfg.moe else ("w1", "w3", "w2"))
        x, _, _ = calibrate_layer(cfg, x, t, {n: w[n][l] for n in names}, cos, sin)
    wcls = w.get("wcls", w["tok"]) if not cfg.tied else w["tok"]
    if last_only:
        x = x[-1:]
    return (_rms32(x, w["rms_final"], cfg.eps) @ wcls.T).astype(F)


def _rms32(x, g, eps):
    return (x * (1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + F(eps))) * g).astype(F)


def _swapneg(v):
    sw = np.empty_like(v)
    sw[..., 0::2], sw[..., 1::2] = -v[..., 1::2], v[..., 0::2]
    return sw


def calibrate_layer(cfg, x, t, f32, cos, sin):
    """One layer of the fp32 model (`compiler/frontend/qhf.py:210-242`
    Fp32Model.forward, all calibration tokens at once with a causal mask):
    returns (x after the layer, max|k|, max|v| per cache channel [kv_dim])."""
    c = cfg
    n = x.shape[0]
    H, Hk, hd, G = c.heads, c.kv_heads, c.head_dim, c.group
    xb = _rms32(x, t["rms_att"], c.eps)
    q = (xb @ f32["wq"].T).reshape(n, H, hd)
    k = (xb @ f32["wk"].T).reshape(n, Hk, hd)
    v = (xb @ f32["wv"].T).reshape(n, Hk, hd)
    if c.qk_norm:
        q, k = _rms32(q, t["q_norm"], c.eps), _rms32(k, t["k_norm"], c.eps)
    cs, sn = cos[:n, None, :], sin[:n, None, :]
    q = (q * cs + _swapneg(q) * sn).astype(F)
    k = (k * cs + _swapneg(k) * sn).astype(F)
    s = np.einsum("qhd,thd->hqt", q, np.repeat(k, G, axis=1)) / F(np.sqrt(hd))
    s = np.where(np.tril(np.ones((n, n), bool))[None], s, -np.inf)
    p = np.exp(s - s.max(-1, keepdims=True))
    p = p / p.sum(-1, keepdims=True)
    att = np.einsum("hqt,thd->qhd", p, np.repeat(v, G, axis=1)).reshape(n, -1).astype(F)
    x = (x + att @ f32["wo"].T).astype(F)
    xb = _rms32(x, t["rms_ffn"], c.eps)
    if c.moe:
        logits = xb @ f32["router"].T
        y = np.zeros_like(x)
        for r in range(n):
            ids = np.argsort(-logits[r], kind="stable")[:c.top_k]
            e = np.exp(logits[r, ids] - logits[r, ids[0]])
            w = e / e.sum()
            for wk, i in zip(w, ids):
                gg, uu = f32["e_gate"][i] @ xb[r], f32["e_up"][i] @ xb[r]
                y[r] += wk * (f32["e_down"][i] @ (gg / (1 + np.exp(-gg)) * uu))
        x = (x + y).astype(F)
    else:
        h1, h3 = xb @ f32["w1"].T, xb @ f32["w3"].T
        if c.act == "gelu_tanh":                     # torch's gelu(approximate="tanh") in fp32
            a = (F(0.5) * h1 * (F(1) + np.tanh(F(np.sqrt(2.0 / np.pi)) * (h1 + F(0.044715) * h1 ** 3)))).astype(F)
        else:
            a = h1 / (1 + np.exp(-h1))
        x = (x + (a * h3) @ f32["w2"].T).astype(F)
    return x, np.abs(k).max(axis=0).reshape(-1), np.abs(v).max(axis=0).reshape(-1)


def from_fp32(cfg, w):
    """QuantWeights from fp32 tensors in the reference's naming
    (`llm/checkpoint.py:33-59`: tok, rms_att, wq, wk, wv, wo, rms_ffn, w1, w2,
    w3, rms_final, optional wcls; q_norm / k_norm for QK-norm models), e.g. a
    llama2.c checkpoint; quantized per output row as `llm/export_w8a8.py:75-99`."""
    cfg.validate()
    qw = QuantWeights.__new__(QuantWeights)
    qw.cfg, qw.seed = cfg, None
    qw.emb_q, qw.emb_s = quantize_rows(w["tok"])
    if cfg.tied or "wcls" not in w or w["wcls"] is w["tok"]:
        qw.cls_q, qw.cls_s = qw.emb_q, qw.emb_s
    else:
        qw.cls_q, qw.cls_s = quantize_rows(w["wcls"])
    qw.rms_final = np.asarray(w["rms_final"], F)
    qw.layers = []
    for l in range(cfg.layers):
        t = {"rms_att": np.asarray(w["rms_att"][l], F), "rms_ffn": np.asarray(w["rms_ffn"][l], F)}
        t["wqkv"], t["s_wqkv"] = quantize_rows(np.concatenate([w["wq"][l], w["wk"][l], w["wv"][l]]))
        t["wo"], t["s_wo"] = quantize_rows(w["wo"][l])
        for n in (("router", "e_gate", "e_up", "e_down") if cfg.moe else ("w1", "w3", "w2")):
            t[n], t["s_" + n] = quantize_rows(w[n][l])            # (experts: per output row of each)
        if cfg.qk_norm:
            t["q_norm"], t["k_norm"] = np.asarray(w["q_norm"][l], F), np.asarray(w["k_norm"][l], F)
        qw.layers.append(t)
    qw.cos, qw.sin = rope_tables(cfg)
    return qw


def fp32_model(cfg, seed, gains="ones", std=0.02, layers=None):
    """The synthetic model's fp32 tensors in the reference's naming."""
    g = lambda n, l=-1: gen_tensor(cfg, seed, n, l, gains, std)
    L = cfg.layers if layers is None else layers
    w = {"tok": g("tok"), "rms_final": g("rms_final")}
    names = ["rms_att", "rms_ffn", "wq", "wk", "wv", "wo"]
    names += ["router", "e_gate", "e_up", "e_down"] if cfg.moe else ["w1", "w2", "w3"]
    if cfg.qk_norm:
        names += ["q_norm", "k_norm"]
    for n in names:
        w[n] = np.stack([g(n, l) for l in range(L)])
    if not cfg.tied:
        w["wcls"] = g("wcls")
    return w
