"""The W8A8 decoder restated on the CPU (test oracle).

`OracleDecoder.forward_rows` computes one sequence's rows (a decode step is one
row, a prefill chunk M rows), each row exactly as a decode step:
- `llm/ref_model.py:216-255` (DeviceModel.forward: embedding, per layer
  quant_act(rmsnorm) -> q/k/v linear -> RoPE -> int8 KV append -> per-head
  attention -> quant_act -> wo -> residual -> FFN with SiLU gating -> residual,
  final quant_act(rmsnorm) -> classifier);
- `compiler/frontend/qhf.py:321-409` (QModel.forward / prefill: fused qkv and
  w13 rows, GQA, QK-norm, the chunk's K/V rows written before its attention);
- `compiler/frontend/hf_generic.py:231-293` (QSUM attention) and
  `compiler/frontend/hf_generic.py:641-657` (MoE router and combine).
All fp32 steps round once (NumPy float32), sums use the fixed D = 16 lane order,
EXP / RECIP / RSQRT are the SFU (`oracle.numerics`).

The KV cache is kept as the reference keeps it: int8 [layers, seq_len, kv_dim]
(`llm/ref_model.py:171-174`).
"""
import numpy as np

from . import numerics as N

F = np.float32


def attention_rows(q, kc, vc, positions, a_k, a_v, heads, kv_heads, head_dim, variant, k_scale=None):
    """Attention of rows q [M, heads*head_dim] (after QK-norm and RoPE) over one
    layer's int8 cache kc / vc [T, kv_heads*head_dim]; row m attends t <= positions[m].
    NORM: `llm/ref_model.py:233-243`; QSUM: `compiler/frontend/hf_generic.py:264-292`.
    Per cache channel scales (`hf_generic.py:241-246`, :290): k_scale
    [kv_heads*head_dim] multiplies each query head's channels (those of its KV
    head) before the query's quantization; a_v may be [kv_heads*head_dim]."""
    M = q.shape[0]
    G = heads // kv_heads
    per_q = lambda v: np.asarray(v, F).reshape(kv_heads, head_dim)[np.arange(heads) // G]   # [H, hd]
    av = per_q(a_v) if np.ndim(a_v) else F(a_v)
    out = np.empty((M, heads * head_dim), F)
    for m in range(M):
        n = int(positions[m]) + 1
        K = kc[:n].reshape(n, kv_heads, head_dim).astype(np.int64)
        V = vc[:n].reshape(n, kv_heads, head_dim).astype(np.int64)
        qh = q[m].reshape(heads, head_dim)
        if k_scale is not None:
            qh = (qh * per_q(k_scale)).astype(F)
        qq, s_q = N.quant_act(qh)                                         # [H, hd], [H]
        kh = K[:, np.arange(heads) // G, :]                                # [n, H, hd]
        acc = np.einsum("hd,thd->ht", qq.astype(np.int64), kh)            # [H, n] exact
        sc = ((acc.astype(F) * s_q[:, None]).astype(F) * F(a_k)).astype(F)
        mx = np.max(sc, axis=1, keepdims=True)
        e = N.sfu_exp((sc - mx).astype(F))
        vh = V[:, np.arange(heads) // G, :]                                # [n, H, hd]
        if variant == "norm":
            r = N.sfu_recip(N.red_sum_rows(e))
            pq = N.to_i8(((e * r[:, None]).astype(F) * F(127)).astype(F)).astype(np.int64)
            pv = np.einsum("ht,thd->hd", pq, vh)
            o = (pv.astype(F) * av).astype(F)
        else:
            eq = N.to_i8((e * F(127.0)).astype(F))
            pv = np.einsum("ht,thd->hd", eq.astype(np.int64), vh)
            ssum = eq.astype(np.int64).sum(axis=1).astype(F)              # exact: at most 127*T < 2^24
            rq = (N.sfu_recip(ssum) * F(127.0)).astype(F)
            o = ((pv.astype(F) * rq[:, None]).astype(F) * av).astype(F)
        out[m] = o.reshape(-1)
    return out


def attn_layer(cfg, qkv, pos, kc, vc, consts, cos_tab, sin_tab, q_norm=None, k_norm=None):
    """One layer's attention for rows qkv [M, q|k|v] at positions pos: QK-norm
    (`qhf.py:335-337`), RoPE, the rows' int8 K/V written into kc / vc
    [T, kv_dim] first (`llm/ref_model.py:228-229`), then attention_rows."""
    c = cfg
    M, H, Hk, hd = qkv.shape[0], c.heads, c.kv_heads, c.head_dim
    inv_sk, inv_sv, a_k, a_v = consts[:4]                               # (arrays: per cache channel)
    k_scale = consts[4] if len(consts) > 4 else None
    pos = np.asarray(pos, np.int64)
    cos, sin = cos_tab[pos], sin_tab[pos]
    q = qkv[:, :c.q_dim].reshape(M, H, hd)
    k = qkv[:, c.q_dim:c.q_dim + c.kv_dim].reshape(M, Hk, hd)
    v = qkv[:, c.q_dim + c.kv_dim:]
    if q_norm is not None:
        q = N.rmsnorm(q.reshape(M * H, hd), q_norm, c.eps).reshape(M, H, hd)
        k = N.rmsnorm(k.reshape(M * Hk, hd), k_norm, c.eps).reshape(M, Hk, hd)
    q = N.rope(q, cos[:, None, :], sin[:, None, :]).reshape(M, -1)
    k = N.rope(k, cos[:, None, :], sin[:, None, :]).reshape(M, -1)
    for m in range(M):
        kc[pos[m]] = N.to_i8((k[m] * inv_sk).astype(F))
        vc[pos[m]] = N.to_i8((v[m] * inv_sv).astype(F))
    return attention_rows(q, kc, vc, pos, a_k, a_v, H, Hk, hd, c.attn, k_scale)


def moe_ffn_row(x, t, cfg):
    """One row of the Mixtral-style MoE block (`hf_generic.QMixtralMoe.route` /
    `_row` :641-657): router W8A8 logits, Top-k (descending; ties -> lower id,
    `docs/moe_native_lowering_design.md:342-345`), w = e*RECIP(sum e) with
    e = EXP(v - v0) (sum in the D = 16 lane order), y = sum_k w_k*y_k folded
    left from 0 in k order; each expert a SwiGLU of W8A8 linears."""
    xq, s_x = N.quant_act(x[None])
    scores, _ = N.linear(xq, s_x, t["router"], t["s_router"])
    sc = scores[0]
    order = np.lexsort((np.arange(sc.size), -sc.astype(np.float64)))   # value desc, id asc
    ids = order[:cfg.top_k]
    v = sc[ids]
    e = N.sfu_exp((v - v[0]).astype(F))
    w = (e * N.sfu_recip(N.red_sum(e))).astype(F)
    y = np.zeros(cfg.dim, F)
    for k, i in enumerate(ids):
        g, _ = N.linear(xq, s_x, t["e_gate"][i], t["s_e_gate"][i])
        u, _ = N.linear(xq, s_x, t["e_up"][i], t["s_e_up"][i])
        hq, s_h = N.quant_act(N.silu_gate(g, u))
        yk, _ = N.linear(hq, s_h, t["e_down"][i], t["s_e_down"][i])
        y = (y + (w[k] * yk[0]).astype(F)).astype(F)
    return y, ids, w


class OracleDecoder:
    """The whole decoder for one sequence. qw: a `QuantWeights`-like object
    (emb_q/emb_s, cls_q/cls_s, rms_final, layers[l] dicts, cos/sin tables);
    kv_scales [layers, 2] (static per-layer K and V scales)."""

    def __init__(self, cfg, qw, kv_scales):
        """kv_scales: [layers, 2] per layer, or [layers, 2, kv_dim] per cache
        channel (`hf_generic.calibrate_kv(channel=...)`; a part whose row holds
        one value is per layer)."""
        self.cfg, self.qw = cfg, qw
        self.kv = np.asarray(kv_scales, F)
        self.consts = []
        for l in range(cfg.layers):
            self.consts.append(self.layer_consts(self.kv[l], cfg.head_dim))
        self._w64 = {}
        self.reset()

    @staticmethod
    def layer_consts(kv_l, hd):
        """(inv_sk, inv_sv, a_k, a_v, k_scale): per layer `llm/ref_model.py:230-231`
        and `llm/export_w8a8.py:68-72`; per channel `hf_generic.SaCache`
        (:153-187): K -- q * s_k before its quantization, F(1) / s_k into the
        cache, scores * F(1 / sqrt(hd)); V -- F(1) / s_v into the cache, the
        output * (s_v * F(1/127)) per channel."""
        if kv_l.ndim == 1:
            s_k, s_v = F(kv_l[0]), F(kv_l[1])
            return F(1.0 / s_k), F(1.0 / s_v), F(float(s_k) / np.sqrt(hd)), F(float(s_v) / 127.0), None
        s_k, s_v = F(kv_l[0, 0]), F(kv_l[1, 0])
        inv_sk, a_k, k_scale = F(1.0 / s_k), F(float(s_k) / np.sqrt(hd)), None
        inv_sv, a_v = F(1.0 / s_v), F(float(s_v) / 127.0)
        if np.any(kv_l[0] != s_k):
            inv_sk, a_k, k_scale = (F(1.0) / kv_l[0]).astype(F), F(1.0 / np.sqrt(hd)), kv_l[0].astype(F)
        if np.any(kv_l[1] != s_v):
            inv_sv, a_v = (F(1.0) / kv_l[1]).astype(F), (kv_l[1] * F(1.0 / 127.0)).astype(F)
        return inv_sk, inv_sv, a_k, a_v, k_scale

    def reset(self):
        c = self.cfg
        self.kc = np.zeros((c.layers, c.seq_len, c.kv_dim), np.int8)
        self.vc = np.zeros((c.layers, c.seq_len, c.kv_dim), np.int8)

    def _lin(self, xq, s_x, key, q, s):
        w = self._w64.get(key)
        if w is None:
            w = self._w64[key] = q.astype(np.float64)
        return N.linear_f64(xq, s_x, w, s)[0]

    def forward_rows(self, tokens, positions, all_logits=False, trace=None):
        """Rows of one sequence at positions (each row computed as a decode
        step); returns the last row's logits [vocab] (all rows' [M, vocab] with
        all_logits). trace: a dict that collects per-layer intermediates."""
        c, qw = self.cfg, self.qw
        tokens = np.asarray(tokens, np.int64)
        pos = np.asarray(positions, np.int64)
        M = tokens.size
        H, Hk, hd = c.heads, c.kv_heads, c.head_dim
        x = (qw.emb_q[tokens].astype(F) * qw.emb_s[tokens][:, None]).astype(F)
        for l in range(c.layers):
            t = qw.layers[l]
            xq, s_x = N.quant_act(N.rmsnorm(x, t["rms_att"], c.eps))
            qkv = self._lin(xq, s_x, ("qkv", l), t["wqkv"], t["s_wqkv"])
            att = attn_layer(c, qkv, pos, self.kc[l], self.vc[l], self.consts[l], qw.cos, qw.sin,
                             t.get("q_norm"), t.get("k_norm"))
            aq, s_a = N.quant_act(att)
            x = (x + self._lin(aq, s_a, ("wo", l), t["wo"], t["s_wo"])).astype(F)
            xn = N.rmsnorm(x, t["rms_ffn"], c.eps)
            if c.moe:
                y = np.stack([moe_ffn_row(xn[m], t, c)[0] for m in range(M)])
                x = (x + y).astype(F)
            else:
                xq, s_x = N.quant_act(xn)
                h1 = self._lin(xq, s_x, ("w1", l), t["w1"], t["s_w1"])
                h3 = self._lin(xq, s_x, ("w3", l), t["w3"], t["s_w3"])
                hq, s_h = N.quant_act(N.gate(h1, h3, getattr(c, "act", "silu")))
                x = (x + self._lin(hq, s_h, ("w2", l), t["w2"], t["s_w2"])).astype(F)
            if trace is not None:
                trace.setdefault("x", []).append(x.copy())
                trace.setdefault("att", []).append(att.copy())
        rows = x if all_logits else x[-1:]
        xq, s_x = N.quant_act(N.rmsnorm(rows, qw.rms_final, c.eps))
        logits = self._lin(xq, s_x, ("cls",), qw.cls_q, qw.cls_s)
        return logits if all_logits else logits[0]

    def forward(self, token, pos):
        return self.forward_rows([token], [pos])

    def cache_rows(self, layer, n):
        """K, V int8 [n, kv_dim] of a layer (the reference's layout)."""
        return self.kc[layer, :n], self.vc[layer, :n]


def rope_tables(cfg):
    """(cos, sin) [seq_len, head_dim], pair-repeated. "llama2c":
    `llm/ref_model.py:34-41`; "hf": `compiler/frontend/qhf.py:183-189`."""
    hs = cfg.head_dim
    if cfg.rope == "llama2c":
        hd = np.arange(0, hs, 2).astype(F)
        freq = F(1.0) / np.power(F(cfg.theta), hd / F(hs))
        val = np.arange(cfg.seq_len, dtype=F)[:, None] * freq[None, :]
    else:
        freq = 1.0 / np.power(cfg.theta, np.arange(0, hs, 2, dtype=np.float64) / hs)
        val = np.arange(cfg.seq_len, dtype=np.float64)[:, None] * freq[None, :]
    return np.repeat(np.cos(val).astype(F), 2, axis=1), np.repeat(np.sin(val).astype(F), 2, axis=1)


class QW:
    """Quantized weights as the oracle holds them."""


def quantize_model(cfg, w):
    """fp32 weights in the reference's naming (`llm/checkpoint.py:33-59`: tok,
    rms_att, wq, wk, wv, wo, rms_ffn, w1, w2, w3, rms_final, wcls; plus q_norm /
    k_norm) -> QW, quantized per output row as `llm/ref_model.py:157-166` and
    `compiler/frontend/qhf.py:262-281` do."""
    qw = QW()
    qw.emb_q, qw.emb_s = N.quantize_rows(w["tok"])
    wcls = w.get("wcls", w["tok"])
    qw.cls_q, qw.cls_s = N.quantize_rows(wcls)
    qw.rms_final = np.asarray(w["rms_final"], F)
    qw.layers = []
    for l in range(cfg.layers):
        t = {"rms_att": np.asarray(w["rms_att"][l], F), "rms_ffn": np.asarray(w["rms_ffn"][l], F)}
        t["wqkv"], t["s_wqkv"] = N.quantize_rows(np.concatenate([w["wq"][l], w["wk"][l], w["wv"][l]]))
        t["wo"], t["s_wo"] = N.quantize_rows(w["wo"][l])
        for n in ("w1", "w2", "w3"):
            t[n], t["s_" + n] = N.quantize_rows(w[n][l])
        if cfg.qk_norm:
            t["q_norm"], t["k_norm"] = np.asarray(w["q_norm"][l], F), np.asarray(w["k_norm"][l], F)
        qw.layers.append(t)
    qw.cos, qw.sin = rope_tables(cfg)
    return qw
