"""One rank of the tensor-parallel decoder restated on the CPU (test helper).

The oracle's per-row program (`oracle/model.py` OracleDecoder.forward_rows)
over the shard `torch2riscv_accelerator_b200.tp.shard` gives this rank, with the
two cross-rank steps as torch.distributed collectives: max|x| of a
column-split activation (all-reduce MAX), the int32 partials of a row-split
linear (all-reduce SUM), and the classifier's vocabulary slices (all-gather).
The GPU path does the same exchanges inside its kernels; both must equal the
unsharded oracle bit for bit.
"""
import numpy as np
import torch
import torch.distributed as dist

from oracle import model as OM
from oracle import numerics as N
from torch2riscv_accelerator_b200.tp import local_config, shard

F = np.float32


def quant_with(x, amax):
    """quant_act with a given max|x| per row (`llm/ref_model.py:191-196`)."""
    s = (np.asarray(amax, F)[..., None] * N.C127).astype(F)
    inv = N.sfu_recip(s)
    with np.errstate(invalid="ignore"):
        return N.to_i8((x * inv).astype(F)), s[..., 0]


def all_max(a):
    t = torch.from_numpy(np.ascontiguousarray(a, F))
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.numpy()


def all_sum_i32(acc):
    t = torch.from_numpy(np.ascontiguousarray(acc).astype(np.int32))
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.numpy().astype(np.int64)


class TpOracle(OM.OracleDecoder):
    def __init__(self, cfg, qw, kv_scales, rank, ranks):
        self.full_cfg, self.rank, self.ranks = cfg, rank, ranks
        super().__init__(local_config(cfg, ranks), shard(cfg, qw, rank, ranks), kv_scales)

    def forward_rows(self, tokens, positions, all_logits=False, trace=None):
        c, fc, sh = self.cfg, self.full_cfg, self.qw
        tokens = np.asarray(tokens, np.int64)
        pos = np.asarray(positions, np.int64)
        x = (sh.emb_q[tokens].astype(F) * sh.emb_s[tokens][:, None]).astype(F)

        def row_split(a, w, s_w):
            aq, s_a = quant_with(a, all_max(np.max(np.abs(a), axis=-1)))
            _, acc = N.linear(aq, s_a, w, s_w)
            acc = all_sum_i32(acc)
            return ((acc.astype(F) * s_w).astype(F) * s_a[:, None]).astype(F)

        for l in range(fc.layers):
            t = sh.layers[l]
            xq, s_x = N.quant_act(N.rmsnorm(x, t["rms_att"], fc.eps))
            qkv, _ = N.linear(xq, s_x, t["wqkv"], t["s_wqkv"])
            att = OM.attn_layer(c, qkv, pos, self.kc[l], self.vc[l], self.consts[l], sh.cos, sh.sin,
                                t.get("q_norm"), t.get("k_norm"))
            x = (x + row_split(att, t["wo"], t["s_wo"])).astype(F)
            xq, s_x = N.quant_act(N.rmsnorm(x, t["rms_ffn"], fc.eps))
            h1, _ = N.linear(xq, s_x, t["w1"], t["s_w1"])
            h3, _ = N.linear(xq, s_x, t["w3"], t["s_w3"])
            x = (x + row_split(N.silu_gate(h1, h3), t["w2"], t["s_w2"])).astype(F)
        rows = x if all_logits else x[-1:]
        xq, s_x = N.quant_act(N.rmsnorm(rows, sh.rms_final, fc.eps))
        part, _ = N.linear(xq, s_x, sh.cls_q, sh.cls_s)
        out = [torch.empty(part.shape, dtype=torch.float32) for _ in range(self.ranks)]
        dist.all_gather(out, torch.from_numpy(np.ascontiguousarray(part)))
        logits = np.concatenate([o.numpy() for o in out], axis=-1)
        return logits if all_logits else logits[0]


def moe_ep_row(x, t, cfg, lo, n):
    """One row of the MoE FFN as an expert-parallel rank computes it: the router
    whole, the terms w_j * y_j of the slots whose expert is in [lo, lo + n)
    (+0 for the others), summed over the ranks, then the k-order fold
    (`oracle/model.py` moe_ffn_row, split by expert)."""
    xq, s_x = N.quant_act(x[None])
    scores, _ = N.linear(xq, s_x, t["router"], t["s_router"])
    sc = scores[0]
    ids = np.lexsort((np.arange(sc.size), -sc.astype(np.float64)))[:cfg.top_k]
    v = sc[ids]
    e = N.sfu_exp((v - v[0]).astype(F))
    w = (e * N.sfu_recip(N.red_sum(e))).astype(F)
    terms = np.zeros((cfg.top_k, cfg.dim), F)
    for k, i in enumerate(ids):
        if not lo <= i < lo + n:
            continue
        g, _ = N.linear(xq, s_x, t["e_gate"][i], t["s_e_gate"][i])
        u, _ = N.linear(xq, s_x, t["e_up"][i], t["s_e_up"][i])
        hq, s_h = N.quant_act(N.silu_gate(g, u))
        yk, _ = N.linear(hq, s_h, t["e_down"][i], t["s_e_down"][i])
        terms[k] = (w[k] * yk[0]).astype(F)
    tt = torch.from_numpy(terms)
    dist.all_reduce(tt, op=dist.ReduceOp.SUM)
    y = np.zeros(cfg.dim, F)
    for k in range(cfg.top_k):
        y = (y + tt.numpy()[k]).astype(F)
    return y
