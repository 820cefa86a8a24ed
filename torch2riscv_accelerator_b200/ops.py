"""The operator surface on CUDA tensors, one function per C-ABI entry point.

Names and argument meanings follow the reference's operators
(`llm/ref_model.py` DeviceModel: quant_act, linear, rmsnorm; `llm/compile_model.py`
ModelCompiler: embed, attention, ffn_up; `llm/runtime.py` Sampler). Every call
runs on the current torch CUDA stream and raises W8A8Error on a nonzero status.
Tensors are passed as raw device pointers; torch only owns the memory.
"""
import ctypes

import numpy as np
import torch

from . import _lib

F32, I8, I32 = torch.float32, torch.int8, torch.int32
SFU_EXP, SFU_RECIP, SFU_RSQRT, SFU_SILU, SFU_GELU = 0, 1, 2, 3, 4
ACTS = {"silu": 0, "gelu_tanh": 1}


def _p(t):
    return None if t is None else t.data_ptr()


def _st():
    return torch.cuda.current_stream().cuda_stream


def _need(t, dtype, name):
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous():
        raise ValueError(f"{name}: a contiguous CUDA {dtype} tensor is required, got {t.dtype} on {t.device}")


def sfu(func, x, out=None):
    _need(x, F32, "x")
    out = torch.empty_like(x) if out is None else out
    _lib.check("w8a8_sfu", _lib.load().w8a8_sfu(func, _p(x), _p(out), x.numel(), _st()))
    return out


def quant_act(x):
    """x [rows, k] fp32 -> (xq int8 [rows, k], s_x [rows])."""
    _need(x, F32, "x")
    x2 = x.reshape(-1, x.shape[-1])
    xq = torch.empty(x2.shape, dtype=I8, device=x.device)
    s = torch.empty(x2.shape[0], dtype=F32, device=x.device)
    _lib.check("w8a8_quant_act", _lib.load().w8a8_quant_act(_p(x2), x2.shape[0], x2.shape[1], _p(xq), _p(s), _st()))
    return xq.reshape(x.shape), s


def rmsnorm(x, g, eps):
    _need(x, F32, "x")
    x2 = x.reshape(-1, x.shape[-1])
    y = torch.empty_like(x2)
    _lib.check("w8a8_rmsnorm", _lib.load().w8a8_rmsnorm(_p(x2), _p(g), x2.shape[0], x2.shape[1], float(eps), _p(y),
                                                       _st()))
    return y.reshape(x.shape)


def embed(tokens, emb_q, emb_s, out=None):
    m, (vocab, dim) = tokens.numel(), emb_q.shape
    out = torch.empty(m, dim, dtype=F32, device=emb_q.device) if out is None else out
    _lib.check("w8a8_embed", _lib.load().w8a8_embed(_p(tokens), m, _p(emb_q), _p(emb_s), vocab, dim, _p(out),
                                                   _st()))
    return out


def error_flags():
    """Read and clear the device error flags (bit 0: an out-of-range token)."""
    v = ctypes.c_uint32(0)
    _lib.check("w8a8_error_flags", _lib.load().w8a8_error_flags(ctypes.byref(v)))
    return v.value


def linear(xq, s_x, w, s_w, out=None, acc=None, resid=None):
    """W8A8 linear on int8 rows: y = (f32(xq . W^T) * s_w) * s_x [+ resid]."""
    _need(xq, I8, "xq")
    _need(w, I8, "w")
    m, k = xq.shape
    n = w.shape[0]
    out = torch.empty(m, n, dtype=F32, device=w.device) if out is None else out
    _lib.check("w8a8_linear", _lib.load().w8a8_linear(_p(xq), _p(s_x), m, k, _p(w), _p(s_w), n, _p(resid), _p(out),
                                                     _p(acc), _st()))
    return out


def linear_fused(x, w, s_w, norm_g=None, eps=0.0, resid=None, out=None, s_x_out=None):
    """[rmsnorm ->] quant_act -> linear [-> + resid] on fp32 rows x [m, k]."""
    _need(x, F32, "x")
    _need(w, I8, "w")
    m, k = x.shape
    n = w.shape[0]
    out = torch.empty(m, n, dtype=F32, device=w.device) if out is None else out
    _lib.check("w8a8_linear_fused", _lib.load().w8a8_linear_fused(
        _p(x), _p(norm_g), float(eps), m, k, _p(w), _p(s_w), n, _p(resid), _p(out), _p(s_x_out), _st()))
    return out


def linear_chain(x, w, s_w, norm_g=None, eps=0.0, x_amax=None, resid=None, out=None, clear=None):
    """The decode chain's fused linear: quant_act(x) with max|x| posted by the
    producer (x_amax), or rmsnorm + quant_act; `clear` zeroed after the wait."""
    _need(x, F32, "x")
    m, k = x.shape
    n = w.shape[0]
    out = torch.empty(m, n, dtype=F32, device=x.device) if out is None else out
    _lib.check("w8a8_linear_chain", _lib.load().w8a8_linear_chain(
        _p(x), _p(norm_g), float(eps), _p(x_amax), m, k, _p(w), _p(s_w), n, _p(resid), _p(out), _p(clear),
        0 if clear is None else clear.numel(), _st()))
    return out


def ffn_swiglu_chain(x, norm_g, eps, w_gate, s_gate, w_up, s_up, h, h_amax, clear=None):
    """The decode chain's SwiGLU: h and max|h| per row posted into h_amax."""
    m, k = x.shape
    _lib.check("w8a8_ffn_swiglu_chain", _lib.load().w8a8_ffn_swiglu_chain(
        _p(x), _p(norm_g), float(eps), m, k, _p(w_gate), _p(s_gate), _p(w_up), _p(s_up), w_gate.shape[0], _p(h),
        _p(h_amax), _p(clear), 0 if clear is None else clear.numel(), _st()))
    return h


def ffn_scratch(rows, device):
    n = _lib.load().w8a8_ffn_scratch_bytes(rows)
    return torch.zeros(n, dtype=torch.uint8, device=device)


def ffn_swiglu(x, norm_g, eps, w_gate, s_gate, w_up, s_up, scratch, h=None, h_q=None, s_h=None, requant=True,
               act="silu"):
    """Decode SwiGLU dispatch: returns (h fp32, h_q int8, s_h); with
    requant=False only h (h_q, s_h None; the down projection quantizes h).
    act: the gate, "silu" or "gelu_tanh"."""
    _need(x, F32, "x")
    m, k = x.shape
    hidden = w_gate.shape[0]
    dev = x.device
    h = torch.empty(m, hidden, dtype=F32, device=dev) if h is None else h
    if requant:
        h_q = torch.empty(m, hidden, dtype=I8, device=dev) if h_q is None else h_q
        s_h = torch.empty(m, dtype=F32, device=dev) if s_h is None else s_h
    else:
        h_q = s_h = scratch = None
    _lib.check("w8a8_ffn_gated", _lib.load().w8a8_ffn_gated(
        _p(x), _p(norm_g), float(eps), m, k, _p(w_gate), _p(s_gate), _p(w_up), _p(s_up), hidden, ACTS[act], _p(h),
        _p(h_q), _p(s_h), _p(scratch), 0 if scratch is None else scratch.numel(), _st()))
    return h, h_q, s_h


def quant_rows(x, norm_g=None, eps=0.0, xq=None, s_x=None):
    """int8 rows and scales of x (quant_act, after rmsnorm when norm_g is given)."""
    _need(x, F32, "x")
    m, k = x.shape
    xq = torch.empty(m, k, dtype=I8, device=x.device) if xq is None else xq
    s_x = torch.empty(m, dtype=F32, device=x.device) if s_x is None else s_x
    _lib.check("w8a8_quant_rows", _lib.load().w8a8_quant_rows(_p(x), _p(norm_g), float(eps), m, k, _p(xq), _p(s_x),
                                                              _st()))
    return xq, s_x


def gemm(xq, s_x, w, s_w, out=None, acc=None, resid=None):
    """Tensor-core W8A8 linear for any row count (same results as linear())."""
    m, k = xq.shape
    n = w.shape[0]
    out = torch.empty(m, n, dtype=F32, device=xq.device) if out is None else out
    _lib.check("w8a8_gemm", _lib.load().w8a8_gemm(_p(xq), _p(s_x), m, k, _p(w), _p(s_w), n, _p(resid), _p(out),
                                                  _p(acc), _st()))
    return out


def gemm_swiglu(xq, s_x, w_gate, s_gate, w_up, s_up, out=None, act="silu"):
    """Tensor-core gated pair: h = act(g) * u for any row count (act "silu"
    or "gelu_tanh")."""
    m, k = xq.shape
    n = w_gate.shape[0]
    out = torch.empty(m, n, dtype=F32, device=xq.device) if out is None else out
    _lib.check("w8a8_gemm_gated", _lib.load().w8a8_gemm_gated(_p(xq), _p(s_x), m, k, _p(w_gate), _p(s_gate),
                                                              _p(w_up), _p(s_up), n, ACTS[act], _p(out), _st()))
    return out


def moe_scratch(rows, dim, top_k, expert_hidden, device):
    n = _lib.load().w8a8_moe_scratch_bytes(rows, dim, top_k, expert_hidden)
    return torch.zeros(n, dtype=torch.uint8, device=device)


def moe_ffn(x, norm_g, eps, router_q, router_s, top_k, gate_q, gate_s, up_q, up_s, down_q, down_s, scratch,
            resid=None, out=None, ids=None, w=None):
    """MoE FFN rows (hf_generic.QMixtralMoe): returns (y = resid + moe(rmsnorm(x)),
    ids [rows, top_k] int32, w [rows, top_k] fp32). resid defaults to x; out may
    be resid (in place)."""
    _need(x, F32, "x")
    m, dim = x.shape
    experts, ih = router_q.shape[0], gate_q.shape[1]
    dev = x.device
    resid = x if resid is None else resid
    out = torch.empty(m, dim, dtype=F32, device=dev) if out is None else out
    ids = torch.empty(m, top_k, dtype=torch.int32, device=dev) if ids is None else ids
    w = torch.empty(m, top_k, dtype=F32, device=dev) if w is None else w
    _lib.check("w8a8_moe_ffn", _lib.load().w8a8_moe_ffn(
        _p(x), _p(norm_g), float(eps), m, dim, _p(router_q), _p(router_s), experts, top_k, _p(gate_q), _p(gate_s),
        _p(up_q), _p(up_s), ih, _p(down_q), _p(down_s), _p(resid), _p(out), _p(ids), _p(w), _p(scratch),
        scratch.numel(), _st()))
    return out, ids, w


def moe_ffn_ep(x, norm_g, eps, router_q, router_s, top_k, expert_lo, gate_q, gate_s, up_q, up_s, down_q, down_s,
               scratch, wy, ids, w):
    """Expert parallelism: the MoE FFN rows over this rank's experts
    [expert_lo, expert_lo + gate_q.shape[0]); wy [rows, top_k, dim] receives
    w_j * y_j of their slots and +0 for the others."""
    _need(x, F32, "x")
    m, dim = x.shape
    experts, (local, ih) = router_q.shape[0], gate_q.shape[:2]
    _lib.check("w8a8_moe_ffn_ep", _lib.load().w8a8_moe_ffn_ep(
        _p(x), _p(norm_g), float(eps), m, dim, _p(router_q), _p(router_s), experts, top_k, int(expert_lo), local,
        _p(gate_q), _p(gate_s), _p(up_q), _p(up_s), ih, _p(down_q), _p(down_s), _p(wy), _p(ids), _p(w),
        _p(scratch), scratch.numel(), _st()))
    return wy


MOE_MAX_ROWS = 4096


def moe_rows_scratch(rows, dim, experts, top_k, expert_hidden, device):
    n = _lib.load().w8a8_moe_rows_scratch_bytes(rows, dim, experts, top_k, expert_hidden)
    return torch.zeros(n, dtype=torch.uint8, device=device)


def moe_ffn_rows(x, norm_g, eps, router_q, router_s, top_k, gate_q, gate_s, up_q, up_s, down_q, down_s, scratch,
                 resid=None, out=None, ids=None, w=None, expert_lo=0, wy=None):
    """moe_ffn (wy None) or moe_ffn_ep (wy given, expert_lo: this rank's first
    expert) for many rows at once, the pairs grouped by expert; scratch from
    moe_rows_scratch."""
    _need(x, F32, "x")
    m, dim = x.shape
    experts, (local, ih) = router_q.shape[0], gate_q.shape[:2]
    dev = x.device
    if wy is None:
        resid = x if resid is None else resid
        out = torch.empty(m, dim, dtype=F32, device=dev) if out is None else out
    ids = torch.empty(m, top_k, dtype=torch.int32, device=dev) if ids is None else ids
    w = torch.empty(m, top_k, dtype=F32, device=dev) if w is None else w
    _lib.check("w8a8_moe_ffn_rows", _lib.load().w8a8_moe_ffn_rows(
        _p(x), _p(norm_g), float(eps), m, dim, _p(router_q), _p(router_s), experts, top_k, int(expert_lo), local,
        _p(gate_q), _p(gate_s), _p(up_q), _p(up_s), ih, _p(down_q), _p(down_s), _p(resid), _p(out), _p(wy),
        _p(ids), _p(w), _p(scratch), scratch.numel(), _st()))
    return (out if wy is None else wy), ids, w


def moe_combine(wy, resid, out):
    """out = resid + the k-order fold of wy [rows, top_k, dim]."""
    m, k, dim = wy.shape
    _lib.check("w8a8_moe_combine", _lib.load().w8a8_moe_combine(_p(wy), m, k, dim, _p(resid), _p(out), _st()))
    return out


def attn_scratch(rows, heads, kv_heads, head_dim, seq_len, device):
    n = _lib.load().w8a8_attn_scratch_bytes(rows, heads, kv_heads, head_dim, seq_len)
    return torch.zeros(n, dtype=torch.uint8, device=device)


VARIANTS = {"norm": 0, "qsum": 1}


def attn_args(cfg, rows, pos, qkv, kc, vc, att, consts, cos, sin, scratch, q_norm=None, k_norm=None, att_amax=None,
              ch=None):
    """The W8A8AttnArgs block of one layer (kept alive by the caller: a CUDA
    graph replays the pointers it captured). ch: the per-channel KV constants
    (device tensors k_scale / inv_sk_ch, inv_sv_ch / a_v_ch) or None."""
    inv_sk, inv_sv, a_k, a_v = consts
    ch = ch or {}
    return _lib.W8A8AttnArgs(
        rows=rows, heads=cfg.heads, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim, seq_len=cfg.seq_len,
        variant=VARIANTS[cfg.attn], pos=_p(pos), qkv=_p(qkv), q_norm=_p(q_norm), k_norm=_p(k_norm),
        eps=float(np.float32(cfg.eps)), rope_cos=_p(cos), rope_sin=_p(sin), inv_sk=float(inv_sk),
        inv_sv=float(inv_sv), a_k=float(a_k), a_v=float(a_v), k_cache=_p(kc), v_cache=_p(vc), att=_p(att),
        scratch=_p(scratch), scratch_bytes=scratch.numel(), att_amax=_p(att_amax), k_scale=_p(ch.get("k_scale")),
        inv_sk_ch=_p(ch.get("inv_sk_ch")), inv_sv_ch=_p(ch.get("inv_sv_ch")), a_v_ch=_p(ch.get("a_v_ch")))


def attn(args):
    import ctypes
    _lib.check("w8a8_attn", _lib.load().w8a8_attn(ctypes.byref(args), _st()))


def kv_append(args):
    """Every row's K / V (args.rows rows, any number) into the cache."""
    _lib.check("w8a8_kv_append", _lib.load().w8a8_kv_append(ctypes.byref(args), _st()))


def attn_prefill(args):
    """The attention of all args.rows rows (their K / V appended before) in one launch."""
    _lib.check("w8a8_attn_prefill", _lib.load().w8a8_attn_prefill(ctypes.byref(args), _st()))


def attn_batch(args, slots, slot_stride):
    """Batched decode attention: slot b = row b of pos / qkv / att, caches at
    + b * slot_stride bytes (args built for one row and slot 0's caches)."""
    import ctypes
    _lib.check("w8a8_attn_batch", _lib.load().w8a8_attn_batch(ctypes.byref(args), slots, slot_stride, _st()))


def argmax(logits, out=None):
    m, n = logits.reshape(-1, logits.shape[-1]).shape
    out = torch.empty(m, dtype=I32, device=logits.device) if out is None else out
    _lib.check("w8a8_argmax", _lib.load().w8a8_argmax(_p(logits), m, n, _p(out), _st()))
    return out


def classifier(x, w, s_w, norm_g, eps, out=None, argmax_key=None):
    """Final rmsnorm -> quant_act -> classifier GEMV [+ fused greedy argmax key]."""
    _need(x, F32, "x")
    m, k = x.shape
    n = w.shape[0]
    out = torch.empty(m, n, dtype=F32, device=w.device) if out is None else out
    _lib.check("w8a8_classifier", _lib.load().w8a8_classifier(
        _p(x), _p(norm_g), float(eps), m, k, _p(w), _p(s_w), n, _p(out), _p(argmax_key), _st()))
    return out


def key_token(key):
    """The token index packed in an argmax key (host side)."""
    return 0xFFFFFFFF - (int(key) & 0xFFFFFFFF)


def decode_advance(tokens, pos, argmax_key, rows, next_token=None):
    _lib.check("w8a8_decode_advance", _lib.load().w8a8_decode_advance(
        _p(tokens), _p(pos), _p(argmax_key), _p(next_token), rows, _st()))


# ------------------------------------------------------------- tensor parallel
def tp_embed(comm, tokens, emb_q, emb_s, out):
    """w8a8_embed that also starts a tensor-parallel step (advances the epoch)."""
    m, (vocab, dim) = tokens.numel(), emb_q.shape
    _lib.check("w8a8_tp_embed", _lib.load().w8a8_tp_embed(ctypes.byref(comm), _p(tokens), m, _p(emb_q), _p(emb_s),
                                                         vocab, dim, _p(out), _st()))
    return out


def tp_linear(args):
    """One decode GEMV of a rank's shard (a prepared W8A8TpLinearArgs)."""
    _lib.check("w8a8_tp_linear", _lib.load().w8a8_tp_linear(ctypes.byref(args), _st()))


def tp_attn(args, comm, amax_out):
    _lib.check("w8a8_tp_attn", _lib.load().w8a8_tp_attn(ctypes.byref(args), ctypes.byref(comm), amax_out, _st()))


def tp_advance(comm, keys, tokens, pos, rows, next_token=None):
    _lib.check("w8a8_tp_advance", _lib.load().w8a8_tp_advance(ctypes.byref(comm), keys, _p(tokens), _p(pos),
                                                             _p(next_token), rows, _st()))


def tp_seed(comm, keys, token):
    _lib.check("w8a8_tp_seed", _lib.load().w8a8_tp_seed(ctypes.byref(comm), keys, int(token), _st()))


def tp_moe_ffn(comm, x, norm_g, eps, router_q, router_s, top_k, expert_lo, gate_q, gate_s, up_q, up_s, down_q,
               down_s, scratch, terms, ids, w):
    """Expert parallelism over the exchange: the terms of this rank's experts'
    slots into every rank's `terms` block (decode rows)."""
    _need(x, F32, "x")
    m, dim = x.shape
    experts, (local, ih) = router_q.shape[0], gate_q.shape[:2]
    _lib.check("w8a8_tp_moe_ffn", _lib.load().w8a8_tp_moe_ffn(
        ctypes.byref(comm), _p(x), _p(norm_g), float(eps), m, dim, _p(router_q), _p(router_s), experts, top_k,
        int(expert_lo), local, _p(gate_q), _p(gate_s), _p(up_q), _p(up_s), ih, _p(down_q), _p(down_s), terms,
        _p(ids), _p(w), _p(scratch), scratch.numel(), _st()))


def tp_moe_combine(comm, terms, rows, top_k, resid, out):
    dim = resid.shape[-1]
    _lib.check("w8a8_tp_moe_combine", _lib.load().w8a8_tp_moe_combine(ctypes.byref(comm), terms, rows, top_k, dim,
                                                                     _p(resid), _p(out), _st()))
    return out


def row_amax(x, out):
    """max|x| per row as float bits (int32 tensor [rows])."""
    m, k = x.shape
    _lib.check("w8a8_row_amax", _lib.load().w8a8_row_amax(_p(x), m, k, _p(out), _st()))
    return out


def quant_rows_posted(x, amax, xq, s_x):
    """quant_act of x rows with the given max|x| bits."""
    m, k = x.shape
    _lib.check("w8a8_quant_rows_posted", _lib.load().w8a8_quant_rows_posted(_p(x), _p(amax), m, k, _p(xq), _p(s_x),
                                                                           _st()))
    return xq, s_x


def dequant_resid(acc, s_x, s_w, out, resid=None):
    """out = [resid +] (f32(acc) * s_w) * s_x over int32 rows acc [rows, n]."""
    m, n = acc.shape
    _lib.check("w8a8_dequant_resid", _lib.load().w8a8_dequant_resid(_p(acc), _p(s_x), _p(s_w), m, n, _p(resid),
                                                                   _p(out), _st()))
    return out

