"""The W8A8 decoder as a program of kernel launches on one GPU.

The B200 counterpart of the overlay's static descriptor list
(`llm/compile_model.py:351-374` ModelCompiler.build): built once per model,
run once per token (or per 16-row prefill chunk), optionally captured as a CUDA
graph so that only the (pos, token) inputs change between runs, as only the
PARAM block and the argument block change between the reference's submits
(`llm/compile_model.py:56-62`).

HBM layout (all resident):
- linear weights int8 row-major [out, in] (K contiguous: each output channel
  one 16-byte aligned run), fp32 scales [out]; q|k|v rows fused (wqkv), gate
  and up rows separate (the SwiGLU kernel reads both for the same channel);
- the embedding int8 [vocab, dim] + fp32 [vocab], shared with a tied
  classifier;
- KV cache int8: K [layers, kv_heads, seq_len, head_dim] (a position's row
  contiguous), V transposed [layers, kv_heads, head_dim, seq_len] (a channel's
  positions contiguous: p.V is a dot product over positions);
- RoPE tables fp32 [seq_len, head_dim], pair-repeated.
Per layer and row: 1 fused rmsnorm+quant+GEMV (wqkv), 1 attention kernel,
1 quant+GEMV+residual (wo), 1 rmsnorm+quant+gate/up GEMV+SiLU kernel, 1
quant+GEMV+residual (w2, quantizing h in its prologue).
"""
import numpy as np
import torch

from . import ops
from .weights import layer_kv_consts

I8, F32, I32 = torch.int8, torch.float32, torch.int32
CHUNK = 16                                         # rows of the GEMV / attention path (the reference's M)
PREFILL = 256                                      # rows per tensor-core prefill chunk
CHAIN_ROWS = 4                                     # rows of the decode GEMV path (the latency chain)


def _upload(obj, cfg, qw, kv_scales, kv_cols=None):
    """The model's tensors in HBM (int8 rows + fp32 scales, gains, RoPE tables)
    and the per-layer KV constants, as attributes of obj. kv_cols: the cache
    channels this decoder holds (a shard's KV heads) of per-channel scales; the
    constants come from the whole row (whether a layer is per channel is the
    whole model's), then the channels are sliced."""
    t = lambda a, dt=None: torch.as_tensor(np.ascontiguousarray(a), dtype=dt).to(obj.dev)
    obj.emb_q, obj.emb_s = t(qw.emb_q, I8), t(qw.emb_s, F32)
    if cfg.tied and qw.cls_q is qw.emb_q:
        obj.cls_q, obj.cls_s = obj.emb_q, obj.emb_s
    else:
        obj.cls_q, obj.cls_s = t(qw.cls_q, I8), t(qw.cls_s, F32)
    obj.rms_final = t(qw.rms_final, F32)
    obj.cos, obj.sin = t(qw.cos, F32), t(qw.sin, F32)
    obj.layers = [{k: t(v) for k, v in lw.items()} for lw in qw.layers]
    kv = np.asarray(kv_scales, np.float32)
    cols = kv_cols if kv_cols is not None else slice(0, cfg.kv_dim)
    if kv.shape[:2] != (cfg.layers, 2) or (kv.ndim == 3 and len(range(kv.shape[2])[cols]) != cfg.kv_dim):
        raise ValueError(f"KV scales {kv.shape}: [layers, 2] or [layers, 2, kv_dim] expected")
    both = [layer_kv_consts(kv[l], cfg.head_dim) for l in range(cfg.layers)]
    obj.consts = [c for c, _ in both]
    obj.kv_ch = [None if ch is None else {k: t(v[cols], F32) for k, v in ch.items()} for _, ch in both]


class DeviceDecoder:
    def __init__(self, cfg, qw, kv_scales, device="cuda", max_rows=CHUNK, prefill_rows=PREFILL, kv_cols=None):
        cfg.validate()
        self.cfg, self.dev, self.max_rows = cfg, torch.device(device), max_rows
        _upload(self, cfg, qw, kv_scales, kv_cols)
        L, Hk, T, hd = cfg.layers, cfg.kv_heads, cfg.seq_len, cfg.head_dim
        self.kc = torch.zeros(L, Hk, T, hd, dtype=I8, device=self.dev)
        self.vc = torch.zeros(L, Hk, hd, T, dtype=I8, device=self.dev)      # V transposed per head
        R = max(max_rows, prefill_rows)
        self.rows_cap = R
        z = lambda *s, dt=F32: torch.zeros(*s, dtype=dt, device=self.dev)
        self.tokens, self.pos = z(R, dt=I32), z(R, dt=I32)
        self.x, self.qkv, self.att = z(R, cfg.dim), z(R, cfg.qkv_dim), z(R, cfg.q_dim)
        self.h, self.hq, self.s_h = z(R, cfg.hidden), z(R, cfg.hidden, dt=I8), z(R)
        self.logits = z(max_rows, cfg.vocab)
        # int8 rows and scales between the row quantizer and the tensor-core GEMMs
        self.xq_buf = z(R * max(cfg.dim, cfg.q_dim, cfg.hidden), dt=I8)
        self.sx_buf = z(R)
        # decode chain: max|att| and max|h| per layer and row (int32 words holding
        # float bits; zero between uses)
        self.amax_att = z(cfg.layers, CHAIN_ROWS, dt=I32)
        self.amax_h = z(cfg.layers, CHAIN_ROWS, dt=I32)
        self.next_token = z(R, dt=I32)
        self.key = z(R, dt=torch.int64)                # packed greedy argmax per row (classifier epilogue)
        self.attn_scratch = ops.attn_scratch(R, cfg.heads, cfg.kv_heads, hd, T, self.dev)
        self.ffn_scratch = ops.ffn_scratch(R, self.dev)
        if cfg.moe:                                # routing of the last run (per layer) and the MoE scratch
            self.moe_ids = z(cfg.layers, R, cfg.top_k, dt=I32)
            self.moe_w = z(cfg.layers, R, cfg.top_k)
            self.moe_scratch = ops.moe_scratch(CHUNK, cfg.dim, cfg.top_k, cfg.expert_hidden, self.dev)
            self.moe_rows_scratch = (ops.moe_rows_scratch(R, cfg.dim, cfg.experts, cfg.top_k, cfg.expert_hidden,
                                                          self.dev) if R > CHUNK and cfg.dim % 32 == 0 else None)
        self._args = {}
        self._sub_args = {}
        self.graphs = {}

    # ------------------------------------------------------------ the program
    def _attn_args(self, rows, chain=False):
        a = self._args.get((rows, chain))
        if a is None:
            c = self.cfg
            a = self._args[(rows, chain)] = [
                ops.attn_args(c, rows, self.pos, self.qkv, self.kc[l], self.vc[l], self.att, self.consts[l],
                              self.cos, self.sin, self.attn_scratch, self.layers[l].get("q_norm"),
                              self.layers[l].get("k_norm"), att_amax=self.amax_att[l] if chain else None,
                              ch=self.kv_ch[l])
                for l in range(c.layers)]
        return a

    def run(self, rows, logits_rows=1, argmax=False):
        """One pass over `rows` rows whose tokens / positions are in self.tokens /
        self.pos: all rows' KV rows written, the logits of the last
        `logits_rows` rows in self.logits[:logits_rows]; with argmax, their
        greedy tokens packed in self.key (which must be zero before)."""
        if rows > CHUNK:
            return self._run_rows(rows, logits_rows, argmax)
        c = self.cfg
        x, qkv, att = self.x[:rows], self.qkv[:rows], self.att[:rows]
        h, hq, s_h = self.h[:rows], self.hq[:rows], self.s_h[:rows]
        if rows <= CHAIN_ROWS and not c.moe and c.act == "silu":
            return self._run_chain(rows, logits_rows, argmax)
        args = self._attn_args(rows)
        self._embed(rows, x)
        for l, w in enumerate(self.layers):
            ops.linear_fused(x, w["wqkv"], w["s_wqkv"], norm_g=w["rms_att"], eps=c.eps, out=qkv)
            ops.attn(args[l])
            ops.linear_fused(att, w["wo"], w["s_wo"], resid=x, out=x)
            if c.moe:                                                          # router, gate/up, down+combine
                self._moe_rows(l, x)
                continue
            ops.ffn_swiglu(x, w["rms_ffn"], c.eps, w["w1"], w["s_w1"], w["w3"], w["s_w3"], None, h=h,
                           requant=False, act=c.act)
            ops.linear_fused(h, w["w2"], w["s_w2"], resid=x, out=x)          # quant_act(h) in the prologue
        xl = self.x[rows - logits_rows:rows]
        ops.classifier(xl, self.cls_q, self.cls_s, self.rms_final, c.eps, out=self.logits[:logits_rows],
                       argmax_key=self.key[:logits_rows] if argmax else None)

    def _run_chain(self, rows, logits_rows, argmax):
        """Decode rows (<= 4, the GEMV path) as the latency chain: the attention
        and the SwiGLU post max|att| / max|h| per row by atomic max into
        per-layer slots, the o and down projections read them instead of
        reducing (the same bits), and each slot is zeroed by the kernel two
        launches later, once its reader has finished."""
        c, L = self.cfg, self.cfg.layers
        x, qkv, att, h = self.x[:rows], self.qkv[:rows], self.att[:rows], self.h[:rows]
        args = self._attn_args(rows, chain=True)
        ops.embed(self.tokens[:rows], self.emb_q, self.emb_s, out=x)
        for l, w in enumerate(self.layers):
            ops.linear_chain(x, w["wqkv"], w["s_wqkv"], norm_g=w["rms_att"], eps=c.eps, out=qkv,
                             clear=self.amax_h[(l - 1) % L])               # the previous layer's h slot
            ops.attn(args[l])
            ops.linear_chain(att, w["wo"], w["s_wo"], x_amax=self.amax_att[l], resid=x, out=x)
            ops.ffn_swiglu_chain(x, w["rms_ffn"], c.eps, w["w1"], w["s_w1"], w["w3"], w["s_w3"], h,
                                 self.amax_h[l], clear=self.amax_att[l])
            ops.linear_chain(h, w["w2"], w["s_w2"], x_amax=self.amax_h[l], resid=x, out=x)
        xl = self.x[rows - logits_rows:rows]
        ops.classifier(xl, self.cls_q, self.cls_s, self.rms_final, c.eps, out=self.logits[:logits_rows],
                       argmax_key=self.key[:logits_rows] if argmax else None)

    def _embed(self, rows, x):
        ops.embed(self.tokens[:rows], self.emb_q, self.emb_s, out=x)

    def _moe(self, l, x, j):
        """The MoE FFN of layer l on rows x (at most 16, starting at row j):
        x = x + moe(rmsnorm(x)); the routing into moe_ids / moe_w."""
        c, w, e = self.cfg, self.layers[l], j + x.shape[0]
        ops.moe_ffn(x, w["rms_ffn"], c.eps, w["router"], w["s_router"], c.top_k, w["e_gate"], w["s_e_gate"],
                    w["e_up"], w["s_e_up"], w["e_down"], w["s_e_down"], self.moe_scratch, resid=x, out=x,
                    ids=self.moe_ids[l, j:e], w=self.moe_w[l, j:e])

    def _moe_rows(self, l, x):
        """The MoE FFN of layer l on all rows of x: more than 16 rows grouped by
        expert (each expert's weights read once), else (or for a dim that is not
        a multiple of 32, which the grouped kernels need) the per-row kernels in
        16-row groups."""
        rows = x.shape[0]
        c, w = self.cfg, self.layers[l]
        if rows <= CHUNK or c.dim % 32:
            for j in range(0, rows, CHUNK):
                self._moe(l, x[j:j + CHUNK], j)
            return
        ops.moe_ffn_rows(x, w["rms_ffn"], c.eps, w["router"], w["s_router"], c.top_k, w["e_gate"], w["s_e_gate"],
                         w["e_up"], w["s_e_up"], w["e_down"], w["s_e_down"], self.moe_rows_scratch, resid=x, out=x,
                         ids=self.moe_ids[l, :rows], w=self.moe_w[l, :rows])

    def _sub_attn_args(self, l, j, m):
        a = self._sub_args.get((l, j, m))
        if a is None:
            c, w = self.cfg, self.layers[l]
            a = self._sub_args[(l, j, m)] = ops.attn_args(
                c, m, self.pos[j:j + m], self.qkv[j:j + m], self.kc[l], self.vc[l], self.att[j:j + m],
                self.consts[l], self.cos, self.sin, self.attn_scratch, w.get("q_norm"), w.get("k_norm"),
                ch=self.kv_ch[l])
        return a

    def _q(self, rows, k):
        return self.xq_buf[:rows * k].view(rows, k), self.sx_buf[:rows]

    def _run_rows(self, rows, logits_rows, argmax):
        """A prefill chunk of more than 16 rows: every linear as one tensor-core
        GEMM over all rows (the row quantizer first); every row's K/V appended,
        then one attention launch over the rows in 16-row groups; the MoE FFN in
        16-row groups (a row's results do not depend on the chunking: each row
        attends positions up to its own, all written first)."""
        c = self.cfg
        x, qkv, att, h = self.x[:rows], self.qkv[:rows], self.att[:rows], self.h[:rows]
        ops.embed(self.tokens[:rows], self.emb_q, self.emb_s, out=x)
        for l, w in enumerate(self.layers):
            xq, sx = self._q(rows, c.dim)
            ops.quant_rows(x, w["rms_att"], c.eps, xq=xq, s_x=sx)
            ops.gemm(xq, sx, w["wqkv"], w["s_wqkv"], out=qkv)
            a = self._sub_attn_args(l, 0, rows)                 # all rows: K / V first, then one attention
            ops.kv_append(a)
            ops.attn_prefill(a)
            aq, sa = self._q(rows, c.q_dim)
            ops.quant_rows(att, None, 0.0, xq=aq, s_x=sa)
            ops.gemm(aq, sa, w["wo"], w["s_wo"], out=x, resid=x)
            if c.moe:
                self._moe_rows(l, x)
                continue
            xq, sx = self._q(rows, c.dim)
            ops.quant_rows(x, w["rms_ffn"], c.eps, xq=xq, s_x=sx)
            ops.gemm_swiglu(xq, sx, w["w1"], w["s_w1"], w["w3"], w["s_w3"], out=h, act=c.act)
            hq, sh = self._q(rows, c.hidden)
            ops.quant_rows(h, None, 0.0, xq=hq, s_x=sh)
            ops.gemm(hq, sh, w["w2"], w["s_w2"], out=x, resid=x)
        xl = self.x[rows - logits_rows:rows]
        ops.classifier(xl, self.cls_q, self.cls_s, self.rms_final, c.eps, out=self.logits[:logits_rows],
                       argmax_key=self.key[:logits_rows] if argmax else None)

    def kernel_launches(self, rows=1):
        """Kernels one run() launches: embed, per layer the qkv GEMV, the
        attention, wo, then SwiGLU and w2 (or the MoE router, gate/up and
        down + combine), then the classifier."""
        return 1 + (6 if self.cfg.moe else 5) * self.cfg.layers + 1

    def capture(self, rows, logits_rows=1):
        """Capture run(rows) as a CUDA graph (after one eager warm-up run)."""
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            self.run(rows, logits_rows)
        torch.cuda.current_stream(self.dev).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.run(rows, logits_rows)
        self.graphs[(rows, logits_rows)] = g
        return g

    def decode_step(self):
        """One on-device greedy decode step: the last step's argmax token at
        the next position (w8a8_decode_advance), then run(1)."""
        ops.decode_advance(self.tokens, self.pos, self.key, 1, next_token=self.next_token)
        self.run(1, argmax=True)

    def capture_decode_step(self, seed_token, seed_pos):
        """decode_step() as a CUDA graph. The warm-up step runs from
        (seed_token, seed_pos + 1); its state change is undone afterwards."""
        self.set_next_token(seed_token)
        self.pos[0] = seed_pos
        saved = self.tokens.clone(), self.pos.clone(), self.key.clone()
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            self.decode_step()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        for dst, src in zip((self.tokens, self.pos, self.key), saved):
            dst.copy_(src)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.decode_step()
        self.graphs["step"] = g
        return g

    def set_next_token(self, token):
        """Seed the on-device decode loop: the next decode_step() feeds `token`."""
        if not 0 <= int(token) < self.cfg.vocab:
            raise ValueError(f"token {token} outside the vocabulary")
        self.key[0] = 0xFFFFFFFF - int(token)

    def launch(self, rows, logits_rows=1, graph=True):
        g = self.graphs.get((rows, logits_rows)) if graph else None
        if graph and g is None:
            g = self.capture(rows, logits_rows)
        if g is not None:
            g.replay()
        else:
            self.run(rows, logits_rows)

    # --------------------------------------------------------------- state
    def reset(self):
        self.kc.zero_()
        self.vc.zero_()

    def kv_rows(self, layer, n):
        """The cache of a layer in the reference's layout: K, V int8 [n, kv_dim]."""
        k = self.kc[layer, :, :n].permute(1, 0, 2).reshape(n, -1)
        v = self.vc[layer, :, :, :n].permute(2, 0, 1).reshape(n, -1)
        return k.cpu().numpy(), v.cpu().numpy()

    def weight_bytes(self):
        """int8 weight bytes streamed per decode token (+ fp32 scales)."""
        c = self.cfg
        per_layer = c.dim * c.qkv_dim + c.q_dim * c.dim
        scales = 4 * (c.qkv_dim + c.dim)
        if c.moe:                                  # the router and the k chosen experts
            per_layer += c.experts * c.dim + c.top_k * 3 * c.dim * c.expert_hidden
            scales += 4 * (c.experts + c.top_k * (2 * c.expert_hidden + c.dim))
        else:
            per_layer += 3 * c.dim * c.hidden
            scales += 4 * (2 * c.hidden + c.dim)
        return c.layers * (per_layer + scales) + c.vocab * c.dim + 4 * c.vocab

    def kv_bytes(self, t):
        """KV bytes read by one decode step attending t positions."""
        return self.cfg.layers * 2 * t * self.cfg.kv_dim


class BatchDecoder:
    """D sequences ("slots") per step, one token each, every slot with its own
    KV cache and position (`llm/runtime.py:155-208` BatchLlamaDevice over
    `compile_batch.BatchCompiler`). A step: every linear one tensor-core GEMM
    over the D rows (the row quantizer first), the attention one launch over all
    slots (grid z = slot), the MoE FFN in 16-row groups, the classifier GEMM for
    all D rows. Each slot's results equal a one-sequence decode bit for bit."""

    def __init__(self, cfg, qw, kv_scales, slots, device="cuda", kv_cols=None):
        cfg.validate()
        if slots < 1:
            raise ValueError("at least one slot")
        self.cfg, self.dev, self.slots = cfg, torch.device(device), slots
        _upload(self, cfg, qw, kv_scales, kv_cols)
        D, L, Hk, T, hd = slots, cfg.layers, cfg.kv_heads, cfg.seq_len, cfg.head_dim
        self.kc = torch.zeros(D, L, Hk, T, hd, dtype=I8, device=self.dev)
        self.vc = torch.zeros(D, L, Hk, hd, T, dtype=I8, device=self.dev)   # V transposed per head
        self.slot_stride = L * Hk * T * hd                                   # bytes between slots' caches
        z = lambda *s, dt=F32: torch.zeros(*s, dtype=dt, device=self.dev)
        self.tokens, self.pos = z(D, dt=I32), z(D, dt=I32)
        self.x, self.qkv, self.att = z(D, cfg.dim), z(D, cfg.qkv_dim), z(D, cfg.q_dim)
        self.h = z(D, cfg.hidden)
        self.logits = z(D, cfg.vocab)
        self.xq_buf = z(D * max(cfg.dim, cfg.q_dim, cfg.hidden), dt=I8)
        self.sx_buf = z(D)
        self.attn_scratch = ops.attn_scratch(1, cfg.heads, cfg.kv_heads, hd, T, self.dev)
        if cfg.moe:
            self.moe_ids = z(L, D, cfg.top_k, dt=I32)
            self.moe_w = z(L, D, cfg.top_k)
            self.moe_scratch = ops.moe_scratch(CHUNK, cfg.dim, cfg.top_k, cfg.expert_hidden, self.dev)
            self.moe_rows_scratch = (ops.moe_rows_scratch(D, cfg.dim, cfg.experts, cfg.top_k, cfg.expert_hidden,
                                                          self.dev) if D > CHUNK and cfg.dim % 32 == 0 else None)
        self.args = [ops.attn_args(cfg, 1, self.pos, self.qkv, self.kc[0, l], self.vc[0, l], self.att,
                                   self.consts[l], self.cos, self.sin, self.attn_scratch, w.get("q_norm"),
                                   w.get("k_norm"), ch=self.kv_ch[l])
                     for l, w in enumerate(self.layers)]
        self.graph = None

    _moe = DeviceDecoder._moe                      # the MoE FFN of all slots
    _moe_rows = DeviceDecoder._moe_rows

    def _q(self, k):
        return self.xq_buf[:self.slots * k].view(self.slots, k), self.sx_buf

    def step(self):
        """One token of every slot (self.tokens / self.pos) -> self.logits [D, vocab]."""
        c, D, x = self.cfg, self.slots, self.x
        ops.embed(self.tokens, self.emb_q, self.emb_s, out=x)
        for l, w in enumerate(self.layers):
            xq, sx = self._q(c.dim)
            ops.quant_rows(x, w["rms_att"], c.eps, xq=xq, s_x=sx)
            ops.gemm(xq, sx, w["wqkv"], w["s_wqkv"], out=self.qkv)
            ops.attn_batch(self.args[l], D, self.slot_stride)
            aq, sa = self._q(c.q_dim)
            ops.quant_rows(self.att, None, 0.0, xq=aq, s_x=sa)
            ops.gemm(aq, sa, w["wo"], w["s_wo"], out=x, resid=x)
            if c.moe:
                self._moe_rows(l, x)
                continue
            xq, sx = self._q(c.dim)
            ops.quant_rows(x, w["rms_ffn"], c.eps, xq=xq, s_x=sx)
            ops.gemm_swiglu(xq, sx, w["w1"], w["s_w1"], w["w3"], w["s_w3"], out=self.h, act=c.act)
            hq, sh = self._q(c.hidden)
            ops.quant_rows(self.h, None, 0.0, xq=hq, s_x=sh)
            ops.gemm(hq, sh, w["w2"], w["s_w2"], out=x, resid=x)
        xq, sx = self._q(c.dim)
        ops.quant_rows(x, self.rms_final, c.eps, xq=xq, s_x=sx)
        ops.gemm(xq, sx, self.cls_q, self.cls_s, out=self.logits)

    def capture(self):
        """The step as a CUDA graph (after one eager warm-up step)."""
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            self.step()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step()
        self.graph = g
        return g

    def clear_slot(self, b):
        self.kc[b].zero_()
        self.vc[b].zero_()

    def kernel_launches(self):
        c = self.cfg
        grouped = self.slots > CHUNK and c.dim % 32 == 0           # router, up, down, combine
        ffn = (4 if grouped else 3 * ((self.slots + CHUNK - 1) // CHUNK)) if c.moe else 4
        return 1 + c.layers * (5 + ffn) + 2
