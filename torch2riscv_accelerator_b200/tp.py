"""Tensor parallelism over the GPUs of one node: one process per GPU, each
holding one shard of every layer.

The split (exact, so every rank's results equal the one-GPU decoder's bit for
bit):
- column split: the q|k|v rows of the rank's heads (whole KV-head groups), the
  gate and up rows of its slice of the hidden dimension, the classifier rows of
  its slice of the vocabulary;
- row split: o and down over the input columns of the rank's heads / hidden
  slice; their int32 accumulators are summed across ranks before the
  dequantization (integer sums: exact in any order);
- quant_act of a column-split activation (att, h) takes max|x| over every rank
  (a maximum: order-free), each rank quantizing its own columns with it;
- RMSNorm, the residual stream, the embedding and the KV constants are
  replicated (identical arithmetic on identical inputs).

Decode rows (at most 4) exchange inside the kernels over NVLink (see
`csrc/tp.cuh`): attention and the SwiGLU post their row maxima, o and down
their partial sums, the classifier its greedy keys, straight into every rank's
exchange region; the consuming kernel polls its own region. Prefill chunks run
as tensor-core GEMMs with the caller's NCCL collectives between them (int32
all-reduce of the partials, max all-reduce of the row maxima).

The reference runs on one device; the sharded configurations (C2 / C3, 2-8
GPUs) are the ones BASELINE.json names for tensor parallelism.
"""
import ctypes

import numpy as np
import torch
import torch.distributed as dist

from . import _lib, ops
from .model import CHUNK, PREFILL, BatchDecoder, DeviceDecoder
from .runtime import BatchLlamaDevice, LlamaDevice

I8, F32, I32 = torch.int8, torch.float32, torch.int32


class Shard:
    """One rank's part of a QuantWeights (numpy, host), in the same attribute
    names: layers (dicts), emb_q / emb_s (replicated), cls_q / cls_s (the
    vocabulary slice), rms_final, cos, sin."""


def check_split(cfg, ranks):
    if cfg.moe:
        raise ValueError(f"{cfg.name}: MoE layers are split by expert, not by tensor parallelism")
    if not 2 <= ranks <= _lib.TP_MAX_RANKS:
        raise ValueError(f"tensor parallelism over 2..{_lib.TP_MAX_RANKS} ranks, not {ranks}")
    for what, n in (("kv_heads", cfg.kv_heads), ("hidden", cfg.hidden), ("vocab", cfg.vocab)):
        if n % ranks:
            raise ValueError(f"{cfg.name}: {what} {n} is not a multiple of {ranks} ranks")
    if (cfg.hidden // ranks) % 16 or (cfg.heads // ranks * cfg.head_dim) % 16:
        raise ValueError(f"{cfg.name}: a rank's hidden / head columns must be multiples of 16")


def local_config(cfg, ranks):
    """The shape of one rank's layers: its heads, KV heads, hidden and
    vocabulary slices (dim, head_dim and the sequence length are whole)."""
    check_split(cfg, ranks)
    return cfg.with_(heads=cfg.heads // ranks, kv_heads=cfg.kv_heads // ranks, hidden=cfg.hidden // ranks,
                     vocab=cfg.vocab // ranks)


def kv_columns(cfg, rank, ranks):
    """The cache channels of a rank's KV heads (per-channel KV scales)."""
    w = cfg.kv_dim // ranks
    return slice(rank * w, (rank + 1) * w)


def shard(cfg, qw, rank, ranks):
    """Rank `rank`'s shard of the quantized model (a host-side view; the
    quantization is the whole model's, so scales are unchanged)."""
    check_split(cfg, ranks)
    H, Hk, hd = cfg.heads, cfg.kv_heads, cfg.head_dim
    hq, hk, hs, vs = H // ranks, Hk // ranks, cfg.hidden // ranks, cfg.vocab // ranks
    q = np.arange(rank * hq * hd, (rank + 1) * hq * hd)
    k = cfg.q_dim + np.arange(rank * hk * hd, (rank + 1) * hk * hd)
    v = cfg.q_dim + cfg.kv_dim + np.arange(rank * hk * hd, (rank + 1) * hk * hd)
    rows = np.concatenate([q, k, v])
    hcols = slice(rank * hs, (rank + 1) * hs)
    c = lambda a: np.ascontiguousarray(a)
    s = Shard()
    s.layers = []
    for t in qw.layers:
        u = {n: t[n] for n in ("rms_att", "rms_ffn", "q_norm", "k_norm") if n in t}
        u["wqkv"], u["s_wqkv"] = c(t["wqkv"][rows]), c(t["s_wqkv"][rows])
        u["wo"], u["s_wo"] = c(t["wo"][:, q]), t["s_wo"]                 # input columns of the rank's heads
        u["w1"], u["s_w1"] = c(t["w1"][hcols]), c(t["s_w1"][hcols])
        u["w3"], u["s_w3"] = c(t["w3"][hcols]), c(t["s_w3"][hcols])
        u["w2"], u["s_w2"] = c(t["w2"][:, hcols]), t["s_w2"]
        s.layers.append(u)
    s.emb_q, s.emb_s = qw.emb_q, qw.emb_s
    s.cls_q, s.cls_s = c(qw.cls_q[rank * vs:(rank + 1) * vs]), c(qw.cls_s[rank * vs:(rank + 1) * vs])
    s.rms_final, s.cos, s.sin = qw.rms_final, qw.cos, qw.sin
    s.vocab_offset = rank * vs
    return s


class TpComm:
    """This rank's exchange region, and every other rank's mapped here (CUDA
    IPC; the handles travel over the torch.distributed group). Collective:
    every rank of the group constructs it with the same model shape."""

    def __init__(self, cfg, device, group=None, sizes=None):
        """sizes: words of each per-layer block kind; by default the tensor-
        parallel decoder's (max|att|, o partials, max|h|, down partials)."""
        self.group = group
        self.rank, self.ranks = dist.get_rank(group), dist.get_world_size(group)
        P, L = self.ranks, cfg.layers
        lib = _lib.load()
        if sizes is None:
            sizes = {"att": _lib.tp_amax_words(P), "o": _lib.tp_part_words(P, cfg.dim), "h": _lib.tp_amax_words(P),
                     "down": _lib.tp_part_words(P, cfg.dim)}
        off, self._off = _lib.TP_HEADER, {}
        for l in range(L):
            for kind, words in sizes.items():
                self._off[(l, kind)] = off
                off += 8 * words
        self._off["keys"] = off
        off += 8 * _lib.tp_key_words(P)
        self.bytes = off
        with torch.cuda.device(device):
            ptr = ctypes.c_void_p()
            _lib.check("w8a8_tp_alloc", lib.w8a8_tp_alloc(off, ctypes.byref(ptr)))
            self.own = ptr.value
            h = (ctypes.c_uint8 * 64)()
            _lib.check("w8a8_ipc_handle", lib.w8a8_ipc_handle(self.own, h))
            handles = [None] * P
            dist.all_gather_object(handles, bytes(h), group=group)
            self.bases, self._opened = [], []
            for r, hb in enumerate(handles):
                if r == self.rank:
                    self.bases.append(self.own)
                    continue
                hr = (ctypes.c_uint8 * 64).from_buffer_copy(hb)
                q = ctypes.c_void_p()
                _lib.check("w8a8_ipc_open", lib.w8a8_ipc_open(hr, ctypes.byref(q)))
                self.bases.append(q.value)
                self._opened.append(q.value)
        self.c = _lib.W8A8TpComm(self.rank, self.ranks, self.bytes,
                                 (ctypes.c_void_p * _lib.TP_MAX_RANKS)(*self.bases))
        dist.barrier(group)                        # every region is mapped everywhere before any kernel writes

    def block(self, layer, kind):
        """Device address of this rank's exchange block (layer, kind)."""
        return self.own + self._off[(layer, kind)]

    @property
    def keys(self):
        return self.own + self._off["keys"]

    def close(self):
        """Unmap the other ranks' regions and free this one (collective: the
        barrier keeps a region alive until nobody writes into it)."""
        if self.own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(self.group)
        lib = _lib.load()
        for q in self._opened:
            lib.w8a8_ipc_close(q)
        dist.barrier(self.group)
        lib.w8a8_tp_free(self.own)
        self.own, self._opened = None, []


class TpDecoder(DeviceDecoder):
    """One rank's decoder: the DeviceDecoder program over this rank's shard
    (its heads, KV heads, hidden and vocabulary slices; self.cfg is the local
    shape, self.full_cfg the model's). Decode rows (<= 4, all rows' logits)
    run as the in-kernel exchange chain; larger chunks as tensor-core GEMMs
    with NCCL collectives. self.logits holds this rank's vocabulary slice;
    gather_logits() assembles the full rows."""

    def __init__(self, cfg, qw, kv_scales, comm, device="cuda", max_rows=CHUNK, prefill_rows=PREFILL):
        cfg.validate()
        self.full_cfg, self.comm = cfg, comm
        sh = shard(cfg, qw, comm.rank, comm.ranks)
        super().__init__(local_config(cfg, comm.ranks), sh, kv_scales, device=device, max_rows=max_rows,
                         prefill_rows=prefill_rows, kv_cols=kv_columns(cfg, comm.rank, comm.ranks))
        self.vocab_offset = sh.vocab_offset
        R, L = self.rows_cap, cfg.layers
        z = lambda *s, dt=F32: torch.zeros(*s, dtype=dt, device=self.dev)
        self.xb = z(R, cfg.dim)                          # the residual stream's second buffer (ping-pong)
        self.sx_o = z(L, _lib.TP_ROWS)                   # activation scales of o / down (their partials' s_x)
        self.sx_d = z(L, _lib.TP_ROWS)
        self.acc = z(R, cfg.dim, dt=I32)                 # row-split partials (prefill path)
        self.ybuf = z(R, cfg.dim)
        self.amax_bits = z(R, dt=I32)
        self.logits_full = z(max_rows, cfg.vocab)
        self._ll = {}

    # ------------------------------------------------------------ the program
    def _ll_args(self, rows):
        a = self._ll.get(rows)
        if a is not None:
            return a
        c, lc, comm, L = self.full_cfg, self.cfg, self.comm, self.full_cfg.layers
        cp = ctypes.pointer(comm.c)
        p = lambda t: t.data_ptr()
        xa, xb = self.x, self.xb
        A = lambda **kw: _lib.W8A8TpLinearArgs(comm=cp, rows=rows, **kw)
        layers = []
        for l, w in enumerate(self.layers):
            if l == 0:
                src = dict(x=p(xa))
            else:                                        # finish the previous layer's down projection
                src = dict(part_in=comm.block(l - 1, "down"), part_s_w=p(self.layers[l - 1]["s_w2"]),
                           part_s_x=p(self.sx_d[l - 1]), resid=p(xb), x_out=p(xa))
            qkv = A(k=c.dim, n=lc.qkv_dim, norm_g=p(w["rms_att"]), eps=c.eps, w=p(w["wqkv"]), s_w=p(w["s_wqkv"]),
                    epilogue=_lib.TP_STORE, y=p(self.qkv), **src)
            o = A(k=lc.q_dim, n=c.dim, x=p(self.att), amax_in=comm.block(l, "att"), w=p(w["wo"]),
                  s_w=p(w["s_wo"]), epilogue=_lib.TP_PARTIAL, part_out=comm.block(l, "o"), s_x_out=p(self.sx_o[l]))
            ffn = A(k=c.dim, n=lc.hidden, part_in=comm.block(l, "o"), part_s_w=p(w["s_wo"]),
                    part_s_x=p(self.sx_o[l]), resid=p(xa), x_out=p(xb), norm_g=p(w["rms_ffn"]), eps=c.eps,
                    w=p(w["w1"]), s_w=p(w["s_w1"]), w_up=p(w["w3"]), s_up=p(w["s_w3"]),
                    epilogue=_lib.TP_SWIGLU, y=p(self.h), amax_out=comm.block(l, "h"), act=ops.ACTS[c.act])
            down = A(k=lc.hidden, n=c.dim, x=p(self.h), amax_in=comm.block(l, "h"), w=p(w["w2"]),
                     s_w=p(w["s_w2"]), epilogue=_lib.TP_PARTIAL, part_out=comm.block(l, "down"),
                     s_x_out=p(self.sx_d[l]))
            layers.append((qkv, o, ffn, down))
        cls = dict(k=c.dim, n=lc.vocab, part_in=comm.block(L - 1, "down"), part_s_w=p(self.layers[-1]["s_w2"]),
                   part_s_x=p(self.sx_d[L - 1]), resid=p(xb), x_out=p(xa), norm_g=p(self.rms_final), eps=c.eps,
                   w=p(self.cls_q), s_w=p(self.cls_s), epilogue=_lib.TP_STORE, y=p(self.logits),
                   n_offset=self.vocab_offset)
        a = self._ll[rows] = {"layers": layers, "cls": A(**cls), "cls_key": A(key_out=comm.keys, **cls)}
        return a

    def run(self, rows, logits_rows=1, argmax=False):
        """As DeviceDecoder.run: every row's KV written, the last logits_rows
        rows' logits (this rank's slice) in self.logits; with argmax, the greedy
        token goes to every rank's key block (decode rows only)."""
        if rows <= _lib.TP_ROWS and logits_rows == rows:
            return self._run_ll(rows, argmax)
        if argmax:
            raise ValueError("the fused greedy argmax runs on decode rows (at most 4, all rows' logits)")
        return self._run_gemm(rows, logits_rows)

    def _run_ll(self, rows, argmax):
        a, comm = self._ll_args(rows), self.comm
        args = self._attn_args(rows)
        ops.tp_embed(comm.c, self.tokens[:rows], self.emb_q, self.emb_s, self.x[:rows])
        for l, (qkv, o, ffn, down) in enumerate(a["layers"]):
            ops.tp_linear(qkv)
            ops.tp_attn(args[l], comm.c, comm.block(l, "att"))
            ops.tp_linear(o)
            ops.tp_linear(ffn)
            ops.tp_linear(down)
        ops.tp_linear(a["cls_key"] if argmax else a["cls"])

    def _run_gemm(self, rows, logits_rows):
        _no_pdl(lambda: self._run_gemm_rows(rows, logits_rows))

    def _run_gemm_rows(self, rows, logits_rows):
        c = self.full_cfg
        x, h = self.x[:rows], self.h[:rows]
        ops.embed(self.tokens[:rows], self.emb_q, self.emb_s, out=x)
        for l, w in enumerate(self.layers):
            xq, sx = self._q(rows, c.dim)
            ops.quant_rows(x, w["rms_att"], c.eps, xq=xq, s_x=sx)
            ops.gemm(xq, sx, w["wqkv"], w["s_wqkv"], out=self.qkv[:rows])
            a = self._sub_attn_args(l, 0, rows)
            ops.kv_append(a)
            ops.attn_prefill(a)
            row_split(self, self.att[:rows], w["wo"], w["s_wo"], x, self.comm.group)
            xq, sx = self._q(rows, c.dim)
            ops.quant_rows(x, w["rms_ffn"], c.eps, xq=xq, s_x=sx)
            ops.gemm_swiglu(xq, sx, w["w1"], w["s_w1"], w["w3"], w["s_w3"], out=h, act=c.act)
            row_split(self, h, w["w2"], w["s_w2"], x, self.comm.group)
        ops.classifier(self.x[rows - logits_rows:rows], self.cls_q, self.cls_s, self.rms_final, c.eps,
                       out=self.logits[:logits_rows])

    def gather_logits(self, rows=1):
        """The full vocabulary of the first `rows` logits rows on every rank
        (NCCL all-gather of the slices) -> self.logits_full[:rows]."""
        P, vs = self.comm.ranks, self.cfg.vocab
        if rows == 1:
            dist.all_gather_into_tensor(self.logits_full[0], self.logits[0], group=self.comm.group)
        else:
            buf = torch.empty(P, rows, vs, dtype=F32, device=self.dev)
            dist.all_gather_into_tensor(buf, self.logits[:rows].contiguous(), group=self.comm.group)
            self.logits_full[:rows].copy_(buf.permute(1, 0, 2).reshape(rows, P * vs))
        return self.logits_full[:rows]

    def kernel_launches(self, rows=1):
        """Kernels of a decode-row run: embed, 5 per layer, the classifier."""
        return 1 + 5 * self.cfg.layers + 1

    # ------------------------------------------------------- decode loop
    def decode_step(self):
        """The greedy token of the last step (every rank's classifier keys) at
        the next position, then one decode row with the fused argmax."""
        ops.tp_advance(self.comm.c, self.comm.keys, self.tokens, self.pos, 1, next_token=self.next_token)
        self._run_ll(1, argmax=True)

    def set_next_token(self, token):
        if not 0 <= int(token) < self.full_cfg.vocab:
            raise ValueError(f"token {token} outside the vocabulary")
        ops.tp_seed(self.comm.c, self.comm.keys, int(token))

    def capture_decode_step(self, seed_token, seed_pos):
        """decode_step() as a CUDA graph (collective: every rank captures). The
        warm-up step runs from (seed_token, seed_pos + 1); its state change is
        undone and the seed written again once every rank has finished it."""
        self.set_next_token(seed_token)
        self.pos[0] = seed_pos
        saved = self.tokens.clone(), self.pos.clone()
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            self.decode_step()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        torch.cuda.synchronize(self.dev)
        dist.barrier(self.comm.group)                 # no rank's warm-up posts are still in flight
        for dst, src in zip((self.tokens, self.pos), saved):
            dst.copy_(src)
        self.set_next_token(seed_token)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.decode_step()
        self.graphs["step"] = g
        return g


class TpLlamaDevice(LlamaDevice):
    """LlamaDevice (`llm/runtime.py:75-152`) over a tensor-parallel decoder:
    every rank of the torch.distributed group constructs it with the same model
    and makes the same calls (forward, prefill, generate, reset, close); every
    rank returns the full logits. model: (cfg, QuantWeights, kv_scales)."""

    def __init__(self, model, comm=None, device=None, graphs=True):
        cfg, qw, kv = model
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.comm = comm if comm is not None else TpComm(cfg, dev)
        super().__init__(TpDecoder(cfg, qw, kv, self.comm, device=dev), graphs=graphs)
        self.cfg = cfg
        self._out = torch.zeros(cfg.vocab, dtype=F32).pin_memory()

    def _launch(self, m, logits):
        # decode rows replay their captured chain; chunks run eagerly (they
        # hold NCCL collectives)
        self.dec.launch(m, 1, graph=self.graphs and m <= _lib.TP_ROWS)
        if logits:
            self._out.copy_(self.dec.gather_logits(1)[0], non_blocking=True)

    def close(self):
        """Release the captured graphs, then the exchange regions (collective)."""
        self.dec.graphs.clear()
        torch.cuda.synchronize()
        self.comm.close()


def _no_pdl(fn):
    """Run fn with programmatic dependent launch off: kernels next to
    torch.distributed collectives are launched plainly (with it, a kernel right
    after a collective was measured to start before the collective's result
    was in place)."""
    lib = _lib.load()
    old = lib.w8a8_set_pdl(0)
    try:
        return fn()
    finally:
        lib.w8a8_set_pdl(old)


def row_split(dec, a, w, s_w, x, group):
    """x += the row-split linear of a (this rank's columns of a [rows, k]):
    max|a| per row over every rank (all-reduce MAX of the float bits), quant_act
    of this rank's columns with it, the GEMM's int32 partials summed over the
    ranks (all-reduce SUM, exact), then the dequantization with the residual."""
    rows, k = a.shape
    am = dec.amax_bits[:rows]
    ops.row_amax(a, am)
    dist.all_reduce(am, op=dist.ReduceOp.MAX, group=group)
    aq, sa = dec.xq_buf[:rows * k].view(rows, k), dec.sx_buf[:rows]
    ops.quant_rows_posted(a, am, aq, sa)
    acc = dec.acc[:rows]
    ops.gemm(aq, sa, w, s_w, out=dec.ybuf[:rows], acc=acc)
    dist.all_reduce(acc, op=dist.ReduceOp.SUM, group=group)
    ops.dequant_resid(acc, sa, s_w, out=x, resid=x)


class TpBatchDecoder(BatchDecoder):
    """BatchDecoder (D slots, one token each per step) over this rank's shard:
    each rank attends its own KV heads of every slot (its part of every slot's
    cache), the linears are the rank's GEMMs with the row-split ones completed
    by NCCL all-reduces. self.logits: this rank's vocabulary slice [D, vocab /
    ranks]; gather_logits() assembles [D, vocab]. Collective: every rank of the
    group constructs it and calls step() in the same order."""

    def __init__(self, cfg, qw, kv_scales, slots, group=None, device="cuda"):
        cfg.validate()
        self.group = group
        self.rank, self.ranks = dist.get_rank(group), dist.get_world_size(group)
        self.full_cfg = cfg
        sh = shard(cfg, qw, self.rank, self.ranks)
        super().__init__(local_config(cfg, self.ranks), sh, kv_scales, slots, device=device,
                         kv_cols=kv_columns(cfg, self.rank, self.ranks))
        D = slots
        z = lambda *s, dt=F32: torch.zeros(*s, dtype=dt, device=self.dev)
        self.acc, self.ybuf, self.amax_bits = z(D, cfg.dim, dt=I32), z(D, cfg.dim), z(D, dt=I32)
        self.logits_full = z(D, cfg.vocab)

    def step(self):
        _no_pdl(self._step)

    def _step(self):
        c, D, x, g = self.full_cfg, self.slots, self.x, self.group
        ops.embed(self.tokens, self.emb_q, self.emb_s, out=x)
        for l, w in enumerate(self.layers):
            xq, sx = self._q(c.dim)
            ops.quant_rows(x, w["rms_att"], c.eps, xq=xq, s_x=sx)
            ops.gemm(xq, sx, w["wqkv"], w["s_wqkv"], out=self.qkv)
            ops.attn_batch(self.args[l], D, self.slot_stride)
            row_split(self, self.att, w["wo"], w["s_wo"], x, g)
            xq, sx = self._q(c.dim)
            ops.quant_rows(x, w["rms_ffn"], c.eps, xq=xq, s_x=sx)
            ops.gemm_swiglu(xq, sx, w["w1"], w["s_w1"], w["w3"], w["s_w3"], out=self.h, act=c.act)
            row_split(self, self.h, w["w2"], w["s_w2"], x, g)
        xq, sx = self._q(c.dim)
        ops.quant_rows(x, self.rms_final, c.eps, xq=xq, s_x=sx)
        ops.gemm(xq, sx, self.cls_q, self.cls_s, out=self.logits)

    def capture(self):
        """The step as one CUDA graph, its NCCL all-reduces included (a
        collective: every rank captures, in the same order, after the eager
        warm-up step inside has run the same collectives). The launches stay
        plain (no programmatic dependent launch). Release the graph (the
        device's close(), or `self.graph = None`) before the process group is
        destroyed: a graph that holds NCCL work keeps its communicator busy."""
        return BatchDecoder.capture(self)

    def gather_logits(self):
        P, D, vs = self.ranks, self.slots, self.cfg.vocab
        buf = torch.empty(P, D, vs, dtype=F32, device=self.dev)
        dist.all_gather_into_tensor(buf, self.logits, group=self.group)
        self.logits_full.copy_(buf.permute(1, 0, 2).reshape(D, P * vs))
        return self.logits_full

    def kernel_launches(self):
        """Kernels of a step: embed; per layer quant, qkv GEMM, attention, then
        per row-split linear amax, quant, GEMM, dequant (x2) and quant + SwiGLU
        GEMM; final quant and classifier GEMM."""
        return 1 + self.cfg.layers * (3 + 4 + 2 + 4) + 2


class TpBatchLlamaDevice(BatchLlamaDevice):
    """BatchLlamaDevice (`llm/runtime.py:155-241`) over a TpBatchDecoder: every
    rank constructs it and calls step() / generate() in the same order; every
    rank returns the full [D, vocab] logits. graphs: replay the step as one
    CUDA graph with its collectives (close() before the process group ends),
    else launch it eagerly."""

    def __init__(self, model, slots=None, group=None, device=None, graphs=True):
        if not isinstance(model, TpBatchDecoder):
            cfg, qw, kv = model
            dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
            model = TpBatchDecoder(cfg, qw, kv, slots, group=group, device=dev)
        super().__init__(model, graphs=graphs)
        self.cfg = model.full_cfg
        self._out = torch.zeros(model.slots, self.cfg.vocab, dtype=F32).pin_memory()

    def _run_step(self):
        self.dec.step()
        return self.dec.gather_logits()

