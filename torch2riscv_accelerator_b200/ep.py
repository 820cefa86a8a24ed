"""Expert parallelism for the MoE decoder: one process per GPU, each holding
every layer's attention and router whole and 1/ranks of its experts.

Per MoE layer and row: the router runs on every rank (identical Top-k ids and
weights); each rank runs the gate/up and down GEMVs of the chosen slots whose
expert it holds and writes w_j * y_j for those slots, +0 for the others, into
[rows, top_k, dim]; an NCCL all-reduce SUM gives every rank every slot's term
(each element has exactly one nonzero contributor, so the sum is that term; a
-0 becoming +0 does not change the fold, which starts from +0), and the combine
folds them in k order onto the residual as the one-GPU kernel does
(`compiler/frontend/hf_generic.py:641-657`). Everything else is replicated, so
each rank holds the full logits.

Decode rows (at most 4) need no collective: the down kernel stores each term
as an epoch-tagged word straight into every rank's exchange block (the term's
expert has one owner, so each word has one writer) together with a presence
word per rank, and the combine kernel polls them (`csrc/tp.cuh`); the step is
then one CUDA graph with programmatic dependent launch, like the one-GPU one.
Larger chunks use the NCCL all-reduce above.

The reference runs on one device; BASELINE.json's MoE config (Granite-1B
shape, 32 experts) names expert parallelism over 2-8 GPUs.
"""
import torch
import torch.distributed as dist

from . import _lib, ops
from .model import CHUNK, PREFILL, BatchDecoder, DeviceDecoder
from .runtime import BatchLlamaDevice, LlamaDevice
from .tp import TpComm, _no_pdl

F32 = torch.float32
EXPERT_KEYS = ("e_gate", "s_e_gate", "e_up", "s_e_up", "e_down", "s_e_down")


def check_ep(cfg, ranks):
    if not cfg.moe:
        raise ValueError(f"{cfg.name}: no experts to split")
    if ranks < 2 or cfg.experts % ranks:
        raise ValueError(f"{cfg.name}: {cfg.experts} experts do not split over {ranks} ranks")


class ExpertShard:
    """A QuantWeights-like view with this rank's experts only (expert_lo ..)."""


def shard_experts(cfg, qw, rank, ranks):
    check_ep(cfg, ranks)
    n = cfg.experts // ranks
    s = ExpertShard()
    for a in ("emb_q", "emb_s", "cls_q", "cls_s", "rms_final", "cos", "sin"):
        setattr(s, a, getattr(qw, a))
    s.layers = [{k: (v[rank * n:(rank + 1) * n] if k in EXPERT_KEYS else v) for k, v in t.items()}
                for t in qw.layers]
    s.expert_lo = rank * n
    return s


class EpDecoder(DeviceDecoder):
    """DeviceDecoder with this rank's experts (collective: every rank of the
    group constructs it and runs the same rows in the same order)."""

    def __init__(self, cfg, qw, kv_scales, group=None, device="cuda", max_rows=CHUNK, prefill_rows=PREFILL,
                 comm=None):
        self.group = group
        self.rank, self.ranks = dist.get_rank(group), dist.get_world_size(group)
        sh = shard_experts(cfg, qw, self.rank, self.ranks)
        super().__init__(cfg, sh, kv_scales, device=device, max_rows=max_rows, prefill_rows=prefill_rows)
        self.expert_lo = sh.expert_lo
        self.wy = torch.zeros(self.rows_cap, cfg.top_k, cfg.dim, dtype=F32, device=self.dev)
        self.comm = comm if comm is not None else TpComm(
            cfg, self.dev, group, sizes={"moe": _lib.tp_moe_words(self.ranks, cfg.top_k, cfg.dim)})

    def _exchange(self, rows):
        return rows <= _lib.TP_ROWS

    def _embed(self, rows, x):
        if self._exchange(rows):                               # a step of the exchange: a new epoch
            ops.tp_embed(self.comm.c, self.tokens[:rows], self.emb_q, self.emb_s, x)
        else:
            ops.embed(self.tokens[:rows], self.emb_q, self.emb_s, out=x)

    def _moe_rows(self, l, x):
        """Decode rows: the terms over the exchange, then the combine. More
        rows: all rows' terms into one buffer (grouped by expert above 16 rows),
        one all-reduce, one k-order combine."""
        c, w, rows = self.cfg, self.layers[l], x.shape[0]
        if hasattr(self, "comm") and self._exchange(rows):
            blk = self.comm.block(l, "moe")
            ops.tp_moe_ffn(self.comm.c, x, w["rms_ffn"], c.eps, w["router"], w["s_router"], c.top_k, self.expert_lo,
                           w["e_gate"], w["s_e_gate"], w["e_up"], w["s_e_up"], w["e_down"], w["s_e_down"],
                           self.moe_scratch, blk, self.moe_ids[l, :rows], self.moe_w[l, :rows])
            ops.tp_moe_combine(self.comm.c, blk, rows, c.top_k, x, x)
            return
        wy = self.wy[:rows]
        if rows > CHUNK and c.dim % 32 == 0:                   # grouped by expert
            ops.moe_ffn_rows(x, w["rms_ffn"], c.eps, w["router"], w["s_router"], c.top_k, w["e_gate"],
                             w["s_e_gate"], w["e_up"], w["s_e_up"], w["e_down"], w["s_e_down"],
                             self.moe_rows_scratch, ids=self.moe_ids[l, :rows], w=self.moe_w[l, :rows],
                             expert_lo=self.expert_lo, wy=wy)
        else:
            for j in range(0, rows, CHUNK):
                e = min(j + CHUNK, rows)
                ops.moe_ffn_ep(x[j:e], w["rms_ffn"], c.eps, w["router"], w["s_router"], c.top_k, self.expert_lo,
                               w["e_gate"], w["s_e_gate"], w["e_up"], w["s_e_up"], w["e_down"], w["s_e_down"],
                               self.moe_scratch, wy[j:e], self.moe_ids[l, j:e], self.moe_w[l, j:e])
        dist.all_reduce(wy, op=dist.ReduceOp.SUM, group=self.group)
        ops.moe_combine(wy, x, out=x)

    def run(self, rows, logits_rows=1, argmax=False):
        if self._exchange(rows):                               # no collective: programmatic launch kept
            return DeviceDecoder.run(self, rows, logits_rows, argmax)
        _no_pdl(lambda: DeviceDecoder.run(self, rows, logits_rows, argmax))

    def capture(self, rows, logits_rows=1):
        if not self._exchange(rows):
            raise RuntimeError("expert-parallel chunks hold NCCL collectives: run them eagerly")
        return DeviceDecoder.capture(self, rows, logits_rows)

    def capture_decode_step(self, seed_token, seed_pos):
        """As DeviceDecoder's (collective: every rank captures); the warm-up
        step's exchange is complete on every rank before the capture."""
        self.set_next_token(seed_token)
        self.pos[0] = seed_pos
        saved = self.tokens.clone(), self.pos.clone(), self.key.clone()
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            self.decode_step()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        torch.cuda.synchronize(self.dev)
        dist.barrier(self.group)
        for dst, src in zip((self.tokens, self.pos, self.key), saved):
            dst.copy_(src)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.decode_step()
        self.graphs["step"] = g
        return g

    def close(self):
        self.graphs.clear()
        torch.cuda.synchronize()
        self.comm.close()

    def kernel_launches(self, rows=1):
        return super().kernel_launches(rows) + self.cfg.layers          # + the combine per layer

    def weight_bytes(self):
        """int8 weight bytes per decode token on this rank (+ scales): its
        share of the k chosen experts on average."""
        c = self.cfg
        full = super().weight_bytes()
        experts = c.layers * c.top_k * (3 * c.dim * c.expert_hidden + 4 * (2 * c.expert_hidden + c.dim))
        return full - experts + experts // self.ranks


class EpLlamaDevice(LlamaDevice):
    """LlamaDevice over an EpDecoder. Every rank makes the same calls and
    returns the full logits."""

    def __init__(self, model, group=None, device=None, graphs=True):
        cfg, qw, kv = model
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        super().__init__(EpDecoder(cfg, qw, kv, group=group, device=dev), graphs=graphs)

    def _launch(self, m, logits):
        # decode rows replay their captured program; chunks run eagerly (they
        # hold NCCL collectives)
        self.dec.launch(m, 1, graph=self.graphs and m <= _lib.TP_ROWS)
        if logits:
            self._out.copy_(self.dec.logits[0], non_blocking=True)

    def close(self):
        self.dec.close()


class EpBatchDecoder(BatchDecoder):
    """BatchDecoder with this rank's experts (every slot's attention on every
    rank; the MoE FFN of all slots with one all-reduce per layer)."""

    def __init__(self, cfg, qw, kv_scales, slots, group=None, device="cuda"):
        self.group = group
        self.rank, self.ranks = dist.get_rank(group), dist.get_world_size(group)
        sh = shard_experts(cfg, qw, self.rank, self.ranks)
        super().__init__(cfg, sh, kv_scales, slots, device=device)
        self.expert_lo = sh.expert_lo
        self.wy = torch.zeros(slots, cfg.top_k, cfg.dim, dtype=F32, device=self.dev)

    _moe_rows = EpDecoder._moe_rows

    def step(self):
        _no_pdl(lambda: BatchDecoder.step(self))

    def capture(self):
        raise RuntimeError("the expert-parallel step holds NCCL collectives: run it eagerly")

    def kernel_launches(self):
        c = self.cfg
        if self.slots > CHUNK and c.dim % 32 == 0:                          # grouped: the combine already counted
            return super().kernel_launches()
        return super().kernel_launches() + c.layers                         # + the combine per layer


class EpBatchLlamaDevice(BatchLlamaDevice):
    def __init__(self, model, slots=None, group=None, device=None):
        if not isinstance(model, EpBatchDecoder):
            cfg, qw, kv = model
            dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
            model = EpBatchDecoder(cfg, qw, kv, slots, group=group, device=dev)
        super().__init__(model, graphs=False)
