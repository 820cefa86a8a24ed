"""Host runtime with the reference's surface (`llm/runtime.py`): LlamaDevice
(load once, per-token forward, generate, reset, close, stats) and run.c's
Sampler, over DeviceDecoder on a B200 instead of the overlay's descriptor ring.

Per token, as the reference does per submit (`llm/runtime.py:107-125`): the
(pos, token) pair goes to the device (an 8-byte host-to-device copy into the
graph's input buffers), the captured program replays, and the logits come back
as a float32 copy. Prompts can also be prefilled in chunks (`compile_model`'s
L6 prefill, `compiler/runtime/tools/sa_llm_run.c:255-300`, `qhf.QModel.prefill`
:356-364): every row is computed exactly as a decode step, so the KV cache and
logits equal the decode-only run bit for bit.

BatchLlamaDevice is the reference's batched runtime (`llm/runtime.py:155-241`):
D slots, each with its own KV cache and position, one token of every slot per
step.
"""
import os
import time

import numpy as np
import torch

from .model import CHUNK, PREFILL, BatchDecoder, DeviceDecoder

F = np.float32
BOS = 1


_U64 = (1 << 64) - 1


class XorShift64Star:
    """run.c's generator (random_u32 / random_f32): the 64-bit state goes
    through xorshift steps 12 (right), 25 (left), 27 (right); an output is the
    high 32 bits of state * 0x2545F4914F6CDD1D, and a uniform float in [0, 1)
    is its top 24 bits over 2^24. A zero seed would stay zero, so it runs as 1."""

    def __init__(self, seed):
        self.state = (int(seed) & _U64) or 1

    def u32(self):
        x = self.state
        x ^= x >> 12
        x = (x ^ (x << 25)) & _U64
        x ^= x >> 27
        self.state = x
        return ((x * 0x2545F4914F6CDD1D) & _U64) >> 32

    def unit(self):
        return (self.u32() >> 8) / float(1 << 24)


def softmax_f32(logits, temperature):
    """float32 softmax of logits / temperature: exp(z - max z) over its float32
    sum (the run.c sampler's probabilities, as llm/runtime.py forms them)."""
    z = np.asarray(logits, F) / F(temperature)
    e = np.exp(z - z.max())
    return e / e.sum(dtype=F)


def first_above(cdf, u):
    """Index of the first cumulative probability above u, or the last index
    when rounding left every entry at or below it (run.c sample_mult)."""
    return min(int(np.searchsorted(cdf, u, side="right")), len(cdf) - 1)


def nucleus_draw(p, topp, u):
    """run.c sample_topp: candidates with p >= (1 - topp) / (n - 1), in
    descending order (equal probabilities by index), kept up to the first
    prefix whose float32 sum exceeds topp; then the draw u * (that sum) over
    the kept prefix."""
    cand = np.flatnonzero(p >= (1.0 - topp) / (p.size - 1))
    order = cand[np.argsort(-p[cand], kind="stable")]
    cdf = np.cumsum(p[order], dtype=F)
    last = first_above(cdf, F(topp))
    return int(order[first_above(cdf[:last + 1], u * float(cdf[last]))])


class Sampler:
    """The next token from a row of logits, as run.c's sampler does it (the
    reference's host runtime keeps that sampler: llm/runtime.py:37-72):
    temperature 0 is greedy (the first maximum); otherwise one uniform draw per
    call over softmax(logits / temperature), from the whole distribution when
    topp is outside (0, 1), else from the top-p nucleus."""

    def __init__(self, temperature=0.0, topp=0.9, seed=1):
        self.temperature, self.topp = float(temperature), float(topp)
        self.rng = XorShift64Star(seed)

    def __call__(self, logits):
        if self.temperature == 0.0:
            return int(np.argmax(logits))
        p = softmax_f32(logits, self.temperature)
        u = self.rng.unit()
        if 0.0 < self.topp < 1.0:
            return nucleus_draw(p, self.topp, u)
        return first_above(np.cumsum(p, dtype=F), u)


def _model_of(model):
    """(cfg, weights, kv_scales) from a .w8a8 path (the reference's device
    model file, `llm/export_w8a8.py`) or the tuple itself."""
    if isinstance(model, (str, bytes, os.PathLike)):
        from .loaders import read_w8a8
        return read_w8a8(os.fspath(model))
    return model


class LlamaDevice:
    """One sequence on one GPU. model: a DeviceDecoder, (cfg, QuantWeights,
    kv_scales) to build one, or the path of a .w8a8 model file as the
    reference's constructor takes it (`llm/runtime.py:75-97`:
    `LlamaDevice(model_path, tokenizer_path=None, bitfile=None, firmware=None,
    use_irq=True, device=None)`). The overlay's bitstream, firmware and
    interrupt mode have no counterpart on a GPU and are accepted for the same
    call; tokenizers are outside this library (token ids in, logits out).
    graphs: replay captured CUDA graphs (default)."""

    def __init__(self, model, tokenizer_path=None, bitfile=None, firmware=None, use_irq=True, device="cuda",
                 graphs=True):
        if isinstance(model, DeviceDecoder):
            self.dec = model
        else:
            self.dec = DeviceDecoder(*_model_of(model), device=device if device is not None else "cuda")
        self.tokenizer_path = tokenizer_path
        self.cfg = self.dec.cfg
        self.graphs = graphs
        self.pos = 0
        self.stats = []                                   # per token: (pos, wall seconds)
        self._rows = self.dec.rows_cap                    # most rows per launch
        self._in = torch.zeros(2 * self._rows, dtype=torch.int32).pin_memory()   # tokens | positions
        self._out = torch.zeros(self.cfg.vocab, dtype=torch.float32).pin_memory()

    @classmethod
    def from_w8a8(cls, path, **kw):
        """A device for the model file at `path` (the reference exporter's .w8a8)."""
        return cls(os.fspath(path), **kw)

    def reset(self):
        """Start a new sequence: empty KV cache, pos 0 (`llm/runtime.py:101-105`)."""
        self.dec.reset()
        self.pos = 0

    def _submit(self, tokens, positions, logits=True, staging=None):
        """Stage (tokens, positions) in pinned memory, copy them to the graph's
        input buffers and launch. staging: a pinned [2*rows_cap] int32 slice that
        stays untouched until the stream has consumed it (default: the
        single-token buffer, safe because forward() synchronizes)."""
        m = len(tokens)
        if min(tokens) < 0 or max(tokens) >= self.cfg.vocab:
            raise ValueError(f"token outside [0, {self.cfg.vocab})")
        buf = self._in if staging is None else staging
        buf[:m] = torch.as_tensor(tokens, dtype=torch.int32)
        R = self._rows
        buf[R:R + m] = torch.as_tensor(positions, dtype=torch.int32)
        self.dec.tokens[:m].copy_(buf[:m], non_blocking=True)
        self.dec.pos[:m].copy_(buf[R:R + m], non_blocking=True)
        self._launch(m, logits)

    def _launch(self, m, logits):
        """Run m staged rows; with logits, the last row's logits into self._out."""
        self.dec.launch(m, 1, graph=self.graphs)
        if logits:
            self._out.copy_(self.dec.logits[0], non_blocking=True)

    def forward(self, token, perf=False):
        """Logits (float32 copy) of token at the current position; advances pos."""
        if self.pos >= self.cfg.seq_len:
            raise ValueError(f"sequence full ({self.cfg.seq_len} positions)")
        t0 = time.perf_counter()
        self._submit([int(token)], [self.pos])
        torch.cuda.current_stream().synchronize()
        out = self._out.numpy().copy()
        self.stats.append((self.pos, time.perf_counter() - t0))
        self.pos += 1
        return out

    def prefill(self, tokens):
        """Feed a prompt from the current position: chunks of up to PREFILL rows
        on the tensor cores while more than 16 rows remain, then a 16-row chunk
        ending at the prompt's last token (it may recompute rows already done:
        the same values are written again). Returns the logits of the last token."""
        toks = [int(t) for t in tokens]
        p0, n = self.pos, len(toks)
        if p0 + n > self.cfg.seq_len:
            raise ValueError("prompt beyond the sequence length")
        if n == 0:
            raise ValueError("empty prompt")
        big = min(PREFILL, self._rows)
        spans, s = [], 0
        while n - s > CHUNK:                              # tensor-core chunks
            e = min(s + big, n)
            spans.append((s, e))
            s = e
        if s < n:                                         # the tail: one GEMV-path chunk of <= 16 rows
            spans.append((max(n - CHUNK, 0), n))
        staging = torch.zeros(len(spans), 2 * self._rows, dtype=torch.int32).pin_memory()
        for i, (s, e) in enumerate(spans):
            self._submit(toks[s:e], list(range(p0 + s, p0 + e)), logits=i == len(spans) - 1, staging=staging[i])
        torch.cuda.current_stream().synchronize()
        self.pos = p0 + n
        return self._out.numpy().copy()

    def generate(self, prompt_tokens, steps=256, temperature=0.0, topp=0.9, seed=1, stop_at_bos=True,
                 forced=None):
        """Yield token ids run.c style (`llm/runtime.py:127-148`): the prompt's
        tokens are fed first, then sampled tokens, until `steps` positions.
        forced: teacher forcing; yields (argmax, logits) per position."""
        self.reset()
        toks = list(forced if forced is not None else prompt_tokens)
        sample = Sampler(temperature, topp, seed)
        token = toks[0]
        for pos in range(min(steps, self.cfg.seq_len)):
            logits = self.forward(token)
            if forced is not None:
                yield int(np.argmax(logits)), logits
                if pos + 1 >= len(forced):
                    return
                token = forced[pos + 1]
                continue
            nxt = toks[pos + 1] if pos + 1 < len(toks) else sample(logits)
            if nxt == BOS and stop_at_bos:
                return
            yield nxt
            token = nxt

    def close(self):
        self.dec = None
        torch.cuda.empty_cache()


class BatchLlamaDevice:
    """D sequences per step (`llm/runtime.py:155-241`). model: a BatchDecoder,
    or (cfg, QuantWeights, kv_scales) to build one with `slots` slots. Slot b
    has its own KV cache and position; step() runs one token of every slot. A
    slot without a sequence runs a dummy token at pos 0 (its KV row 0 is
    rewritten when a sequence starts in it)."""
    DUMMY = BOS

    def __init__(self, model, slots=None, device="cuda", graphs=True):
        self.dec = model if isinstance(model, BatchDecoder) else BatchDecoder(*model, slots=slots, device=device)
        self.cfg, self.d = self.dec.cfg, self.dec.slots
        self.graphs = graphs
        self.stats = []                                   # per step: wall seconds
        self._in = torch.zeros(2 * self.d, dtype=torch.int32).pin_memory()   # tokens | positions
        self._out = torch.zeros(self.d, self.cfg.vocab, dtype=torch.float32).pin_memory()

    def clear_slot(self, b):
        """Empty the KV cache of slot b (`llm/runtime.py:187-191`)."""
        if not 0 <= b < self.d:
            raise ValueError(f"slot {b} outside [0, {self.d})")
        self.dec.clear_slot(b)

    def step(self, poses, tokens, perf=False):
        """One token for each of the D slots; returns the D x vocab logits (copy)."""
        d = self.d
        if len(poses) != d or len(tokens) != d:
            raise ValueError(f"{d} positions and {d} tokens expected")
        if min(tokens) < 0 or max(tokens) >= self.cfg.vocab:
            raise ValueError(f"token outside [0, {self.cfg.vocab})")
        if min(poses) < 0 or max(poses) >= self.cfg.seq_len:
            raise ValueError(f"position outside [0, {self.cfg.seq_len})")
        t0 = time.perf_counter()
        self._in[:d] = torch.as_tensor(tokens, dtype=torch.int32)
        self._in[d:] = torch.as_tensor(poses, dtype=torch.int32)
        self.dec.tokens.copy_(self._in[:d], non_blocking=True)
        self.dec.pos.copy_(self._in[d:], non_blocking=True)
        self._out.copy_(self._run_step(), non_blocking=True)
        torch.cuda.current_stream().synchronize()
        self.stats.append(time.perf_counter() - t0)
        return self._out.numpy().copy()

    def _run_step(self):
        """Run the staged step; the [D, vocab] logits tensor."""
        if self.graphs:
            g = self.dec.graph or self.dec.capture()
            g.replay()
        else:
            self.dec.step()
        return self.dec.logits

    def generate(self, prompts, steps, stagger=0, temperature=0.0, topp=0.9, seed=1, on_logits=None):
        """Generate for len(prompts) <= D sequences at once (`llm/runtime.py:210-241`):
        sequence b starts at step b * stagger and runs `steps` positions (its
        prompt tokens first, then sampled; BOS does not stop it). prompts are
        token lists. on_logits(b, pos, logits) sees every position. Returns the
        token lists."""
        d, n = self.d, len(prompts)
        if n > d:
            raise ValueError(f"at most {d} sequences")
        toks = [list(p) for p in prompts]
        samplers = [Sampler(temperature, topp, seed + b) for b in range(n)]
        out = [[t[0]] for t in toks]
        start = [b * stagger for b in range(n)]
        for b in range(d):
            self.clear_slot(b)
        total = max(start) + steps if n else 0
        for s in range(total):
            poses, cur, live = [0] * d, [self.DUMMY] * d, [False] * d
            for b in range(n):
                p = s - start[b]
                if 0 <= p < steps:
                    poses[b], cur[b], live[b] = p, out[b][p], True
            logits = self.step(poses, cur)
            for b in range(n):
                if not live[b]:
                    continue
                p = poses[b]
                if on_logits:
                    on_logits(b, p, logits[b])
                if p + 1 < steps:
                    out[b].append(toks[b][p + 1] if p + 1 < len(toks[b]) else samplers[b](logits[b]))
        return out

    def close(self):
        if self.dec is not None:
            self.dec.graph = None                         # a graph may hold NCCL work (tensor parallel)
            torch.cuda.synchronize()
        self.dec = None
        torch.cuda.empty_cache()


class DeviceRig:
    """The B200 in the place of the overlay's functional simulator in the
    reference's tests: `llm/test_l4.py:58-85` (Rig: the model, io area and KV
    cache in the simulator's DDR, `run(dl, pos, token)` executing the list with
    `SaFuncSim.run_list`, `llm/sa_funcsim.py:420`, then `logits()`, `x()`,
    `kv_cache()` read back). Here `program()` builds the decoder's one-token
    program once (the counterpart of `ModelCompiler(m).build()`: a CUDA graph
    of the step, its inputs (pos, token) read from device memory as the list
    reads PARAM and the argument block); `run(program, pos, token)` executes
    it for any position and token and returns the number of kernels launched
    (the list's count of decoded descriptors); the readers give the reference
    rig's layouts (kv_cache [layers, 2, seq_len, kv_dim] int8). A device error
    flag raised by the step (a token outside the vocabulary, a bounded wait
    that gave up) is raised as RuntimeError, as the simulator raises SaError.
    model: as LlamaDevice (a .w8a8 path, (cfg, weights, kv_scales) or a
    DeviceDecoder)."""

    def __init__(self, model, device="cuda"):
        self.dec = model if isinstance(model, DeviceDecoder) else DeviceDecoder(*_model_of(model), device=device)
        self.cfg = self.dec.cfg
        self._prog = None

    def program(self):
        if self._prog is None:
            self._prog = self.dec.capture(1, 1)
        return self._prog

    def run(self, program, pos, token):
        from . import ops
        c = self.cfg
        if not 0 <= int(pos) < c.seq_len:
            raise ValueError(f"position {pos} outside [0, {c.seq_len})")
        self.dec.tokens[0] = int(token)
        self.dec.pos[0] = int(pos)
        program.replay()
        torch.cuda.current_stream().synchronize()
        flags = ops.error_flags()
        if flags:
            raise RuntimeError(f"pos {pos}: device error flags {flags:#x}")
        return self.dec.kernel_launches(1)

    def logits(self):
        return self.dec.logits[0].cpu().numpy().copy()

    def x(self):
        return self.dec.x[0].cpu().numpy().copy()

    def kv_cache(self):
        c = self.cfg
        out = np.empty((c.layers, 2, c.seq_len, c.kv_dim), np.int8)
        for l in range(c.layers):
            out[l, 0], out[l, 1] = self.dec.kv_rows(l, c.seq_len)
        return out
