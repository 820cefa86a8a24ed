#!/usr/bin/env python3
"""Decode throughput of the Qwen3-0.6B-shape W8A8 decoder at T = 2048 on B200,
with the int8 GEMV's HBM bandwidth against the measured peak.

Workload (batch 1): synthetic N(0, 0.02) weights
(seed 0) quantized per output channel, static KV scales from an fp32
calibration run on 16 seeded tokens; a seeded uniform prompt of
2048 - warmup - steps tokens (2032 by default) prefilled in 16-row chunks; then
`warmup` untimed and `steps` timed greedy decode steps, ending at position 2047.

value  device-resident decode: the captured step graph (on-device advance of
       token and position + the whole forward + argmax) replayed back to back,
       CUDA events on the launching stream, tokens / s (sum over ranks).
e2e    the same steps through LlamaDevice.forward: per step a pinned
       host-to-device copy of (token, pos) and a device-to-host copy of the
       logits [vocab] fp32, greedy sampling on the host.
roofline  the classifier GEMV (151936 x 1024, the largest weight stream of the
       step) timed alone with CUDA events; algorithmic bytes N*K + 4N + K + 4N.
cpu_baseline  the CPU oracle (NumPy restatement of the reference's device
       numerics) decoding on this host's cores from the same KV-cache state.

--impl reference times the reference's CPU path (the oracle port: the reference
is Python and does not travel) on the same config and metric; rank 0 only.
Multi-GPU (one process per GPU): tensor parallelism by default ("scaling":
"strong", one sequence over all GPUs; `--parallel tp`): each rank holds a shard
of every layer, the decode kernels exchange row maxima, int32 partial sums and
greedy keys over NVLink inside the kernels, e2e gathers the logits with NCCL.
`--parallel replicas` (or a config whose heads do not split) runs independent
batch-1 replicas instead ("scaling": "weak").
"""
import argparse
import json
import os
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s (Qwen3-0.6B shape W8A8, T=2048)"
# DRAM bytes (read + write) per launch of a kernel kind of the C2 step, from one
# ncu capture each; the commands and the figures are in the named profiles.
_LAYER = "profiles/decode_layer_c2_kernels.md"
NCU_TRAFFIC = {"classifier GEMV (rmsnorm + quant)": {"bytes": 152923904 + 6045184,
                                                       "source": "profiles/classifier_gemv_c2.txt"},
               "attention (cluster kernel, KV cache)": {"bytes": 4279040, "source": _LAYER},
               "qkv GEMV (rmsnorm + quant prologue)": {"bytes": 4252672, "source": _LAYER},
               "o_proj GEMV (+ residual)": {"bytes": 2144512, "source": _LAYER},
               "gate|up GEMV (rmsnorm + quant, SiLU gate)": {"bytes": 6370560, "source": _LAYER},
               "down GEMV (+ residual)": {"bytes": 3197440, "source": _LAYER}}
FPGA_TOKS = 3.41          # the reference's KV260 overlay, Qwen3-0.6B decode at T = 2048 (docs/results_v2.3.md:93-94)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """SM clock and clock-event reasons sampled through NVML every 2 ms while the
    timed region runs (read only; nothing is set)."""
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, cuda_index):
        self.cuda_index, self.samples, self.stop, self.h, self.nv = cuda_index, [], threading.Event(), None, None

    def _handle(self):
        import pynvml
        pynvml.nvmlInit()
        self.nv = pynvml
        try:
            import torch
            pr = torch.cuda.get_device_properties(self.cuda_index)
            bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(self.cuda_index)

    def _loop(self):
        nv = self.nv
        reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while True:
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM), int(reasons(self.h))))
            except Exception:
                pass
            if self.stop.wait(0.002):
                break

    def __enter__(self):
        try:
            self.h = self._handle()
            self.max_mhz = self.nv.nvmlDeviceGetMaxClockInfo(self.h, self.nv.NVML_CLOCK_SM)
            self.t = threading.Thread(target=self._loop, daemon=True)
            self.t.start()
        except Exception:
            self.h = None
        return self

    def __exit__(self, *a):
        self.stop.set()
        if self.h is not None:
            self.t.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [s for s, _ in self.samples]
        bits = 0
        for _, r in self.samples:
            bits |= r
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(self.max_mhz),
                "reasons": sorted(n for b, n in self.REASONS.items() if bits & b), "samples": len(sm),
                "source": "NVML every 2 ms"}


def dist_init():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=None)
    return ws, rank, local


def max_over_ranks(v, ws):
    if ws == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def cpu_threads():
    try:
        from threadpoolctl import threadpool_info
        return max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:
        return os.cpu_count() or 1


def oracle_decode(cfg, qw, kv_scales, kc, vc, start, tokens, logits=None):
    """Time the oracle's decode steps at positions start, start + 1, ... from a
    given cache state (kc / vc [layers, seq_len, kv_dim] int8); each step's
    logits appended to `logits` when it is a list."""
    from oracle import model as OM
    ora = OM.OracleDecoder(cfg, qw, kv_scales)
    ora.kc[:], ora.vc[:] = kc, vc
    ora._w64 = _NoCache()
    t0 = time.perf_counter()
    for i, t in enumerate(tokens):
        out = ora.forward(int(t), start + i)
        if logits is not None:
            logits.append(np.asarray(out, np.float32).copy())
    return time.perf_counter() - t0


class _NoCache(dict):
    """Convert the int8 weights to float64 per use instead of keeping 8 bytes
    per parameter resident (the C2 model would hold 4.8 GB)."""

    def __setitem__(self, k, v):
        pass


def build_model(cfg, seed):
    from torch2riscv_accelerator_b200.weights import QuantWeights
    calib = np.random.default_rng(seed + 1).integers(0, cfg.vocab, 16)
    return QuantWeights(cfg, seed=seed, calib_tokens=calib)


def run_reference(args, cfg, ws, rank):
    """The reference's CPU path on the host cores: the oracle port (NumPy
    restatement of DeviceModel / hf_generic numerics) decoding batch-1 steps at
    T ~ 2048 from a seeded synthetic int8 KV-cache state (the prompt is not
    prefilled on the CPU: 2032 oracle prefill steps would take hours)."""
    if rank != 0:
        return
    tp, ep = split_kind(cfg, args, ws)
    qw = build_model(cfg, args.seed)
    P = prompt_len(cfg, args)
    rng = np.random.default_rng(args.seed + 2)
    kc = np.zeros((cfg.layers, cfg.seq_len, cfg.kv_dim), np.int8)
    vc = np.zeros_like(kc)
    kc[:, :P] = rng.integers(-127, 128, (cfg.layers, P, cfg.kv_dim), dtype=np.int8)
    vc[:, :P] = rng.integers(-127, 128, (cfg.layers, P, cfg.kv_dim), dtype=np.int8)
    toks = rng.integers(0, cfg.vocab, args.warmup + args.steps)
    oracle_decode(cfg, qw, qw.kv_scales, kc, vc, P, toks[:args.warmup])
    dt = oracle_decode(cfg, qw, qw.kv_scales, kc, vc, P + args.warmup, toks[args.warmup:])
    cores = len(os.sched_getaffinity(0))
    # the repo arm's configuration at this N: one sequence (tensor / expert
    # parallel) or N replicas; the CPU decodes the same sequences either way
    seqs = 1 if (tp or ep) else ws
    v = seqs * args.steps / (seqs * dt)
    line = {"impl": "reference", "metric": metric_of(cfg, args), "value": v, "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps, "higher_is_better": True,
            "scaling": "strong" if (tp or ep) else "weak", "vs_baseline": v / FPGA_TOKS, "dtype": "int8",
            "data": "synthetic", "config": config_of(cfg, args, ws, tp, ep),
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cpu_threads(), "kind": "port",
                             "sample": f"{args.steps} full decode steps (all {cfg.layers} layers + classifier) at "
                                       f"positions {P + args.warmup}..{cfg.seq_len - 1} from a seeded int8 KV cache; "
                                       f"{cores} cores visible"},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_batch(args, cfg, qw, ws, rank, local):
    """Batched decode (BatchLlamaDevice): `batch` sequences per step, each with
    its own cache of T = 2048 positions, positions 2048 - warmup - steps ... 2047.
    The caches hold seeded random int8 values (the step reads the same bytes
    whatever they hold); value: replays of the captured step with the positions
    advanced on the device; e2e: BatchLlamaDevice.step with host tokens and
    positions and the [batch, vocab] logits back."""
    import torch
    from torch2riscv_accelerator_b200.model import BatchDecoder
    from torch2riscv_accelerator_b200.runtime import BatchLlamaDevice
    D = args.batch
    tp, ep = split_kind(cfg, args, ws)
    if tp:
        from torch2riscv_accelerator_b200.tp import TpBatchDecoder, TpBatchLlamaDevice
        dec = TpBatchDecoder(cfg, qw, qw.kv_scales, slots=D)
    elif ep:
        from torch2riscv_accelerator_b200.ep import EpBatchDecoder, EpBatchLlamaDevice
        dec = EpBatchDecoder(cfg, qw, qw.kv_scales, slots=D)
    else:
        dec = BatchDecoder(cfg, qw, qw.kv_scales, slots=D)
    split = tp or ep
    seqs = D if split else ws * D                      # sequences per step over all GPUs
    # seeded caches of the whole model, the same on every rank (a tensor-parallel
    # rank keeps its KV heads)
    L, Hk, T, hd = cfg.layers, cfg.kv_heads, cfg.seq_len, cfg.head_dim
    g = torch.Generator(device=dec.dev).manual_seed(args.seed + 11)
    kfull = torch.randint(-127, 128, (D, L, Hk, T, hd), dtype=torch.int8, device=dec.dev, generator=g)
    vfull = torch.randint(-127, 128, (D, L, Hk, hd, T), dtype=torch.int8, device=dec.dev, generator=g)
    heads = slice(rank * (Hk // ws), (rank + 1) * (Hk // ws)) if tp else slice(0, Hk)
    dec.kc.copy_(kfull[:, :, heads])
    dec.vc.copy_(vfull[:, :, heads])
    P = cfg.seq_len - args.warmup - args.steps
    rng = np.random.default_rng(args.seed + 3)
    tok0 = torch.as_tensor(rng.integers(0, cfg.vocab, D), dtype=torch.int32)
    dec.tokens.copy_(tok0)
    dec.pos.fill_(P)
    # parity: the first step (position P of every slot) against a one-GPU
    # BatchDecoder of the whole model (N > 1) or the oracle on two slots (N = 1)
    dec.step()
    got = (dec.gather_logits() if tp else dec.logits).cpu().numpy()
    parity = None
    if rank == 0:
        if split:
            ref = BatchDecoder(cfg, qw, qw.kv_scales, slots=D)
            ref.kc.copy_(kfull)
            ref.vc.copy_(vfull)
            ref.tokens.copy_(tok0)
            ref.pos.fill_(P)
            ref.step()
            want = ref.logits.cpu().numpy()
            parity = {"reference": f"one-GPU BatchDecoder of the whole model, the first step of all {D} slots",
                      "logits_equal": bool(np.array_equal(got.view(np.uint32), want.view(np.uint32))),
                      "tokens_equal": bool(np.array_equal(got.argmax(1), want.argmax(1)))}
            del ref
        elif not args.no_cpu_baseline:
            ok = []
            for b in sorted({0, D - 1}):
                kc = kfull[b].permute(0, 2, 1, 3).reshape(L, T, Hk * hd).cpu().numpy()
                vc = vfull[b].permute(0, 3, 1, 2).reshape(L, T, Hk * hd).cpu().numpy()
                ora = []
                oracle_decode(cfg, qw, qw.kv_scales, kc, vc, P, [int(tok0[b])], logits=ora)
                ok.append(np.array_equal(ora[0].view(np.uint32), got[b].view(np.uint32)))
            parity = {"reference": f"the oracle: slots {sorted({0, D - 1})}, the first step at position {P} "
                                   "from the seeded cache state", "logits_equal": all(ok), "tokens_equal": all(ok)}
    del kfull, vfull
    torch.cuda.empty_cache()
    # one step: the captured graph (the tensor-parallel one with its NCCL
    # all-reduces; the expert-parallel step runs eagerly)
    run = dec.step if ep else dec.capture().replay      # (a capture's warm-up step writes the rows of position P)
    st = torch.cuda.current_stream()
    for _ in range(args.warmup):
        run()
        dec.pos.add_(1)
    barrier(ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        torch.cuda.nvtx.range_push("batch")               # ncu --nvtx-include batch/ selects these launches
        e0.record(st)
        for _ in range(args.steps):
            run()
            dec.pos.add_(1)
        e1.record(st)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    barrier(ws)
    dt = max_over_ranks(e0.elapsed_time(e1) / 1e3, ws)
    # e2e: host tokens / positions in, [D, vocab] logits out, per step
    dev = TpBatchLlamaDevice(dec) if tp else EpBatchLlamaDevice(dec) if ep else BatchLlamaDevice(dec)
    toks = rng.integers(0, cfg.vocab, (args.warmup + args.steps, D))
    for i in range(args.warmup):
        dev.step([P + i] * D, [int(v) for v in toks[i]])
    barrier(ws)
    torch.cuda.synchronize()
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0.record(st)
    for i in range(args.steps):
        dev.step([P + args.warmup + i] * D, [int(v) for v in toks[args.warmup + i]])
    h1.record(st)
    torch.cuda.synchronize()
    barrier(ws)
    dt_e2e = max_over_ranks(h0.elapsed_time(h1) / 1e3, ws)
    if rank == 0:
        kv_step = D * dec.slot_stride * 2 * (P + args.warmup + args.steps // 2) // cfg.seq_len
        line = {
            "metric": metric_of(cfg, args), "value": seqs * args.steps / dt, "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps, "higher_is_better": True,
            "scaling": "strong" if split else "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (N(0,0.02) weights seed 0, uniform token ids, seeded random int8 caches)",
            "config": {"workload": f"{cfg.name}-shape W8A8 batched decode: {D} sequences per step, each at "
                                   f"positions {P}..{cfg.seq_len - 1} of its own T=2048 cache",
                       "model": cfg.name, "global_batch": seqs, "seq_len": cfg.seq_len,
                       "parallelism": f"tp{ws}" if tp else f"ep{ws}" if ep else f"replicas x{ws}",
                       "attention": cfg.attn,
                       "l2": "no flush: the step reads the weights and every slot's cache, far over the 126 MB L2"},
            "e2e": {"value": seqs * args.steps / dt_e2e, "unit": "tok/s", "h2d_bytes_per_step": 8 * D,
                    "d2h_bytes_per_step": 4 * D * cfg.vocab},
            "step_bytes": {"kv_read": kv_step,
                           "weights": sum(t.numel() for w in dec.layers for t in w.values()
                                          if t.dtype == torch.int8) + dec.cls_q.numel()},
            "gpu_launches": args.steps * dec.kernel_launches(),
            "clocks": clk.summary(), "mode": "batch", "parity": parity,
        }
        print(json.dumps(line), flush=True)
        if parity is not None and not (parity["logits_equal"] and parity["tokens_equal"]):
            raise RuntimeError(f"parity failed: {parity}")
    barrier(ws)
    run = None
    dev.close()                                         # the step graph (NCCL work at N > 1) released first
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# BASELINE.json's batched workloads as written: slots, prompt-length range,
# decode tokens per sequence (C1, C3, C4; C2's batch 128 is run_batch's case)
STATED = {"SmolLM2-135M": (64, (40, 40), 256), "Llama-3.2-1B": (256, (64, 1024), 128),
          "Granite-3.1-1B-A400M": (64, (64, 64), 128), "Qwen3-0.6B": (128, (2032, 2032), 16)}


def run_stated(args, cfg, qw, ws, rank, local):
    """The config's batched workload as BASELINE.json states it, on one GPU:
    D sequences with seeded prompt lengths and token ids; every step runs one
    token of every live slot (its prompt's next token, then its greedy token)
    at the slot's own position, as the reference's BatchLlamaDevice.generate
    loop does (llm/runtime.py:210-241), until every sequence has its decode
    tokens; a finished slot runs the dummy token at position 0. value: the
    captured step replayed with the schedule on the device (tokens chosen by
    device argmax), all slots' tokens per second; e2e: BatchLlamaDevice.step
    with host tokens and the [D, vocab] logits back, on the first 48 steps."""
    import torch
    from torch2riscv_accelerator_b200 import ops
    from torch2riscv_accelerator_b200.model import BatchDecoder
    from torch2riscv_accelerator_b200.runtime import BOS, BatchLlamaDevice
    if ws > 1 or cfg.name not in STATED:
        raise SystemExit("--workload stated: one GPU and a config with a stated batched workload")
    D, (lo, hi), gen = STATED[cfg.name]
    rng = np.random.default_rng(args.seed + 7)
    lens = rng.integers(lo, hi + 1, D)
    prompts = rng.integers(0, cfg.vocab, (D, hi))
    total = int(lens.max()) + gen
    dec = BatchDecoder(cfg, qw, qw.kv_scales, slots=D)
    dev = dec.dev
    pr = torch.as_tensor(prompts, dtype=torch.int32, device=dev)
    ln = torch.as_tensor(lens, dtype=torch.int32, device=dev)
    greedy = torch.zeros(D, dtype=torch.int32, device=dev)
    g = dec.capture()
    st = torch.cuda.current_stream()

    def step(s):
        live = ln + gen > s
        tok = torch.where(ln > s, pr[:, min(s, hi - 1)], greedy)
        dec.tokens.copy_(torch.where(live, tok, torch.full_like(tok, BOS)))
        dec.pos.copy_(torch.where(live, torch.full_like(ln, s), torch.zeros_like(ln)))
        g.replay()
        ops.argmax(dec.logits, out=greedy)

    for s in range(args.warmup):
        step(s)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record(st)
        for s in range(total):
            step(s)
        e1.record(st)
        torch.cuda.synchronize()
    dt = e0.elapsed_time(e1) / 1e3
    processed = int((lens + gen).sum())
    # e2e: the same schedule through the runtime API, host tokens and logits
    bdev = BatchLlamaDevice(dec)
    n_e2e = min(48, total)
    hg = np.zeros(D, np.int64)
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    live_e2e = 0
    h0.record(st)
    for s in range(n_e2e):
        live = lens + gen > s
        tok = np.where(lens > s, prompts[:, min(s, hi - 1)], hg)
        lg = bdev.step([s if live[b] else 0 for b in range(D)], [int(tok[b]) if live[b] else BOS for b in range(D)])
        hg = lg.argmax(1)
        live_e2e += int(live.sum())
    h1.record(st)
    torch.cuda.synchronize()
    dt_e2e = h0.elapsed_time(h1) / 1e3
    # bytes: every step streams the weights and each live slot's cache up to its position
    wbytes = sum(t.numel() for w in dec.layers for t in w.values() if t.dtype == torch.int8) + dec.cls_q.numel()
    kv = sum(2 * cfg.layers * cfg.kv_dim * int(min(s, l + gen - 1) + 1)
             for l in lens for s in range(int(l) + gen))
    nbytes = total * wbytes + kv
    peak, peak_src = peaks()
    if rank == 0:
        line = {
            "metric": metric_of(cfg, args), "value": processed / dt, "unit": "tok/s", "n_gpus": ws, "steps": total,
            "warmup": args.warmup, "ms_per_step": 1e3 * dt / total, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (N(0,0.02) weights seed 0, seeded prompt lengths and uniform token ids)",
            "config": {"workload": f"{cfg.name}-shape W8A8 batched decode as stated: {D} sequences, prompt lengths "
                                   f"U[{lo}, {hi}] fed one token per step, then {gen} greedy decode tokens each; "
                                   f"{total} steps, every live slot one token per step",
                       "model": cfg.name, "global_batch": D, "seq_len": cfg.seq_len, "parallelism": "replicas x1",
                       "attention": cfg.attn, "l2": "no flush: every step streams the weights and the live caches"},
            "decode_tok_s": D * gen / dt, "tokens_processed": processed,
            "e2e": {"value": live_e2e / dt_e2e, "unit": "tok/s", "steps": n_e2e, "h2d_bytes_per_step": 8 * D,
                    "d2h_bytes_per_step": 4 * D * cfg.vocab},
            "roofline": {"bound": "hbm", "achieved": nbytes / dt / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": nbytes / dt / 1e9 / peak, "peak_source": peak_src, "traffic": None,
                         "kernel": "the whole step (weights once per step + each live slot's KV up to its position)",
                         "bytes": nbytes},
            "gpu_launches": total * dec.kernel_launches(), "clocks": clk.summary(), "mode": "stated",
        }
        print(json.dumps(line), flush=True)


def run_kernel(args, cfg):
    """One kernel timed alone (the profiling case of `profiles/`): the batched
    decode attention of one layer, --batch slots each attending 2041 positions
    of its own seeded random int8 cache (K, V 2 x 2041 x head_dim bytes per
    slot and KV head)."""
    import hashlib

    import torch
    from torch2riscv_accelerator_b200 import ops
    from torch2riscv_accelerator_b200.weights import kv_consts, rope_tables
    D, Hk, hd, T = args.batch, cfg.kv_heads, cfg.head_dim, cfg.seq_len
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(args.seed + 1)
    kc = torch.randint(-127, 128, (D, Hk, T, hd), dtype=torch.int8, device=dev, generator=g)
    vc = torch.randint(-127, 128, (D, Hk, hd, T), dtype=torch.int8, device=dev, generator=g)
    qkv = torch.randn(D, cfg.qkv_dim, device=dev, generator=g)
    pos = torch.full((D,), T - 8, dtype=torch.int32, device=dev)
    att = torch.zeros(D, cfg.q_dim, device=dev)
    cos, sin = [torch.as_tensor(a).to(dev) for a in rope_tables(cfg)]
    gain = torch.ones(hd, device=dev) if cfg.qk_norm else None
    scratch = ops.attn_scratch(1, cfg.heads, Hk, hd, T, dev)
    a = ops.attn_args(cfg, 1, pos, qkv, kc[0], vc[0], att, kv_consts(0.05, 0.04, hd), cos, sin, scratch, gain, gain)
    for _ in range(args.warmup):
        ops.attn_batch(a, D, Hk * T * hd)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        ops.attn_batch(a, D, Hk * T * hd)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / args.steps * 1e3
    nbytes = D * Hk * 2 * (T - 7) * hd
    peak, peak_src = peaks()
    print(json.dumps({"kernel": "attn_stream_kernel", "config": {"model": cfg.name, "slots": D, "positions": T - 7},
                      "us_per_launch": us, "bytes_per_launch": nbytes, "GBs": nbytes / us / 1e3,
                      "frac": nbytes / us / 1e3 / peak, "peak": peak, "peak_source": peak_src,
                      "att_sha": hashlib.sha256(att.cpu().numpy().tobytes()).hexdigest()[:16],
                      "error_flags": ops.error_flags()}), flush=True)


def run_moe_kernel(args, cfg):
    """The MoE FFN of one layer alone (the profiling case of `profiles/`):
    --batch rows (more than 16) of a seeded random activation through
    w8a8_moe_ffn_rows (router, grouped gate/up, grouped down, k-order combine:
    4 launches a call) over seeded random int8 experts of the config's shape.
    Algorithmic bytes: every expert's weights once, their scales, the router,
    the rows in and out."""
    import hashlib

    import torch
    from torch2riscv_accelerator_b200 import ops
    if not cfg.moe or args.batch <= 16:
        raise SystemExit("--kernel moe_rows wants a MoE config and --batch > 16")
    D, dim, E, K, ih = args.batch, cfg.dim, cfg.experts, cfg.top_k, cfg.expert_hidden
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(args.seed + 2)
    i8 = lambda *s: torch.randint(-127, 128, s, dtype=torch.int8, device=dev, generator=g)
    sc = lambda *s: torch.rand(*s, device=dev, generator=g) * 1e-3 + 1e-4
    router, s_router = i8(E, dim), sc(E)
    gq, gs, uq, us, dq, ds = i8(E, ih, dim), sc(E, ih), i8(E, ih, dim), sc(E, ih), i8(E, dim, ih), sc(E, dim)
    x = torch.randn(D, dim, device=dev, generator=g)
    resid = torch.randn(D, dim, device=dev, generator=g)
    norm_g = torch.ones(dim, device=dev)
    out = torch.empty_like(x)
    ids = torch.empty(D, K, dtype=torch.int32, device=dev)
    w = torch.empty(D, K, device=dev)
    scratch = ops.moe_rows_scratch(D, dim, E, K, ih, dev)

    def call():
        ops.moe_ffn_rows(x, norm_g, cfg.eps, router, s_router, K, gq, gs, uq, us, dq, ds, scratch, resid=resid,
                         out=out, ids=ids, w=w)

    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        call()
    e1.record()
    torch.cuda.synchronize()
    us_call = e0.elapsed_time(e1) / args.steps * 1e3
    nbytes = E * 3 * ih * dim + 4 * E * (2 * ih + dim) + E * dim + 4 * E + 3 * 4 * D * dim
    int_ops = 2 * D * K * 3 * ih * dim + 2 * D * E * dim
    peak, peak_src = peaks()
    print(json.dumps({"kernel": "moe_rows (router, up, down, combine)", "config": {"model": cfg.name, "rows": D,
                      "experts": E, "top_k": K}, "us_per_call": us_call, "bytes_per_call": nbytes,
                      "GBs": nbytes / us_call / 1e3, "frac": nbytes / us_call / 1e3 / peak, "peak": peak,
                      "peak_source": peak_src, "int8_tops": int_ops / us_call / 1e6,
                      "y_sha": hashlib.sha256(out.cpu().numpy().tobytes()).hexdigest()[:16],
                      "error_flags": ops.error_flags()}), flush=True)


def kernel_table(dec, reps=5):
    """Each kernel kind of a batch-1 decode step (one sequence, this GPU's
    shard), launched for every layer back to back with plain stream ordering
    (no overlap between launches) inside a CUDA graph, timed with CUDA events:
    microseconds per launch, algorithmic bytes per launch, GB/s. Every layer
    reads its own weights and cache, so the loop's data is far over the L2;
    the classifier (one matrix, one launch per step) is launched 8 times per
    replay. The residual stream is restored afterwards."""
    import torch

    from torch2riscv_accelerator_b200 import _lib, ops
    c, L = dec.cfg, dec.cfg.layers
    w, x, qkv, att, h = dec.layers, dec.x[:1], dec.qkv[:1], dec.att[:1], dec.h[:1]
    t = int(dec.pos[0].item()) + 1                      # positions attended
    aa = dec._attn_args(1)
    kinds = [
        ("qkv GEMV (rmsnorm + quant prologue)", "gemv_kernel", L,
         lambda l: ops.linear_fused(x, w[l]["wqkv"], w[l]["s_wqkv"], norm_g=w[l]["rms_att"], eps=c.eps, out=qkv),
         c.qkv_dim * c.dim + 8 * c.qkv_dim + c.dim),
        ("attention (cluster kernel, KV cache)", "attn_kernel", L, lambda l: ops.attn(aa[l]),
         2 * t * c.kv_dim + 4 * (c.qkv_dim + c.q_dim)),
        ("o_proj GEMV (+ residual)", "gemv_kernel", L,
         lambda l: ops.linear_fused(att, w[l]["wo"], w[l]["s_wo"], resid=x, out=x),
         c.dim * c.q_dim + 8 * c.dim + c.q_dim + 4 * c.dim),
    ]
    if not c.moe:
        kinds += [
            ("gate|up GEMV (rmsnorm + quant, SiLU gate)", "gemv_kernel", L,
             lambda l: ops.ffn_swiglu(x, w[l]["rms_ffn"], c.eps, w[l]["w1"], w[l]["s_w1"], w[l]["w3"], w[l]["s_w3"],
                                      None, h=h, requant=False, act=c.act),
             2 * c.hidden * c.dim + 8 * c.hidden + c.dim + 4 * c.hidden),
            ("down GEMV (+ residual)", "gemv_kernel", L,
             lambda l: ops.linear_fused(h, w[l]["w2"], w[l]["s_w2"], resid=x, out=x),
             c.dim * c.hidden + 8 * c.dim + c.hidden + 4 * c.dim)]
    # the classifier: one launch per step, timed over 8 back-to-back launches
    # of the same weights (151936 x 1024 = 156 MB: above the 126 MB L2, read
    # in the same order every launch)
    kinds.append(("classifier GEMV (rmsnorm + quant)", "gemv_kernel", 1,
                  lambda l: ops.classifier(x, dec.cls_q, dec.cls_s, dec.rms_final, c.eps, out=dec.logits[:1]),
                  dec.cls_q.shape[0] * (c.dim + 8) + c.dim))
    reps_of = {kinds[-1][0]: 8}
    saved = dec.x.clone()
    lib = _lib.load()
    old = lib.w8a8_set_pdl(0)
    out = []
    try:
        for name, kern, n, fn, nbytes in kinds:
            per = n * reps_of.get(name, 1)              # launches per graph replay
            for l in range(n):                          # first calls outside the capture
                fn(l)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for i in range(per):
                    fn(i % n)
            for _ in range(2):
                g.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.nvtx.range_push(f"kernels:{name.split()[0]}")   # ncu --nvtx-include "kernels:classifier/"
            e0.record()
            for _ in range(reps):
                g.replay()
            e1.record()
            torch.cuda.nvtx.range_pop()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (reps * per)
            out.append({"kind": name, "kernel": kern, "launches_per_step": n, "us_per_launch": us,
                        "bytes_per_launch": nbytes, "GBs": nbytes / us / 1e3})
            del g
    finally:
        lib.w8a8_set_pdl(old)
        dec.x.copy_(saved)
        torch.cuda.synchronize()
    return out


def split_kind(cfg, args, ws):
    """(tensor parallel, expert parallel) for N GPUs: a MoE config splits its
    experts, a dense one its heads; independent replicas when the shape does
    not split or --parallel replicas."""
    if ws <= 1 or args.parallel != "tp":
        return False, False
    from torch2riscv_accelerator_b200.ep import check_ep
    from torch2riscv_accelerator_b200.tp import check_split
    try:
        (check_ep if cfg.moe else check_split)(cfg, ws)
    except ValueError as e:
        if int(os.environ.get("RANK", "0")) == 0:
            print(f"# {e}: independent replicas instead", file=sys.stderr)
        return False, False
    return not cfg.moe, cfg.moe


def metric_of(cfg, args):
    """BASELINE.json's metric for its workload (Qwen3 shape, batch 1, T = 2048);
    other workloads name their own."""
    if cfg.name == "Qwen3-0.6B" and args.batch <= 1 and not args.prompt:
        return METRIC
    return f"decode tok/s ({cfg.name} shape W8A8)"


def prompt_len(cfg, args):
    """Batch-1 prompt length: --prompt, else the context filled to its last
    warmup + steps positions (T = 2048 for the Qwen3 shape)."""
    return args.prompt if args.prompt else cfg.seq_len - args.warmup - args.steps


def config_of(cfg, args, ws, tp=False, ep=False):
    P = prompt_len(cfg, args)
    if ep:
        return {"workload": f"{cfg.name}-shape W8A8 MoE decode, batch 1, T=2048, experts split over {ws} GPUs: "
                            f"{P}-token prompt prefilled, then {args.warmup} untimed + {args.steps} timed greedy "
                            f"decode steps (the experts' terms exchanged inside the kernels over NVLink)",
                "model": cfg.name, "global_batch": 1, "seq_len": cfg.seq_len, "prompt": P,
                "parallelism": f"ep{ws}", "attention": cfg.attn,
                "l2": "no flush: the step streams the attention weights, the chosen experts and the KV cache"}
    if tp:
        return {"workload": f"{cfg.name}-shape W8A8 decode, batch 1, T=2048, tensor parallel over {ws} GPUs: "
                            f"{P}-token prompt prefilled in chunks of up to 256 rows, then {args.warmup} untimed + "
                            f"{args.steps} timed greedy decode steps",
                "model": cfg.name, "global_batch": 1, "seq_len": cfg.seq_len, "prompt": P,
                "parallelism": f"tp{ws}", "attention": cfg.attn,
                "l2": "no flush: each rank's step streams its shard of the weights and KV cache (over the L2 "
                      "size at every rank count)"}
    return {"workload": f"{cfg.name}-shape W8A8 decode, batch 1 per GPU, T={cfg.seq_len}: {P}-token prompt prefilled "
                        f"in chunks, then {args.warmup} untimed + {args.steps} timed greedy decode steps",
            "model": cfg.name, "global_batch": ws, "seq_len": cfg.seq_len, "prompt": P,
            "parallelism": f"replicas x{ws}", "attention": cfg.attn,
            "l2": "no flush: the step streams the whole model's weights (596 MB for the Qwen3 shape) and its KV "
                  "cache, over the 126 MB L2"}


def build_parser():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=13)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="Qwen3-0.6B")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sustain", type=float, default=1.0,
                    help="seconds of rewound decode windows replayed after the timed steps (0: none)")
    ap.add_argument("--cpu-steps", type=int, default=2)
    ap.add_argument("--pdl", type=int, default=1, help="programmatic dependent launch between kernels (1) or not (0)")
    ap.add_argument("--batch", type=int, default=1,
                    help="sequences per step (BatchLlamaDevice); > 1 measures batched decode instead")
    ap.add_argument("--parallel", default="tp", choices=["tp", "replicas"],
                    help="with several GPUs: one sequence tensor-parallel (tp) or independent replicas")
    ap.add_argument("--prompt", type=int, default=0,
                    help="batch 1: prompt length (default: the context filled to its last warmup + steps positions)")
    ap.add_argument("--workload", default="bench", choices=["bench", "stated"],
                    help="with --batch: 'stated' runs BASELINE.json's batched workload of the config as written "
                         "(seeded prompts fed one token per step, then greedy decode; every slot its own lengths)")
    ap.add_argument("--kernel", choices=["attn_batch", "moe_rows"],
                    help="time one kernel alone instead (profiling): attn_batch = the batched decode attention "
                         "over one layer's caches of --batch slots at position 2040; moe_rows = one layer's MoE "
                         "FFN over --batch rows (a MoE --config)")
    return ap


def main():
    args = build_parser().parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    from torch2riscv_accelerator_b200.config import CONFIGS
    cfg = CONFIGS[args.config]
    ws, rank, local = dist_init()
    if args.prompt:
        if not 1 <= args.prompt <= cfg.seq_len - args.warmup - args.steps:
            raise SystemExit(f"--prompt + warmup + steps must fit the context of {cfg.seq_len}")
    elif args.warmup + args.steps > 64:
        raise SystemExit("warmup + steps must leave a prompt of >= 1984 tokens (at most 64)")
    if args.impl == "reference":
        run_reference(args, cfg, ws, rank)
        barrier(ws)
        return
    if args.kernel:
        (run_moe_kernel if args.kernel == "moe_rows" else run_kernel)(args, cfg)
        return

    import torch

    from torch2riscv_accelerator_b200 import ops
    from torch2riscv_accelerator_b200.model import DeviceDecoder
    from torch2riscv_accelerator_b200.runtime import LlamaDevice
    torch.cuda.set_device(local)
    from torch2riscv_accelerator_b200 import _lib
    _lib.load().w8a8_set_pdl(args.pdl)
    qw = build_model(cfg, args.seed)
    if args.batch > 1 and args.workload == "stated":
        run_stated(args, cfg, qw, ws, rank, local)
        return
    if args.batch > 1:
        run_batch(args, cfg, qw, ws, rank, local)
        return
    tp, ep = split_kind(cfg, args, ws)
    if tp:
        from torch2riscv_accelerator_b200.tp import TpLlamaDevice
        dev = TpLlamaDevice((cfg, qw, qw.kv_scales))
        dec = dev.dec
    elif ep:
        from torch2riscv_accelerator_b200.ep import EpLlamaDevice
        dev = EpLlamaDevice((cfg, qw, qw.kv_scales))
        dec = dev.dec
    else:
        dec = DeviceDecoder(cfg, qw, qw.kv_scales)
        dev = LlamaDevice(dec)
    split = tp or ep
    seqs = 1 if split else ws                            # sequences decoded per step over all GPUs
    P = prompt_len(cfg, args)
    prompt = np.random.default_rng(args.seed + 3).integers(0, cfg.vocab, P)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    start_tok = int(np.argmax(dev.prefill(prompt)))
    prefill_first_s = time.perf_counter() - t0        # includes the first-call graph captures
    dev.pos = 0                                        # again, warm: the same rows rewritten with the same values
    barrier(ws)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    warm_tok = int(np.argmax(dev.prefill(prompt)))
    prefill_s = time.perf_counter() - t0
    if warm_tok != start_tok:
        raise RuntimeError("a second prefill of the prompt changed its last token")
    st = torch.cuda.current_stream()

    # ---- value: device-resident decode steps (captured step graph)
    g = dec.capture_decode_step(start_tok, P - 1)

    def rewind():
        dec.pos[0] = P - 1
        dec.set_next_token(start_tok)

    rewind()
    for _ in range(args.warmup):
        g.replay()
    barrier(ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        torch.cuda.nvtx.range_push("decode")             # ncu --nvtx-include decode/ selects these launches
        e0.record(st)
        for _ in range(args.steps):
            g.replay()
        e1.record(st)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    barrier(ws)
    dt = max_over_ranks(e0.elapsed_time(e1) / 1e3, ws)
    value = seqs * args.steps / dt
    final_pos = int(dec.pos[0].item())
    if ops.error_flags():
        raise RuntimeError("device error flags set during the decode steps")

    # ---- sustained: the window of warmup + steps positions replayed from its
    # start (the same tokens, the same cache rows rewritten with the same
    # values) for about a second, clocks sampled throughout; every rank runs
    # the same number of passes
    window = args.warmup + args.steps
    passes = max(1, int(args.sustain / (dt / args.steps * window))) if args.sustain > 0 else 0
    sustained = None
    if passes:
        barrier(ws)
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with Clocks(local) as clk_s:
            s0.record(st)
            for _ in range(passes):
                rewind()
                for _ in range(window):
                    g.replay()
            s1.record(st)
            torch.cuda.synchronize()
        barrier(ws)
        dts = max_over_ranks(s0.elapsed_time(s1) / 1e3, ws)
        if ops.error_flags():
            raise RuntimeError("device error flags set during the sustained steps")
        sustained = {"value": seqs * passes * window / dts, "unit": "tok/s", "steps": passes * window,
                     "seconds": dts, "clocks": clk_s.summary(),
                     "timing": f"CUDA events around {passes} replays of the {window}-step window (positions "
                               f"{P}..{P + window - 1}), each rewound to its first position (a device copy)"}

    # ---- e2e: LlamaDevice.forward with host inputs / outputs
    rewind()
    dev.pos = P
    tok = start_tok
    e2e_toks = [tok]
    for _ in range(args.warmup):
        tok = int(np.argmax(dev.forward(tok)))
        e2e_toks.append(tok)
    barrier(ws)
    torch.cuda.synchronize()
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0.record(st)
    for _ in range(args.steps):
        logits = dev.forward(tok)
        tok = int(np.argmax(logits))
        e2e_toks.append(tok)
    h1.record(st)
    torch.cuda.synchronize()
    barrier(ws)
    dt_e2e = max_over_ranks(h0.elapsed_time(h1) / 1e3, ws)

    # ---- parity of the measured steps: the graph's own tokens step by step
    # (untimed replays of the same graph from the same start) and its last
    # logits, against the e2e run and, at N > 1, a one-GPU decoder of the same
    # model on rank 0 (itself bit-exact with the oracle, checked at N = 1 below)
    rewind()
    graph_toks = []
    for _ in range(args.warmup + args.steps):
        g.replay()
        graph_toks.append(int(dec.next_token[0].item()))
    if not tp:                                          # the last step's greedy key (tensor parallel: per rank)
        graph_toks.append(int(0xFFFFFFFF - (int(dec.key[0].item()) & 0xFFFFFFFF)))
    graph_logits = (dec.gather_logits(1)[0] if tp else dec.logits[0]).cpu().numpy()
    parity = {"graph_tokens_equal_e2e": graph_toks == e2e_toks[:len(graph_toks)],
              "graph_logits_equal_e2e": bool(np.array_equal(graph_logits.view(np.uint32),
                                                            np.asarray(logits, np.float32).view(np.uint32)))}
    if split and rank == 0:
        ref = LlamaDevice(DeviceDecoder(cfg, qw, qw.kv_scales))
        rt = int(np.argmax(ref.prefill(prompt)))
        ref_toks = [rt]
        for _ in range(args.warmup + args.steps):
            ref_logits = ref.forward(rt)
            rt = int(np.argmax(ref_logits))
            ref_toks.append(rt)
        parity.update({"reference": "one-GPU DeviceDecoder of the same model, same prompt and steps",
                       "tokens_equal": ref_toks == e2e_toks,
                       "logits_equal": bool(np.array_equal(np.asarray(ref_logits, np.float32).view(np.uint32),
                                                           np.asarray(logits, np.float32).view(np.uint32)))})
        ref.close()

    # ---- roofline: every kernel kind of the step, the dominant one (most
    # time per step) reported
    peak, peak_src = peaks()
    table = kernel_table(dec) if not ep else []
    for k in table:
        k["frac"] = k["GBs"] / peak
        k["us_per_step"] = k["us_per_launch"] * k["launches_per_step"]
        if cfg.name == "Qwen3-0.6B" and ws == 1 and k["kind"] in NCU_TRAFFIC:
            k["traffic"] = NCU_TRAFFIC[k["kind"]]["bytes"]
    dom = max(table, key=lambda k: k["us_per_step"]) if table else None
    step_bytes = dec.weight_bytes() + dec.kv_bytes(cfg.seq_len - 8)

    # ---- CPU baseline: the oracle from the same cache state (rank 0, N = 1)
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        L = cfg.layers
        kc = np.stack([dec.kv_rows(l, cfg.seq_len)[0] for l in range(L)])
        vc = np.stack([dec.kv_rows(l, cfg.seq_len)[1] for l in range(L)])
        toks = np.random.default_rng(5).integers(0, cfg.vocab, args.cpu_steps)
        ora_logits = []
        cdt = oracle_decode(cfg, qw, qw.kv_scales, kc, vc, P, toks, logits=ora_logits)
        dev.pos = P                                     # the same steps on the GPU, from the same cache state
        gpu_logits = [dev.forward(int(t)) for t in toks]
        parity.update({"reference": f"the oracle: {args.cpu_steps} full decode steps at positions "
                                    f"{P}..{P + args.cpu_steps - 1} from the GPU's KV-cache state",
                       "logits_equal": all(np.array_equal(a.view(np.uint32), b.view(np.uint32))
                                           for a, b in zip(ora_logits, gpu_logits)),
                       "tokens_equal": [int(np.argmax(a)) for a in ora_logits] ==
                                       [int(np.argmax(b)) for b in gpu_logits]})
        cpu = {"value": args.cpu_steps / cdt, "unit": "tok/s", "cores": cpu_threads(), "kind": "port",
               "sample": f"{args.cpu_steps} full decode steps (all {L} layers + classifier) at positions "
                         f"{P}..{P + args.cpu_steps - 1} from the GPU's KV-cache state (NumPy oracle, float64 "
                         f"BLAS for exact int dots)"}

    if rank == 0:
        line = {
            "metric": metric_of(cfg, args), "value": value, "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps, "higher_is_better": True,
            "scaling": "strong" if split else "weak", "vs_baseline": value / FPGA_TOKS, "dtype": "int8",
            "data": "synthetic (N(0,0.02) weights seed 0, uniform prompt ids)",
            "config": config_of(cfg, args, ws, tp, ep),
            "e2e": {"value": seqs * args.steps / dt_e2e, "unit": "tok/s", "h2d_bytes_per_step": 8,
                    "d2h_bytes_per_step": 4 * cfg.vocab},
            "roofline": None if dom is None else {
                "bound": "hbm", "achieved": dom["GBs"], "peak": peak, "unit": "GB/s", "frac": dom["frac"],
                "traffic": NCU_TRAFFIC.get(dom["kind"], {}).get("bytes") if cfg.name == "Qwen3-0.6B" and ws == 1
                else None,
                "traffic_source": NCU_TRAFFIC.get(dom["kind"], {}).get("source", "not captured for this shape"),
                "peak_source": peak_src, "kernel": f"{dom['kernel']}: {dom['kind']}",
                "bytes_per_launch": dom["bytes_per_launch"], "us_per_launch": dom["us_per_launch"],
                "timing": "CUDA events over the kernel's launches for every layer, back to back without overlap"},
            "kernels": table,
            "step_roofline": {"bytes_per_step": step_bytes, "achieved_gbs": step_bytes / (dt / args.steps) / 1e9,
                              "frac": step_bytes / (dt / args.steps) / 1e9 / peak},
            "cpu_baseline": cpu,
            "gpu_launches": args.steps * (1 + dec.kernel_launches(1)),
            "clocks": clk.summary(),
            "sustained": sustained,
            "prefill": {"tokens": P, "seconds": prefill_s, "tok_s": P / prefill_s,
                        "first_call_seconds": prefill_first_s,
                        "timing": "host clock around LlamaDevice.prefill (synchronized), second call"},
            "final_pos": final_pos, "pdl": bool(args.pdl), "parity": parity,
        }
        print(json.dumps(line), flush=True)
        if not all(v for k, v in parity.items() if k != "reference"):
            raise RuntimeError(f"parity failed: {parity}")
    barrier(ws)
    if ws > 1:
        import torch.distributed as dist
        del g
        dec.graphs.clear()
        if split:
            dev.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
