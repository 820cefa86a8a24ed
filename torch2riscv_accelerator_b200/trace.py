"""Device timeline of the one-sequence decode step (the trace build's marks).

The B200 counterpart of the overlay's profile dump (`SA_PROFILE=1`,
`compiler/runtime/sa/sa_context.c:507-535`; event counters `rtl/sysarray/sa_perf.v`):
with the trace build of the library (`python -m torch2riscv_accelerator_b200.build
--trace`, `csrc/trace.cuh`), every CTA of the decode kernels records the global
timer and its SM clock at fixed points (entry, the return from the
programmatic-launch wait, the end of each phase). This module captures the
records of a few replays of the captured decode step and summarises them per
kernel kind: the gap from one launch's end to the next one's release, the time
from release to end, and the median duration of each phase (SM clock between
consecutive marks of a CTA, converted at the clock given).

    python -m torch2riscv_accelerator_b200.trace [--config Qwen3-0.6B] [--steps 3]
        [--batch D] [--out timeline.npy] [--sm-ghz 1.965]

--batch D traces the batched step instead (D slots at position T - 8 of
seeded random caches): the instrumented kernels it launches (embed).

Mark numbers per kernel (csrc/gemv.cu, csrc/attn.cu): GEMV 0 entry, 12
constants staged (before the wait), 1 wait returned, 6 x staged, 7 RMSNorm
factor, 8 row max, 9 scale, 2 prologue done, 10 first tile landed, 11 its dot
products, 3 tiles done, 4 epilogue, 5 SwiGLU requant; attention 0 entry, 14
cache tiles and constants staged (before the wait), 1 wait returned, 8
barrier, 10 q loaded, 11 QK-norm and RoPE, 12 q quantized, 2 K / V row and
barrier, 3 scores, 4 maxima exchanged, 13 probabilities, 5 p.V pushed, 6
partials exchanged, 7 end.
"""
import argparse
import os
import sys
from collections import defaultdict

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
TRACE_LIB = os.path.join(HERE, "libw8a8_b200_trace.so")
MARKS = 16                                         # records reserved per CTA (kTraceMarks)
KIND = {1: "gemv", 2: "attn", 3: "embed", 4: "advance"}


def _bind(rec, cnt, cap):
    from . import _lib
    _lib.check("w8a8_trace_bind", _lib.load().w8a8_trace_bind(rec.data_ptr(), cnt.data_ptr(), cap))


def _load_trace_lib():
    os.environ["W8A8_B200_LIB"] = TRACE_LIB
    from . import _lib
    if _lib._LIB is not None and _lib.LIB_PATH != TRACE_LIB:
        raise RuntimeError("the plain library is already loaded in this process")
    _lib.LIB_PATH = TRACE_LIB
    return _lib.load(TRACE_LIB)


def capture_batch(config="Qwen3-0.6B", slots=128, steps=3, seed=0):
    """The batched step (BatchDecoder, `slots` slots at position T - 8 of
    seeded random int8 caches), captured and replayed `steps` times with the
    records bound; returns (records, ms per step)."""
    lib = _load_trace_lib()
    import torch

    from .config import CONFIGS
    from .model import BatchDecoder
    from .weights import QuantWeights
    cfg = CONFIGS[config]
    qw = QuantWeights(cfg, seed=seed, calib_tokens=np.random.default_rng(seed + 1).integers(0, cfg.vocab, 16))
    dec = BatchDecoder(cfg, qw, qw.kv_scales, slots=slots)
    g = torch.Generator(device=dec.dev).manual_seed(seed + 11)
    for t in (dec.kc, dec.vc):
        t.copy_(torch.randint(-127, 128, t.shape, dtype=torch.int8, device=dec.dev, generator=g))
    dec.tokens.copy_(torch.as_tensor(np.random.default_rng(seed + 3).integers(0, cfg.vocab, slots), dtype=torch.int32))
    dec.pos.fill_(cfg.seq_len - 8)
    graph = dec.capture()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    cap = 1 << 21
    rec = torch.zeros(cap * 3, dtype=torch.int64, device=dec.dev)
    cnt = torch.zeros(1, dtype=torch.int32, device=dec.dev)
    _bind(rec, cnt, cap)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    lib.w8a8_trace_bind(None, None, 0)
    n = min(int(cnt.item()), cap)
    return rec[:n * 3].view(n, 3).cpu().numpy().view(np.uint64), e0.elapsed_time(e1) / steps


def capture(config="Qwen3-0.6B", steps=3, seed=0):
    """Prefill a seeded prompt to T - 16 positions, capture the decode step,
    replay it `steps` times with the records bound; returns the records
    [n, 3] uint64 and the mean ms per step (the trace build is slower than the
    plain one: its marks are extra stores)."""
    lib = _load_trace_lib()
    import torch

    from . import _lib
    from .config import CONFIGS
    from .model import DeviceDecoder
    from .runtime import LlamaDevice
    from .weights import QuantWeights
    cfg = CONFIGS[config]
    qw = QuantWeights(cfg, seed=seed, calib_tokens=np.random.default_rng(seed + 1).integers(0, cfg.vocab, 16))
    dec = DeviceDecoder(cfg, qw, qw.kv_scales)
    dev = LlamaDevice(dec)
    P = cfg.seq_len - 16
    start = int(np.argmax(dev.prefill(np.random.default_rng(seed + 3).integers(0, cfg.vocab, P))))
    g = dec.capture_decode_step(start, P - 1)
    dec.pos[0] = P - 1
    dec.set_next_token(start)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    cap = 1 << 20
    rec = torch.zeros(cap * 3, dtype=torch.int64, device=dec.dev)
    cnt = torch.zeros(1, dtype=torch.int32, device=dec.dev)
    _lib.check("w8a8_trace_bind", lib.w8a8_trace_bind(rec.data_ptr(), cnt.data_ptr(), cap))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    lib.w8a8_trace_bind(None, None, 0)
    n = min(int(cnt.item()), cap)
    return rec[:n * 3].view(n, 3).cpu().numpy().view(np.uint64), e0.elapsed_time(e1) / steps


def launches(raw):
    """Group the records into launches: CTAs' record blocks in reservation
    order (a launch's CTAs all reserve before the next launch's first CTA: it
    starts only after every CTA of this one has passed its wait), a new launch
    when the kernel kind or the launch's CTA count changes, a CTA index repeats
    or the launch has all its CTAs."""
    meta = raw[:, 2]
    kind = (meta >> np.uint64(56)).astype(int)
    tag = ((meta >> np.uint64(48)) & np.uint64(0xFF)).astype(int)
    grid = ((meta >> np.uint64(16)) & np.uint64(0xFFFF)).astype(int)
    cta = (meta & np.uint64(0xFFFF)).astype(int)
    out, cur = [], None
    for i in range(0, len(raw) - MARKS + 1, MARKS):
        if raw[i, 0] == 0 or tag[i] != 0:
            continue
        if (cur is None or cur["k"] != kind[i] or cur["grid"] != grid[i] or cta[i] in cur["ctas"]
                or len(cur["ctas"]) == cur["grid"]):
            cur = {"k": kind[i], "kind": KIND.get(int(kind[i]), str(kind[i])), "grid": grid[i], "ctas": {}}
            out.append(cur)
        blk = raw[i:i + MARKS]
        cur["ctas"][cta[i]] = {j: (int(blk[j, 0]), int(blk[j, 1])) for j in range(MARKS) if blk[j, 0] != 0}
    return out


def summarise(raw, sm_ghz=1.965):
    """Per kernel kind: launches, median release-after-previous-end gap (us),
    median release-to-end time (us), and the median phase durations (us)."""
    ls = launches(raw)
    rows = []
    for L in ls:
        ms = L["ctas"].values()
        rel = min((m[1][0] for m in ms if 1 in m), default=None)
        end = max(max(v[0] for v in m.values()) for m in ms)
        seg = defaultdict(list)
        for m in ms:
            order = sorted(m, key=lambda t: m[t][1])
            for a, b in zip(order, order[1:]):
                seg[f"{a}-{b}"].append((m[b][1] - m[a][1]) / sm_ghz / 1e3)
        rows.append({"kind": L["kind"], "ctas": len(L["ctas"]), "release": rel, "end": end, "seg": seg})
    kinds = defaultdict(lambda: {"n": 0, "gap": [], "crit": [], "seg": defaultdict(list), "ctas": set()})
    for a, b in zip(rows, rows[1:]):
        k = kinds[b["kind"]]
        k["n"] += 1
        k["ctas"].add(b["ctas"])
        if b["release"] is not None:
            k["gap"].append((b["release"] - a["end"]) / 1e3)
            k["crit"].append((b["end"] - b["release"]) / 1e3)
        for s, v in b["seg"].items():
            k["seg"][s].append(float(np.median(v)))
    out = {}
    for name, k in kinds.items():
        out[name] = {"launches": k["n"], "ctas": sorted(k["ctas"]),
                     "gap_us": float(np.median(k["gap"])) if k["gap"] else None,
                     "release_to_end_us": float(np.median(k["crit"])) if k["crit"] else None,
                     "phases_us": {s: round(float(np.median(v)), 2) for s, v in k["seg"].items()}}
    span = (rows[-1]["end"] - min(min(v[0][0] for v in L["ctas"].values()) for L in ls[:1])) / 1e3
    return out, span, len(rows)


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--config", default="Qwen3-0.6B")
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--batch", type=int, default=0, help="trace the batched step of this many slots")
    ap.add_argument("--out", default=None, help="save the raw records (.npy)")
    ap.add_argument("--sm-ghz", type=float, default=1.965, help="SM clock for the clock64 durations")
    a = ap.parse_args()
    raw, ms = capture_batch(a.config, a.batch, a.steps) if a.batch else capture(a.config, a.steps)
    if a.out:
        np.save(a.out, raw)
    kinds, span, n = summarise(raw, a.sm_ghz)
    print(f"{a.config}: {a.steps} replays of the decode step, {ms:.3f} ms per step (trace build), "
          f"{n} launches over {span:.1f} us")
    for name, k in kinds.items():
        gap = "-" if k["gap_us"] is None else f"{k['gap_us']:.2f}"
        rel = "-" if k["release_to_end_us"] is None else f"{k['release_to_end_us']:.2f}"
        print(f"{name:8s} launches {k['launches']:4d} CTAs {k['ctas']} gap {gap} us, release to end {rel} us")
        print(f"         phases (us): {k['phases_us']}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
