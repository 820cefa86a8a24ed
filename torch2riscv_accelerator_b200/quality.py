"""Quantization quality of the W8A8 device path against the fp32 model
(`llm/eval_quant.py`, `compiler/tests/quality_eval.py`).

The fp32 model (`weights.fp32_forward`) generates greedily from each prompt;
the device model is teacher-forced on the same tokens. Per position: top-1
agreement, the device's top-1 within the fp32 top-5, and KL(p_fp32 || p_device)
(mean and 99th percentile) -- `eval_quant.evaluate`'s measures. Free running:
the position where the device's own greedy text first differs from the fp32
text. KV scales from an fp32 calibration run on separate prompts, per layer or
per cache channel (`calibrate_kv(channel=...)`).

    python -m torch2riscv_accelerator_b200.quality --config SmolLM2-135M --layers 4 --steps 48

No checkpoints or text travel with this repository: the weights are the
seeded synthetic ones of the benchmarks and the prompts seeded token ids, so
the numbers measure the arithmetic's fidelity, not a language model's.
"""
import argparse
import json

import numpy as np

from . import weights as W

F = np.float32


def log_softmax(x):
    x = np.asarray(x, np.float64)
    m = x.max(-1, keepdims=True)
    return x - m - np.log(np.exp(x - m).sum(-1, keepdims=True))


def compare(lg32, lgd):
    """Measures of device logits lgd against fp32 logits lg32 [positions, vocab]."""
    pa, pb = log_softmax(lg32), log_softmax(lgd)
    kl = (np.exp(pa) * (pa - pb)).sum(-1)
    ta, tb = lg32.argmax(-1), lgd.argmax(-1)
    top5 = np.argsort(lg32, axis=-1)[:, -5:]
    return {"top1": float((ta == tb).mean()), "top5": float(np.mean([tb[i] in top5[i] for i in range(len(tb))])),
            "kl_mean": float(kl.mean()), "kl_p99": float(np.percentile(kl, 99)), "positions": int(len(tb))}


def fp32_generate(cfg, w, prompt, steps):
    """Greedy fp32 text: the prompt, then argmax continuations up to `steps`
    tokens; the logits of every position."""
    toks = [int(t) for t in prompt]
    while len(toks) < steps:
        toks.append(int(np.argmax(W.fp32_forward(cfg, w, toks, last_only=True)[0])))
    return toks, W.fp32_forward(cfg, w, toks)


def device_logits(dev, toks):
    """Teacher-forced device logits (dev: a LlamaDevice-like object, reset)."""
    dev.reset()
    return np.stack([dev.forward(int(t)) for t in toks])


def device_generate(dev, prompt, steps):
    dev.reset()
    toks = [int(t) for t in prompt]
    lg = None
    for p in range(steps):
        lg = dev.forward(toks[p])
        if p + 1 >= len(toks) and len(toks) < steps:
            toks.append(int(np.argmax(lg)))
    return toks


def first_divergence(a, b):
    for i, (x, y) in enumerate(zip(a, b)):
        if x != y:
            return i
    return min(len(a), len(b))


def evaluate(cfg, w, kv, prompts, steps, make_device):
    """make_device(kv) -> a LlamaDevice-like object over the quantized model."""
    refs = [fp32_generate(cfg, w, p, steps) for p in prompts]
    dev = make_device(kv)
    a = np.concatenate([lg for _, lg in refs])
    b = np.concatenate([device_logits(dev, t) for t, _ in refs])
    r = compare(a, b)
    r["first_divergence"] = [first_divergence(t, device_generate(dev, p, steps)) for (t, _), p in zip(refs, prompts)]
    return r


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--config", default="SmolLM2-135M")
    ap.add_argument("--layers", type=int, default=0, help="first layers only (0: all)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--steps", type=int, default=48, help="tokens per prompt (prompt + greedy continuation)")
    ap.add_argument("--prompts", type=int, default=4)
    ap.add_argument("--gains", default="random", help="RMSNorm gains: ones or random")
    ap.add_argument("--out", help="write the results as JSON")
    args = ap.parse_args()
    from .config import CONFIGS
    from .runtime import LlamaDevice
    cfg = CONFIGS[args.config]
    if args.layers:
        cfg = cfg.with_(layers=args.layers)
    w = W.fp32_model(cfg, args.seed, gains=args.gains)
    qw = W.from_fp32(cfg, w)
    rng = np.random.default_rng(args.seed + 7)
    calib = [rng.integers(0, cfg.vocab, 12) for _ in range(4)]
    prompts = [rng.integers(0, cfg.vocab, 6) for _ in range(args.prompts)]
    calib_runs = [fp32_generate(cfg, w, c, args.steps)[0] for c in calib]
    results = {}
    for name, channel in (("per-layer", ""), ("per-channel", "kv")):
        kv = W.calibrate_kv(cfg, w, calib_runs, channel=channel)
        r = evaluate(cfg, w, kv, prompts, args.steps, lambda k: LlamaDevice((cfg, qw, k)))
        results[name] = r
        print(f"{cfg.name} ({cfg.layers} layers) KV {name:>11}: top-1 {100 * r['top1']:5.1f}%  in fp32 top-5 "
              f"{100 * r['top5']:5.1f}%  KL mean {r['kl_mean']:.4f} p99 {r['kl_p99']:.4f}  ({r['positions']} "
              f"positions)  greedy text diverges at {r['first_divergence']}", flush=True)
    if args.out:
        with open(args.out, "w") as f:
            json.dump(results, f, indent=1)


if __name__ == "__main__":
    main()
