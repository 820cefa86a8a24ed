#!/usr/bin/env python3
"""Generate the golden fixtures that pin the oracle to the reference.

Runs the reference's OWN code (Torch2RISCV-accelerator, imported unchanged
from the checkout named by the REF_ROOT environment variable, which is
required) and saves its inputs and outputs as
small .npz files beside this script. Only this generator touches the reference;
the tests read the .npz files (the reference is absent on GPU boxes).

Fixtures:
  sfu.npz       llm/sfu.py exp / recip / rsqrt on random bit patterns, ranges
                and specials; the SFU tables (sfu.tables()).
  convert.npz   ref_model.to_i8 and ref_model.quantize_rows.
  dm_tiny.npz   two random tiny models (llm/test_l4.tiny_model, D = 16): fp32
                weights, KV scales, tokens; DeviceModel(SfuExact, d=16) logits
                and int8 KV cache per token; the compile_model list run in
                SaFuncSim is checked bit-exact against them here.
  dm_c0.npz     the stories15M-shape model with this repo's seeded synthetic
                weights: DeviceModel(SfuExact, d=16) logits per token (sha256
                of the bytes, argmax, a slice), KV cache sha256, with
                SaFuncSim agreement checked here on the first tokens.
  hf_qwen3.npz  a tiny Qwen3 (QK-norm, GQA, tied, theta 1e6) through
                hf_generic.SaDecoder (QSUM attention) under the device SFU.
  qhf_qwen3.npz the same weights through qhf.QModel (NORM attention) under the
                device SFU.
  hf_qwen3_ch.npz  the same tiny Qwen3 with KV scales per cache channel from
                hf_generic.calibrate_kv(channel="kv"), through SaDecoder
  gelu.npz      hf_generic.SaGELUTanh (GELU-tanh gate) under the device SFU
  moe.npz       hf_generic.QMixtralMoe rows of a synthetic Mixtral block
                (compiler/tests/test_hf_moe.synthetic_model's shape).
  tiny_a_d8.w8a8  tiny model "a" of dm_tiny.npz written by the reference's
                exporter (llm/export_w8a8.export, D = 8).
  sampler.npz   llm/runtime.py's Sampler (run.c's sampler) token streams on
                seeded logits for several temperatures, top-p values and seeds.
  tiny_a.bin    the same fp32 weights as a llama2.c legacy checkpoint
                (separate classifier), checked against llm/checkpoint.load.

    REF_ROOT=<reference checkout> python tests/golden/make_golden.py [--skip-c0]
"""
import argparse
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.abspath(os.path.join(HERE, "..", ".."))
REF = os.environ.get("REF_ROOT")
if not REF or not os.path.isdir(os.path.join(REF, "llm")):
    raise SystemExit("set REF_ROOT to a checkout of Torch2RISCV-accelerator (the directory holding llm/)")
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REF, "llm"))
sys.path.insert(0, os.path.join(REF, "driver"))
sys.path.insert(0, os.path.join(REF, "compiler", "frontend"))
sys.path.insert(0, os.path.join(REF, "compiler", "tests"))

F = np.float32
D = 16


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def save(name, **arrays):
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **arrays)
    print(f"  wrote {name}: {os.path.getsize(path) / 1024:.1f} KB")


def gen_sfu():
    import fp32 as RF
    import sfu as RS
    rng = np.random.default_rng(5)
    x = np.concatenate([
        rng.integers(0, 2**32, 4096, dtype=np.uint64).astype(np.uint32),
        rng.uniform(-110, 95, 4096).astype(F).view(np.uint32),
        np.exp(rng.uniform(-85, 85, 4096)).astype(F).view(np.uint32),
        (-np.exp(rng.uniform(-85, 85, 1024))).astype(F).view(np.uint32),
        np.array([0, 0x80000000, 0x7F800000, 0xFF800000, 0x7FC00000, 0x7F800001, 1, 0x807FFFFF, 0x00800000,
                  0x3F800000, 0xBF800000, 0x42B20000, 0xC2D00000, 0x42B1FFFF, 0xC2CFFFFF, 0x7F7FFFFF,
                  0xFF7FFFFF, 0x3F000000, 0x40000000, 0x40800000], np.uint32)])
    t = RS.tables()
    save("sfu.npz", x=x, exp=RS.exp(x), recip=RS.recip(x), rsqrt=RS.rsqrt(x),
         **{f"T_{k}": v[0] for k, v in t.items()}, **{f"S_{k}": v[1] for k, v in t.items()},
         fabs=RS.fabs(x), add=RF.add(x[:4096], x[4096:8192]), mul=RF.mul(x[:4096], x[4096:8192]))


def gen_convert():
    from ref_model import quantize_rows, to_i8
    rng = np.random.default_rng(6)
    v = np.concatenate([rng.uniform(-200, 200, 4096), np.arange(-260, 261) * 0.5,
                        [np.nan, np.inf, -np.inf, -0.0, 0.0, 126.5, 127.5, -127.5, 1e30, -1e30]]).astype(F)
    w = (rng.standard_normal((48, 40)) * np.exp(rng.uniform(-6, 3, (48, 1)))).astype(F)
    q, s = quantize_rows(w)
    save("convert.npz", v=v, i8=to_i8(v), w=w, q=q, s=s)


def tiny_models():
    import test_l4
    a = test_l4.tiny_model(seed=3)
    b = test_l4.tiny_model(seed=11, dim=64, hidden=128, heads=4, kv_heads=2)
    return {"a": a, "b": b}


def run_funcsim(cfg, w, kv, tokens):
    """compile_model's list in SaFuncSim at D = 16: logits and KV per token."""
    import tempfile

    import compile_model as CM
    import test_l4
    from export_w8a8 import W8A8, export
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "m.w8a8")
        export(cfg, w, kv, D, path)
        m = W8A8(path)
        dl = CM.ModelCompiler(m).build()
        rig = test_l4.Rig(m, len(dl))
        out = []
        for pos, t in enumerate(tokens):
            rig.run(dl, pos, int(t))
            out.append((rig.logits().copy(), rig.kv_cache().copy()))
        return out


def gen_dm_tiny():
    from ref_model import DeviceModel, SfuExact
    arrays = {}
    toks = np.random.default_rng(7).integers(0, 64, 16)
    for key, (cfg, w, kv) in tiny_models().items():
        dm = DeviceModel(cfg, w, kv, d=D, sfu=SfuExact)
        logits = np.stack([dm.forward(int(t), pos) for pos, t in enumerate(toks)]).astype(F)
        fs = run_funcsim(cfg, w, kv, toks)
        for pos in range(len(toks)):
            assert fs[pos][0].tobytes() == logits[pos].tobytes(), f"funcsim != DeviceModel at pos {pos}"
        kc = fs[-1][1]
        assert np.array_equal(kc[:, 0, :len(toks)], dm.kc[:, :len(toks)])
        print(f"  tiny {key}: SaFuncSim == DeviceModel(SfuExact) for {len(toks)} tokens (logits, KV)")
        arrays[f"{key}_cfg"] = np.array([cfg.dim, cfg.hidden, cfg.layers, cfg.heads, cfg.kv_heads, cfg.vocab,
                                         cfg.seq_len])
        for n, v in w.items():
            arrays[f"{key}_w_{n}"] = np.asarray(v, F)
        arrays[f"{key}_kv"] = kv
        arrays[f"{key}_logits"] = logits
        arrays[f"{key}_kc"] = dm.kc
        arrays[f"{key}_vc"] = dm.vc
    arrays["tokens"] = toks
    save("dm_tiny.npz", **arrays)


C0_SEED, C0_TOKENS, C0_FUNCSIM = 1234, 4, 2


def c0_weights():
    """stories15M-shape fp32 weights from this repo's seeded generator (gains
    1 + 0.1 N, so the norm gains are exercised)."""
    import checkpoint
    from torch2riscv_accelerator_b200.config import C0
    from torch2riscv_accelerator_b200.weights import gen_tensor
    cfg = checkpoint.Config(C0.dim, C0.hidden, C0.layers, C0.heads, C0.kv_heads, C0.vocab, C0.seq_len)
    g = lambda n, l=-1: gen_tensor(C0, C0_SEED, n, l, gains="random")
    w = {"tok": g("tok"), "rms_final": g("rms_final")}
    for n in ("rms_att", "rms_ffn", "wq", "wk", "wv", "wo", "w1", "w2", "w3"):
        w[n] = np.stack([g(n, l) for l in range(C0.layers)])
    w["wcls"] = w["tok"]
    return cfg, w


def gen_dm_c0():
    from ref_model import DeviceModel, Fp32Model, SfuExact
    cfg, w = c0_weights()
    rng = np.random.default_rng(8)
    calib = rng.integers(0, cfg.vocab, 16)
    fm = Fp32Model(cfg, w)
    for pos, t in enumerate(calib):
        fm.forward(int(t), pos)
    kv = (np.stack([np.abs(fm.kc).max(axis=(1, 2)), np.abs(fm.vc).max(axis=(1, 2))], 1) / F(127)).astype(F)
    toks = rng.integers(0, cfg.vocab, C0_TOKENS)
    dm = DeviceModel(cfg, w, kv, d=D, sfu=SfuExact)
    logits = [dm.forward(int(t), pos).astype(F) for pos, t in enumerate(toks)]
    fs = run_funcsim(cfg, w, kv, toks[:C0_FUNCSIM])
    for pos in range(C0_FUNCSIM):
        assert fs[pos][0].tobytes() == logits[pos].tobytes(), f"C0 funcsim != DeviceModel at pos {pos}"
    print(f"  C0: SaFuncSim == DeviceModel(SfuExact) for {C0_FUNCSIM} tokens")
    n = len(toks)
    save("dm_c0.npz", seed=C0_SEED, kv=kv, tokens=toks, argmax=np.array([int(np.argmax(x)) for x in logits]),
         logits_sha=np.array([sha(x) for x in logits]), head=np.stack([x[:64] for x in logits]),
         kc_sha=sha(dm.kc[:, :n]), vc_sha=sha(dm.vc[:, :n]), funcsim_tokens=C0_FUNCSIM)


# ------------------------------------------------------------ HF-path fixtures
QCFG = dict(dim=64, hidden=128, layers=2, heads=4, kv_heads=2, head_dim=32, vocab=96, seq_len=64, theta=1e6,
            eps=1e-6, seed=21)


def qwen3_weights():
    """Tiny Qwen3 fp32 weights in the interleaved-pair RoPE layout of this repo
    (llama2.c's), from the repo's seeded generator with random gains."""
    from torch2riscv_accelerator_b200.config import ModelConfig
    from torch2riscv_accelerator_b200.weights import gen_tensor
    q = QCFG
    cfg = ModelConfig("tiny-qwen3", q["dim"], q["hidden"], q["layers"], q["heads"], q["kv_heads"], q["head_dim"],
                      q["vocab"], q["seq_len"], theta=q["theta"], eps=q["eps"], tied=True, qk_norm=True, attn="qsum",
                      rope="hf")
    g = lambda n, l=-1: gen_tensor(cfg, q["seed"], n, l, gains="random", std=0.2)
    w = {"tok": g("tok"), "rms_final": g("rms_final")}
    for n in ("rms_att", "rms_ffn", "wq", "wk", "wv", "wo", "w1", "w2", "w3", "q_norm", "k_norm"):
        w[n] = np.stack([g(n, l) for l in range(cfg.layers)])
    return cfg, w


def _deinterleave_rows(x, heads, hd):
    """interleaved pairs -> HF rotate-half halves (the inverse of the
    reference's interleave permutation, `hf_generic.interleave_perm` :753-756)."""
    x = np.asarray(x)
    sh = x.shape
    return x.reshape(heads, hd // 2, 2, *sh[1:]).swapaxes(1, 2).reshape(sh)


def calib_kv(cfg, w, toks):
    """Static per-layer KV scales from qhf.calibrate_kv (the reference's fp32 run)."""
    import qhf
    hc = hf_cfg(cfg)
    wq = dict(w)
    wq["wcls"] = w["tok"]
    return qhf.calibrate_kv(hc, wq, [int(t) for t in toks])


def hf_cfg(cfg):
    import types
    return types.SimpleNamespace(arch="Qwen3ForCausalLM", dim=cfg.dim, hidden=cfg.hidden, layers=cfg.layers,
                                 heads=cfg.heads, kv_heads=cfg.kv_heads, head_size=cfg.head_dim, vocab=cfg.vocab,
                                 theta=cfg.theta, eps=cfg.eps, tie=True, qk_norm=True, seq_len=cfg.seq_len,
                                 q_dim=cfg.q_dim, kv_dim=cfg.kv_dim)


def gen_hf():
    import torch
    import hf_generic as H
    import qhf
    import test_hf_generic as THG
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from torch2riscv_accelerator_b200.weights import rope_tables
    torch.set_grad_enabled(False)
    cfg, w = qwen3_weights()
    rng = np.random.default_rng(22)
    kv = calib_kv(cfg, w, rng.integers(0, cfg.vocab, 24))
    toks = rng.integers(0, cfg.vocab, 10)
    # qhf.QModel (NORM attention) under the device SFU
    wq = dict(w)
    wq["wcls"] = w["tok"]
    qm = qhf.QModel(hf_cfg(cfg), wq, kv)
    cos, sin = rope_tables(cfg)
    assert np.array_equal(qm.rope_cos.numpy(), cos) and np.array_equal(qm.rope_sin.numpy(), sin)
    with qhf.device_sfu():
        qlog = np.stack([qm(torch.tensor([int(t)]), torch.tensor([p]), torch.zeros(cfg.seq_len)).numpy()
                         for p, t in enumerate(toks)]).astype(F)
    # hf_generic.SaDecoder (QSUM attention) on an HF Qwen3 with the same weights
    hc = Qwen3Config(vocab_size=cfg.vocab, hidden_size=cfg.dim, intermediate_size=cfg.hidden,
                     num_hidden_layers=cfg.layers, num_attention_heads=cfg.heads, num_key_value_heads=cfg.kv_heads,
                     head_dim=cfg.head_dim, max_position_embeddings=cfg.seq_len, tie_word_embeddings=True,
                     rms_norm_eps=cfg.eps, rope_theta=cfg.theta, attention_bias=False)
    m = Qwen3ForCausalLM(hc).eval()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, F))
    m.model.embed_tokens.weight.copy_(t(w["tok"]))
    m.model.norm.weight.copy_(t(w["rms_final"]))
    for l, layer in enumerate(m.model.layers):
        a = layer.self_attn
        a.q_proj.weight.copy_(t(_deinterleave_rows(w["wq"][l], cfg.heads, cfg.head_dim)))
        a.k_proj.weight.copy_(t(_deinterleave_rows(w["wk"][l], cfg.kv_heads, cfg.head_dim)))
        a.v_proj.weight.copy_(t(w["wv"][l]))
        a.o_proj.weight.copy_(t(w["wo"][l]))
        a.q_norm.weight.copy_(t(_deinterleave_rows(w["q_norm"][l], 1, cfg.head_dim)))
        a.k_norm.weight.copy_(t(_deinterleave_rows(w["k_norm"][l], 1, cfg.head_dim)))
        layer.mlp.gate_proj.weight.copy_(t(w["w1"][l]))
        layer.mlp.up_proj.weight.copy_(t(w["w3"][l]))
        layer.mlp.down_proj.weight.copy_(t(w["w2"][l]))
        layer.input_layernorm.weight.copy_(t(w["rms_att"][l]))
        layer.post_attention_layernorm.weight.copy_(t(w["rms_ffn"][l]))
    H.rope_rewrite(m, cfg.seq_len)
    H.norm_rewrite(m)
    H.quantize(m)
    for mod in m.modules():                        # the repo's tables (qhf.rope_tables' method)
        if isinstance(mod, H.RopeTable):
            mod.cos_t.copy_(t(cos))
            mod.sin_t.copy_(t(sin))
    dec = H.SaDecoder(m, cfg.seq_len, kv)
    with THG.device_sfu():
        hlog = np.stack([dec(torch.tensor([[int(tk)]]), torch.tensor([[p]]))[0, 0].numpy()
                         for p, tk in enumerate(toks)]).astype(F)
    L, T = cfg.layers, len(toks)
    kc = dec.kc.numpy().reshape(L, cfg.seq_len, cfg.kv_dim)[:, :T]
    save("hf_qwen3.npz", kv=kv, tokens=toks, logits=hlog, kc=kc)
    save("qhf_qwen3.npz", kv=kv, tokens=toks, logits=qlog)
    print(f"  hf QSUM argmax {hlog.argmax(1).tolist()}, qhf NORM argmax {qlog.argmax(1).tolist()}")


def gen_hf_channel():
    """Per cache channel KV scales: the reference's own calibration
    (hf_generic.calibrate_kv(channel="kv") on the fp32 model after the RoPE /
    norm rewrites) and its SaDecoder (QSUM attention, SaCache per-channel
    constants) under the device SFU, on the tiny Qwen3 of gen_hf."""
    import torch
    import hf_generic as H
    import test_hf_generic as THG
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from torch2riscv_accelerator_b200.weights import rope_tables
    torch.set_grad_enabled(False)
    cfg, w = qwen3_weights()
    rng = np.random.default_rng(23)
    calib = rng.integers(0, cfg.vocab, 40)
    toks = rng.integers(0, cfg.vocab, 10)
    hc = Qwen3Config(vocab_size=cfg.vocab, hidden_size=cfg.dim, intermediate_size=cfg.hidden,
                     num_hidden_layers=cfg.layers, num_attention_heads=cfg.heads, num_key_value_heads=cfg.kv_heads,
                     head_dim=cfg.head_dim, max_position_embeddings=cfg.seq_len, tie_word_embeddings=True,
                     rms_norm_eps=cfg.eps, rope_theta=cfg.theta, attention_bias=False)
    m = Qwen3ForCausalLM(hc).eval()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, F))
    m.model.embed_tokens.weight.copy_(t(w["tok"]))
    m.model.norm.weight.copy_(t(w["rms_final"]))
    for l, layer in enumerate(m.model.layers):
        a = layer.self_attn
        a.q_proj.weight.copy_(t(_deinterleave_rows(w["wq"][l], cfg.heads, cfg.head_dim)))
        a.k_proj.weight.copy_(t(_deinterleave_rows(w["wk"][l], cfg.kv_heads, cfg.head_dim)))
        a.v_proj.weight.copy_(t(w["wv"][l]))
        a.o_proj.weight.copy_(t(w["wo"][l]))
        a.q_norm.weight.copy_(t(_deinterleave_rows(w["q_norm"][l], 1, cfg.head_dim)))
        a.k_norm.weight.copy_(t(_deinterleave_rows(w["k_norm"][l], 1, cfg.head_dim)))
        layer.mlp.gate_proj.weight.copy_(t(w["w1"][l]))
        layer.mlp.up_proj.weight.copy_(t(w["w3"][l]))
        layer.mlp.down_proj.weight.copy_(t(w["w2"][l]))
        layer.input_layernorm.weight.copy_(t(w["rms_att"][l]))
        layer.post_attention_layernorm.weight.copy_(t(w["rms_ffn"][l]))
    H.rope_rewrite(m, cfg.seq_len)
    H.norm_rewrite(m)
    cos, sin = rope_tables(cfg)
    for mod in m.modules():                        # the repo's tables (qhf.rope_tables' method)
        if isinstance(mod, H.RopeTable):
            mod.cos_t.copy_(t(cos))
            mod.sin_t.copy_(t(sin))
    kv = H.calibrate_kv(m, [int(x) for x in calib], cfg.seq_len, channel="kv")
    assert kv.shape == (cfg.layers, 2, cfg.kv_dim)
    H.quantize(m)
    dec = H.SaDecoder(m, cfg.seq_len, kv)
    with THG.device_sfu():
        hlog = np.stack([dec(torch.tensor([[int(tk)]]), torch.tensor([[p]]))[0, 0].numpy()
                         for p, tk in enumerate(toks)]).astype(F)
    L, T = cfg.layers, len(toks)
    kc = dec.kc.numpy().reshape(L, cfg.seq_len, cfg.kv_dim)[:, :T]
    save("hf_qwen3_ch.npz", kv=kv, calib=calib, tokens=toks, logits=hlog, kc=kc)
    print(f"  hf QSUM per-channel argmax {hlog.argmax(1).tolist()}")


def gen_gelu():
    """hf_generic.SaGELUTanh (the GELU-tanh gate of Gemma-class models) under the
    device SFU on ranges, random values and special values."""
    import torch
    import hf_generic as H
    import test_hf_generic as THG
    torch.set_grad_enabled(False)
    rng = np.random.default_rng(31)
    x = np.concatenate([np.linspace(-12, 12, 2401, dtype=F), (rng.standard_normal(4000) * 3).astype(F),
                        np.array([0.0, -0.0, 1e-30, -1e-30, 60.0, -60.0, 1e4, -1e4, 3e38, -3e38, np.inf, -np.inf,
                                  np.nan], F)]).astype(F)
    with THG.device_sfu():
        y = H.SaGELUTanh()(torch.from_numpy(x)).numpy().astype(F)
    save("gelu.npz", x=x, y=y, a=np.float32(H.SaGELUTanh.A), b=np.float32(H.SaGELUTanh.B))


def gen_moe():
    import torch
    import hf_generic as H
    import test_hf_generic as THG
    import test_hf_moe
    torch.set_grad_enabled(False)
    m = test_hf_moe.synthetic_model()
    block = m.model.layers[0].mlp
    q = H.QMixtralMoe(block)
    torch.manual_seed(1)
    x = torch.randn(12, 1, block.gate.weight.shape[1])
    ys, ids, ws = [], [], []
    with THG.device_sfu():
        for r in range(x.shape[0]):
            _, i, wt = q.route(x[r])
            ys.append(q._row(x[r]).numpy()[0])
            ids.append(i.numpy()[0])
            ws.append(wt.numpy()[0])
    E = q.E
    save("moe.npz", x=x.numpy()[:, 0], y=np.stack(ys).astype(F), ids=np.stack(ids), w=np.stack(ws).astype(F),
         rq=q.rq.numpy()[:E], rs=q.rs.numpy()[:E], gq=q.gq.numpy(), gs=q.gs.numpy(), uq=q.uq.numpy(),
         us=q.us.numpy(), dq=q.dq.numpy(), ds=q.ds.numpy(), top_k=q.k)


def gen_sampler():
    """llm/runtime.py's Sampler (run.c's xorshift / softmax / top-p) on seeded
    logits rows: the token stream of each (temperature, topp, seed)."""
    src = open(os.path.join(REF, "llm", "runtime.py")).read()
    a = src.index("class Sampler")
    b = src.index("\nclass ", a + 1)
    ns = {"np": np, "F": F}
    exec(src[a:b], ns)                       # the class alone (the module imports the board tooling)
    rng = np.random.default_rng(17)
    logits = (rng.standard_normal((48, 512)) * 3).astype(F)
    logits[::5, :12] = logits[::5, :1]       # tied maxima and tied probabilities
    cfgs = np.array([(0.0, 0.9, 1), (1.0, 0.9, 1), (0.7, 0.95, 7), (1.3, 0.0, 3), (0.5, 1.0, 0), (1.0, 0.5, 42),
                     (2.0, 0.99, 5)], np.float64)
    streams = []
    for t, p, seed in cfgs:
        smp = ns["Sampler"](float(t), float(p), int(seed))
        streams.append([smp(row) for row in logits])
    save("sampler.npz", logits=logits, cfgs=cfgs, tokens=np.array(streams, np.int64))


def gen_files():
    import checkpoint
    from export_w8a8 import export
    from torch2riscv_accelerator_b200 import config as C
    from torch2riscv_accelerator_b200.loaders import write_llama2c
    cfg, w, kv = tiny_models()["a"]
    out = os.path.join(HERE, "tiny_a_d8.w8a8")
    n = export(cfg, w, kv, 8, out)
    print(f"  {out}: {n} bytes (reference exporter, D = 8)")
    mc = C.ModelConfig("tiny-a", cfg.dim, cfg.hidden, cfg.layers, cfg.heads, cfg.kv_heads, cfg.head_size, cfg.vocab,
                       cfg.seq_len, theta=10000.0, eps=1e-5, tied=False, attn="norm", rope="llama2c")
    path = os.path.join(HERE, "tiny_a.bin")
    write_llama2c(path, mc, {k: np.asarray(v, F) for k, v in w.items()})
    rc, rw = checkpoint.load(path)
    assert (rc.dim, rc.hidden, rc.layers, rc.heads, rc.kv_heads, rc.vocab, rc.seq_len) == \
        (cfg.dim, cfg.hidden, cfg.layers, cfg.heads, cfg.kv_heads, cfg.vocab, cfg.seq_len)
    for k in w:
        assert np.array_equal(np.asarray(rw[k]), np.asarray(w[k], F)), k
    print(f"  {path}: llm/checkpoint.load reads it back exactly")


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--skip-c0", action="store_true")
    ap.add_argument("--only", help="comma list: sfu,convert,tiny,c0,hf,hfch,gelu,moe,sampler,files")
    a = ap.parse_args()
    only = set(a.only.split(",")) if a.only else None
    steps = [("sfu", gen_sfu), ("convert", gen_convert), ("tiny", gen_dm_tiny), ("c0", gen_dm_c0),
             ("hf", gen_hf), ("hfch", gen_hf_channel), ("gelu", gen_gelu), ("moe", gen_moe), ("sampler", gen_sampler),
             ("files", gen_files)]
    for name, fn in steps:
        if (only and name not in only) or (name == "c0" and a.skip_c0):
            continue
        print(name)
        fn()


if __name__ == "__main__":
    main()
