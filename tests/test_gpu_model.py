"""Whole-decoder parity on the GPU: the runtime (LlamaDevice over the C-ABI
kernels, CUDA graphs) against the reference's golden outputs and the oracle."""
import hashlib

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import model as OM
from torch2riscv_accelerator_b200 import config as C
from torch2riscv_accelerator_b200 import weights as W
from torch2riscv_accelerator_b200.model import DeviceDecoder
from torch2riscv_accelerator_b200.runtime import LlamaDevice

pytestmark = pytest.mark.gpu
F = np.float32


def _tiny(key):
    g = golden("dm_tiny.npz")
    dim, hidden, layers, heads, kv_heads, vocab, seq = [int(v) for v in g[f"{key}_cfg"]]
    cfg = C.ModelConfig(f"tiny-{key}", dim, hidden, layers, heads, kv_heads, dim // heads, vocab, seq,
                        theta=10000.0, eps=1e-5, tied=False, attn="norm", rope="llama2c")
    w = {n[len(key) + 3:]: g[n] for n in g.files if n.startswith(f"{key}_w_")}
    return g, cfg, w


@pytest.mark.parametrize("key", ["a", "b"])
@pytest.mark.parametrize("graphs", [True, False])
def test_decode_equals_reference_devicemodel(key, graphs):
    """Logits bit-exact with DeviceModel(SfuExact) (and SaFuncSim) every token;
    the int8 KV cache bit-exact after the run."""
    g, cfg, w = _tiny(key)
    dev = LlamaDevice((cfg, W.from_fp32(cfg, w), g[f"{key}_kv"]), graphs=graphs)
    for pos, t in enumerate(g["tokens"]):
        lg = dev.forward(int(t))
        assert lg.tobytes() == g[f"{key}_logits"][pos].tobytes(), f"pos {pos}"
    n = len(g["tokens"])
    for l in range(cfg.layers):
        k, v = dev.dec.kv_rows(l, n)
        assert np.array_equal(k, g[f"{key}_kc"][l, :n]) and np.array_equal(v, g[f"{key}_vc"][l, :n])


def test_c0_shape_equals_reference_devicemodel():
    """stories15M shape with seeded synthetic weights: sha256 of every token's
    logits equals DeviceModel(SfuExact, d=16)'s."""
    g = golden("dm_c0.npz")
    cfg = C.C0
    w = W.fp32_model(cfg, int(g["seed"]), gains="random")
    dev = LlamaDevice((cfg, W.from_fp32(cfg, w), g["kv"]))
    for pos, t in enumerate(g["tokens"]):
        lg = dev.forward(int(t))
        assert int(np.argmax(lg)) == int(g["argmax"][pos])
        assert hashlib.sha256(lg.tobytes()).hexdigest() == str(g["logits_sha"][pos]), f"pos {pos}"


def _qwen3_tiny(attn):
    cfg = C.ModelConfig("tiny-qwen3", 64, 128, 2, 4, 2, 32, 96, 64, theta=1e6, eps=1e-6, tied=True, qk_norm=True,
                        attn=attn, rope="hf")
    return cfg, W.fp32_model(cfg, 21, gains="random", std=0.2)


@pytest.mark.parametrize("attn,fixture", [("qsum", "hf_qwen3.npz"), ("norm", "qhf_qwen3.npz")])
def test_hf_path_equals_oracle_and_near_reference(attn, fixture):
    """QK-norm, GQA, tied, theta 1e6: bit-exact with the oracle; within the
    reduction-order tolerance of the reference's eager HF-path model."""
    g = golden(fixture)
    cfg, w = _qwen3_tiny(attn)
    qw = W.from_fp32(cfg, w)
    dev = LlamaDevice((cfg, qw, g["kv"]))
    ora = OM.OracleDecoder(cfg, OM.quantize_model(cfg, w), g["kv"])
    for pos, t in enumerate(g["tokens"]):
        lg = dev.forward(int(t))
        want = ora.forward(int(t), pos)
        assert lg.tobytes() == want.tobytes(), f"pos {pos}"
        ref = g["logits"][pos]
        assert np.max(np.abs(lg - ref)) <= 2e-3 * float(ref.max() - ref.min())


@pytest.mark.parametrize("attn", ["qsum", "norm"])
def test_per_channel_kv_equals_oracle(attn):
    """Per cache channel K and V scales (the reference's own calibration,
    hf_qwen3_ch.npz; hf_generic.SaCache): a 9-token prefill (the cluster
    kernel's 16-row path) then decode rows, logits and KV bit-exact with the
    oracle; QSUM within the reduction-order tolerance of the reference."""
    g = golden("hf_qwen3_ch.npz")
    cfg, w = _qwen3_tiny(attn)
    dev = LlamaDevice((cfg, W.from_fp32(cfg, w), g["kv"]))
    ora = OM.OracleDecoder(cfg, OM.quantize_model(cfg, w), g["kv"])
    toks = g["tokens"]
    assert dev.prefill(toks[:4]).tobytes() == ora.forward_rows(toks[:4], range(4)).tobytes()
    for pos in range(4, len(toks)):
        lg = dev.forward(int(toks[pos]))
        assert lg.tobytes() == ora.forward(int(toks[pos]), pos).tobytes(), f"pos {pos}"
        if attn == "qsum":
            ref = g["logits"][pos]
            assert np.max(np.abs(lg - ref)) <= 2e-3 * float(ref.max() - ref.min())
    n = len(toks)
    for l in range(cfg.layers):
        k, v = dev.dec.kv_rows(l, n)
        assert np.array_equal(k, ora.kc[l, :n]) and np.array_equal(v, ora.vc[l, :n])


def test_per_channel_kv_c2_dims_prefill_and_decode():
    """C2 dimensions with per-channel K and V scales from this repo's
    calibration: a 40-row tensor-core prefill (attention in 16-row
    sub-chunks) and decode rows, bit-exact with the oracle."""
    cfg = C.C2.with_(layers=2, vocab=4096)
    w = W.fp32_model(cfg, 2, gains="random")
    kv = W.calibrate_kv(cfg, w, np.arange(12), channel="kv")
    dev = LlamaDevice((cfg, W.from_fp32(cfg, w), kv))
    ora = OM.OracleDecoder(cfg, OM.quantize_model(cfg, w), kv)
    toks = np.random.default_rng(2).integers(0, cfg.vocab, 43)
    assert dev.prefill(toks[:40]).tobytes() == ora.forward_rows(toks[:40], range(40)).tobytes()
    for p in range(40, 43):
        assert dev.forward(int(toks[p])).tobytes() == ora.forward(int(toks[p]), p).tobytes()


@pytest.mark.parametrize("attn", ["qsum", "norm"])
def test_gelu_tanh_model_equals_oracle(attn):
    """A Gemma-style gated MLP (GELU-tanh gate, hf_generic.SaGELUTanh): a
    40-row tensor-core prefill, a 9-row chunk (the 5-16 row linear path) and
    decode rows (the GEMV path), logits and KV bit-exact with the oracle."""
    cfg = C.ModelConfig("gelu", 128, 256, 2, 8, 2, 16, 200, 128, theta=1e4, eps=1e-6, tied=True, attn=attn,
                        rope="hf", act="gelu_tanh")
    w = W.fp32_model(cfg, 8, gains="random", std=0.1)
    kv = W.calibrate_kv(cfg, w, np.arange(10))
    dev = LlamaDevice((cfg, W.from_fp32(cfg, w), kv))
    ora = OM.OracleDecoder(cfg, OM.quantize_model(cfg, w), kv)
    toks = np.random.default_rng(5).integers(0, cfg.vocab, 52)
    assert dev.prefill(toks[:40]).tobytes() == ora.forward_rows(toks[:40], range(40)).tobytes()
    assert dev.prefill(toks[40:49]).tobytes() == ora.forward_rows(toks[40:49], range(40, 49)).tobytes()
    for p in range(49, 52):
        assert dev.forward(int(toks[p])).tobytes() == ora.forward(int(toks[p]), p).tobytes()
    for l in range(cfg.layers):
        k, v = dev.dec.kv_rows(l, 52)
        assert np.array_equal(k, ora.kc[l, :52]) and np.array_equal(v, ora.vc[l, :52])


def test_prefill_chunks_equal_decode_steps():
    """A prompt prefilled in 16-row chunks (the last at P - 16) gives the same
    KV cache and last logits as feeding it token by token
    (`docs/results_v2.3.md:33-37`: prefill vs decode-only bit-exact)."""
    cfg = C.ModelConfig("pf", 128, 256, 2, 8, 2, 16, 200, 256, theta=5e5, eps=1e-5, tied=True, attn="qsum",
                        rope="hf")
    qw = W.QuantWeights(cfg, seed=5, gains="random")
    kv = np.full((cfg.layers, 2), 0.02, F)
    toks = np.random.default_rng(3).integers(0, cfg.vocab, 45)
    a = LlamaDevice((cfg, qw, kv))
    la = a.prefill(toks)
    b = LlamaDevice((cfg, qw, kv))
    for t in toks:
        lb = b.forward(int(t))
    assert la.tobytes() == lb.tobytes()
    for l in range(cfg.layers):
        ka, va = a.dec.kv_rows(l, len(toks))
        kb, vb = b.dec.kv_rows(l, len(toks))
        assert np.array_equal(ka, kb) and np.array_equal(va, vb)


@pytest.mark.parametrize("attn", ["qsum", "norm"])
def test_long_context_equals_oracle(attn):
    """Positions across the 128-position chunk boundaries (127, 128, 129, 255,
    256, 300): GPU logits and KV bit-exact with the oracle."""
    cfg = C.ModelConfig("long", 64, 128, 2, 4, 2, 16, 128, 512, theta=1e4, eps=1e-5, tied=False, attn=attn,
                        rope="hf")
    w = W.fp32_model(cfg, 9, gains="random", std=0.1)
    kv = np.array([[0.05, 0.04], [0.06, 0.05]], F)
    dev = LlamaDevice((cfg, W.from_fp32(cfg, w), kv))
    ora = OM.OracleDecoder(cfg, OM.quantize_model(cfg, w), kv)
    toks = np.random.default_rng(1).integers(0, cfg.vocab, 301)
    dev.prefill(toks[:127])
    ora.forward_rows(toks[:127], range(127))
    for p in range(127, 301):
        lg = dev.forward(int(toks[p]))
        want = ora.forward(int(toks[p]), p)
        if p in (127, 128, 129, 255, 256, 300):
            assert lg.tobytes() == want.tobytes(), f"pos {p}"
    for l in range(cfg.layers):
        k, v = dev.dec.kv_rows(l, 301)
        assert np.array_equal(k, ora.kc[l, :301]) and np.array_equal(v, ora.vc[l, :301])


def test_c2_full_dims_two_layers_equals_oracle():
    """Qwen3-0.6B dimensions (dim 1024, 16/8 heads of 128, QK-norm, hidden 3072)
    truncated to 2 layers and a 4096-token vocabulary: bit-exact with the
    oracle for a 20-token prefill and 3 decode steps."""
    cfg = C.C2.with_(layers=2, vocab=4096)
    w = W.fp32_model(cfg, 2, gains="random")
    kv = np.array([[0.04, 0.03], [0.05, 0.02]], F)
    dev = LlamaDevice((cfg, W.from_fp32(cfg, w), kv))
    ora = OM.OracleDecoder(cfg, OM.quantize_model(cfg, w), kv)
    toks = np.random.default_rng(2).integers(0, cfg.vocab, 23)
    assert dev.prefill(toks[:20]).tobytes() == ora.forward_rows(toks[:20], range(20)).tobytes()
    for p in range(20, 23):
        assert dev.forward(int(toks[p])).tobytes() == ora.forward(int(toks[p]), p).tobytes()


def test_c4_moe_two_layers_equals_oracle():
    """Granite-MoE dimensions (dim 1024, 16/8 heads of 64, 32 experts, Top-8,
    expert hidden 512) truncated to 2 layers and a 4096-token vocabulary: the
    MoE FFN bit-exact with the oracle for a 20-token prefill (the 20 rows'
    MoE grouped by expert, each row with its own Top-k) and 3 decode steps
    (the per-row kernels)."""
    cfg = C.C4.with_(layers=2, vocab=4096)
    qw = W.QuantWeights(cfg, seed=5, gains="random", calib_tokens=np.arange(8))
    dev = LlamaDevice((cfg, qw, qw.kv_scales))
    ora = OM.OracleDecoder(cfg, qw, qw.kv_scales)
    toks = np.random.default_rng(4).integers(0, cfg.vocab, 23)
    assert dev.prefill(toks[:20]).tobytes() == ora.forward_rows(toks[:20], range(20)).tobytes()
    for p in range(20, 23):
        assert dev.forward(int(toks[p])).tobytes() == ora.forward(int(toks[p]), p).tobytes()


def test_generate_greedy_matches_forward_argmax():
    g, cfg, w = _tiny("b")
    dev = LlamaDevice((cfg, W.from_fp32(cfg, w), g["b_kv"]))
    prompt = [int(t) for t in g["tokens"][:4]]
    out = list(dev.generate(prompt, steps=12, stop_at_bos=False))
    want = [int(np.argmax(g["b_logits"][p])) for p in range(3, 11)]
    assert out[:3] == prompt[1:4]
    assert out[3:4] == want[:1]


def test_device_decode_loop_equals_host_loop():
    """The captured on-device greedy step (w8a8_decode_advance + forward +
    fused classifier argmax) feeds the same tokens and leaves the same KV cache
    as the host loop of forward() + np.argmax."""
    g, cfg, w = _tiny("b")
    qw = W.from_fp32(cfg, w)
    prompt = [int(t) for t in g["tokens"][:5]]
    a = LlamaDevice((cfg, qw, g["b_kv"]))
    t0 = int(np.argmax(a.prefill(prompt)))
    fed, t = [], t0
    for _ in range(6):
        fed.append(t)
        t = int(np.argmax(a.forward(t)))
    b = DeviceDecoder(cfg, qw, g["b_kv"])
    LlamaDevice(b).prefill(prompt)
    step = b.capture_decode_step(t0, len(prompt) - 1)
    got = []
    for _ in range(6):
        step.replay()
        got.append(int(b.next_token[0].item()))
    assert got == fed
    for l in range(cfg.layers):
        ka, va = a.dec.kv_rows(l, 11)
        kb, vb = b.kv_rows(l, 11)
        assert np.array_equal(ka, kb) and np.array_equal(va, vb)


def test_pdl_on_and_off_give_identical_results():
    """Programmatic dependent launch only changes when kernels start: the logits
    and cache of a prefill + decode run are the same bytes with and without it."""
    from torch2riscv_accelerator_b200 import _lib
    cfg = C.C2.with_(layers=2, vocab=2048, seq_len=256)
    qw = W.QuantWeights(cfg, seed=4, gains="random")
    kv = np.array([[0.04, 0.03], [0.05, 0.02]], F)
    toks = np.random.default_rng(6).integers(0, cfg.vocab, 40)
    out = []
    lib = _lib.load()
    old = lib.w8a8_set_pdl(1)
    try:
        for pdl in (1, 0):
            lib.w8a8_set_pdl(pdl)
            d = LlamaDevice((cfg, qw, kv))
            lg = [d.prefill(toks[:33])] + [d.forward(int(t)) for t in toks[33:]]
            out.append((np.stack(lg), d.dec.kv_rows(1, 40)))
    finally:
        lib.w8a8_set_pdl(old)
    assert out[0][0].tobytes() == out[1][0].tobytes()
    assert np.array_equal(out[0][1][0], out[1][1][0]) and np.array_equal(out[0][1][1], out[1][1][1])
