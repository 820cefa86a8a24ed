"""The oracle pinned to the reference's own outputs (tests/golden/*.npz, made
by tests/golden/make_golden.py from the reference's code). CPU only."""
import hashlib

import numpy as np
import pytest

from conftest import golden
from oracle import model as OM
from oracle import numerics as N
from torch2riscv_accelerator_b200 import config as C
from torch2riscv_accelerator_b200 import weights as W

F = np.float32


def test_sfu_tables_match_reference():
    g = golden("sfu.npz")
    t = N.sfu_tables()
    for k in ("exp", "recip", "rsqrt"):
        assert np.array_equal(N.bits(t[k][0]), g[f"T_{k}"]), k
        assert np.array_equal(N.bits(t[k][1]), g[f"S_{k}"]), k


@pytest.mark.parametrize("fn", ["exp", "recip", "rsqrt"])
def test_sfu_bit_exact(fn):
    g = golden("sfu.npz")
    x = g["x"].view(F)
    got = N.bits(getattr(N, "sfu_" + fn)(x))
    bad = np.flatnonzero(got != g[fn])
    assert bad.size == 0, [(hex(g["x"][i]), hex(g[fn][i]), hex(got[i])) for i in bad[:5]]


def test_fp32_add_mul_match_reference_in_normal_range():
    g = golden("sfu.npz")
    a, b = g["x"][:4096].view(F), g["x"][4096:8192].view(F)
    with np.errstate(all="ignore"):
        add, mul = N.bits((a + b).astype(F)), N.bits((a * b).astype(F))
    for got, want in ((add, g["add"]), (mul, g["mul"])):
        e = (want >> 23) & 0xFF
        nan = (e == 255) & ((want & 0x7FFFFF) != 0)
        normal = (e != 0) & ~nan
        assert np.array_equal(got[normal], want[normal])


def test_to_i8_and_quantize_rows():
    g = golden("convert.npz")
    assert np.array_equal(N.to_i8(g["v"]), g["i8"])
    q, s = N.quantize_rows(g["w"])
    assert np.array_equal(q, g["q"]) and np.array_equal(N.bits(s), N.bits(g["s"]))
    q2, s2 = W.quantize_rows(g["w"])                 # the product's offline quantizer agrees
    assert np.array_equal(q2, g["q"]) and np.array_equal(N.bits(s2), N.bits(g["s"]))


def _tiny(key, g):
    dim, hidden, layers, heads, kv_heads, vocab, seq = [int(v) for v in g[f"{key}_cfg"]]
    cfg = C.ModelConfig(f"tiny-{key}", dim, hidden, layers, heads, kv_heads, dim // heads, vocab, seq,
                        theta=10000.0, eps=1e-5, tied=False, attn="norm", rope="llama2c")
    w = {n[len(key) + 3:]: g[n] for n in g.files if n.startswith(f"{key}_w_")}
    return cfg, w


@pytest.mark.parametrize("key", ["a", "b"])
def test_oracle_equals_devicemodel_tiny(key):
    """Bit-exact with DeviceModel(SfuExact, d=16) (and so with SaFuncSim,
    checked when the fixture was made): logits and the int8 KV cache per token."""
    g = golden("dm_tiny.npz")
    cfg, w = _tiny(key, g)
    dec = OM.OracleDecoder(cfg, OM.quantize_model(cfg, w), g[f"{key}_kv"])
    for pos, t in enumerate(g["tokens"]):
        lg = dec.forward(int(t), pos)
        assert lg.tobytes() == g[f"{key}_logits"][pos].tobytes(), f"pos {pos}"
    n = len(g["tokens"])
    assert np.array_equal(dec.kc[:, :n], g[f"{key}_kc"][:, :n])
    assert np.array_equal(dec.vc[:, :n], g[f"{key}_vc"][:, :n])


def test_oracle_prefill_rows_equal_decode_rows():
    """A chunk of rows gives the decode steps' KV cache and last logits
    (`compiler/frontend/qhf.py:356-364`: each row computed as a decode step)."""
    g = golden("dm_tiny.npz")
    cfg, w = _tiny("b", g)
    qw = OM.quantize_model(cfg, w)
    toks = [int(t) for t in g["tokens"]]
    d1 = OM.OracleDecoder(cfg, qw, g["b_kv"])
    lg = d1.forward_rows(toks[:8], range(8))
    lg2 = d1.forward_rows(toks[8:], range(8, 16))
    assert lg.tobytes() == g["b_logits"][7].tobytes() and lg2.tobytes() == g["b_logits"][15].tobytes()
    assert np.array_equal(d1.kc[:, :16], g["b_kc"][:, :16])


def _c0_weights(seed):
    cfg = C.C0
    g = lambda n, l=-1: W.gen_tensor(cfg, seed, n, l, gains="random")
    w = {"tok": g("tok"), "rms_final": g("rms_final")}
    for n in ("rms_att", "rms_ffn", "wq", "wk", "wv", "wo", "w1", "w2", "w3"):
        w[n] = np.stack([g(n, l) for l in range(cfg.layers)])
    return cfg, w


def test_oracle_equals_devicemodel_c0_shape():
    """stories15M shape, seeded synthetic weights: logits bit-exact (sha256 of
    the bytes) and KV cache bit-exact with DeviceModel(SfuExact, d=16)."""
    g = golden("dm_c0.npz")
    cfg, w = _c0_weights(int(g["seed"]))
    dec = OM.OracleDecoder(cfg, OM.quantize_model(cfg, w), g["kv"])
    toks = g["tokens"]
    for pos, t in enumerate(toks):
        lg = dec.forward(int(t), pos)
        assert int(np.argmax(lg)) == int(g["argmax"][pos])
        assert np.array_equal(lg[:64], g["head"][pos])
        assert hashlib.sha256(lg.tobytes()).hexdigest() == str(g["logits_sha"][pos]), f"pos {pos}"
    n = len(toks)
    assert hashlib.sha256(np.ascontiguousarray(dec.kc[:, :n]).tobytes()).hexdigest() == str(g["kc_sha"])
    assert hashlib.sha256(np.ascontiguousarray(dec.vc[:, :n]).tobytes()).hexdigest() == str(g["vc_sha"])


def _qwen3():
    cfg = C.ModelConfig("tiny-qwen3", 64, 128, 2, 4, 2, 32, 96, 64, theta=1e6, eps=1e-6, tied=True,
                        qk_norm=True, attn="qsum", rope="hf")
    g = lambda n, l=-1: W.gen_tensor(cfg, 21, n, l, gains="random", std=0.2)
    w = {"tok": g("tok"), "rms_final": g("rms_final")}
    for n in ("rms_att", "rms_ffn", "wq", "wk", "wv", "wo", "w1", "w2", "w3", "q_norm", "k_norm"):
        w[n] = np.stack([g(n, l) for l in range(cfg.layers)])
    return cfg, w


@pytest.mark.parametrize("variant,fixture", [("qsum", "hf_qwen3.npz"), ("norm", "qhf_qwen3.npz"),
                                             ("qsum", "hf_qwen3_ch.npz")])
def test_oracle_close_to_hf_path(variant, fixture):
    """QK-norm + GQA + tied + theta 1e6: the oracle against the reference's
    eager HF-path models under the device SFU (hf_generic.SaDecoder for QSUM,
    qhf.QModel for NORM). Those sum in torch's order, the device (and the
    oracle) in the D = 16 lane order, so the check is "up to reduction order"
    (`compiler/tests/test_c55.py`): logits within 2e-3 of the logit range,
    argmax equal."""
    g = golden(fixture)
    cfg, w = _qwen3()
    cfg = cfg.with_(attn=variant)
    dec = OM.OracleDecoder(cfg, OM.quantize_model(cfg, w), g["kv"])
    for pos, t in enumerate(g["tokens"]):
        lg = dec.forward(int(t), pos)
        want = g["logits"][pos]
        rng = float(want.max() - want.min())
        assert np.max(np.abs(lg - want)) <= 2e-3 * rng, f"pos {pos}"
        top2 = np.sort(want)[-2:]
        if top2[1] - top2[0] > 4e-3 * rng:
            assert int(np.argmax(lg)) == int(np.argmax(want)), f"pos {pos}"
    if "kc" in g.files:
        n = len(g["tokens"])
        diff = np.abs(dec.kc[:, :n].astype(int) - g["kc"].astype(int))
        assert diff.max() <= 1 and (diff > 0).mean() < 0.01


def test_oracle_moe_rows_match_reference():
    """hf_generic.QMixtralMoe rows (router Top-k, softmax over the k logits,
    expert SwiGLUs, combine in k order) under the device SFU."""
    g = golden("moe.npz")
    E, top_k = g["rq"].shape[0], int(g["top_k"])
    cfg = C.ModelConfig("moe", g["x"].shape[1], 16, 1, 1, 1, 16, 16, 16, experts=E, top_k=top_k,
                        expert_hidden=g["gq"].shape[1])
    t = {"router": g["rq"], "s_router": g["rs"], "e_gate": g["gq"], "s_e_gate": g["gs"], "e_up": g["uq"],
         "s_e_up": g["us"], "e_down": g["dq"], "s_e_down": g["ds"]}
    for r in range(g["x"].shape[0]):
        y, ids, w = OM.moe_ffn_row(g["x"][r].astype(F), t, cfg)
        assert list(ids) == list(g["ids"][r])
        assert np.array_equal(w, g["w"][r])
        assert np.array_equal(y, g["y"][r]), f"row {r}: max diff {np.max(np.abs(y - g['y'][r]))}"


def test_per_channel_calibration_matches_the_reference():
    """KV scales per cache channel from this repo's fp32 calibration run equal
    the reference's calibrate_kv(channel="kv") (hf_qwen3_ch.npz) up to fp32
    summation order; a part whose row is constant stays per layer."""
    g = golden("hf_qwen3_ch.npz")
    cfg, w = _qwen3()
    kv = W.calibrate_kv(cfg, w, g["calib"], channel="kv")
    assert kv.shape == g["kv"].shape == (cfg.layers, 2, cfg.kv_dim)
    np.testing.assert_allclose(kv, g["kv"], rtol=1e-4)
    per_layer = W.calibrate_kv(cfg, w, g["calib"])
    np.testing.assert_allclose(per_layer, g["kv"].max(-1), rtol=1e-4)
    k_only = W.calibrate_kv(cfg, w, g["calib"], channel="k")
    assert np.all(k_only[:, 1] == k_only[:, 1, :1])             # V: one value per layer
    consts, ch = W.layer_kv_consts(k_only[0], cfg.head_dim)
    assert set(ch) == {"k_scale", "inv_sk_ch"} and consts[2] == np.float32(1.0 / np.sqrt(cfg.head_dim))


def test_gelu_gate_equals_reference():
    """The oracle's GELU-tanh gate equals hf_generic.SaGELUTanh under the device
    SFU bit for bit (ranges, random values, +-0, huge, inf, NaN), with the
    reference's constants."""
    g = golden("gelu.npz")
    assert g["a"] == N.GELU_A and g["b"] == N.GELU_B
    y = N.gelu_gate(g["x"], np.float32(1))
    assert np.array_equal(y.view(np.uint32), g["y"].view(np.uint32))     # (NumPy and torch: the same host NaN)
    with pytest.raises(ValueError):
        C.C4.with_(act="gelu_tanh").validate()                # MoE experts are SiLU

