"""Kernel parity on the GPU, through the C ABI, against the CPU oracle
(bit-exact: int32 accumulators, int8 activations, KV rows and fp32 results)."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import model as OM
from oracle import numerics as N
from torch2riscv_accelerator_b200 import config as C
from torch2riscv_accelerator_b200 import ops
from torch2riscv_accelerator_b200.weights import kv_consts, quantize_rows, rope_tables

pytestmark = pytest.mark.gpu
F = np.float32
DEV = "cuda"


def cu(a, dt=None):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=dt).to(DEV)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def same_bits(got, want):
    g, w = np.asarray(got, F).view(np.uint32), np.asarray(want, F).view(np.uint32)
    bad = np.flatnonzero(g.ravel() != w.ravel())
    return bad.size == 0, bad[:5]


# ------------------------------------------------------------------ SFU
@pytest.mark.parametrize("func,fn", [(0, N.sfu_exp), (1, N.sfu_recip), (2, N.sfu_rsqrt)])
def test_sfu_bit_exact_random_bits_and_golden(func, fn):
    rng = np.random.default_rng(func)
    x = np.concatenate([rng.integers(0, 2**32, 1 << 20, dtype=np.uint64).astype(np.uint32),
                        golden("sfu.npz")["x"]]).view(F)
    got = host(ops.sfu(func, cu(x)))
    ok, bad = same_bits(got, fn(x))
    assert ok, [(hex(x.view(np.uint32)[i]), hex(got.view(np.uint32)[i])) for i in bad]
    g = golden("sfu.npz")
    name = {0: "exp", 1: "recip", 2: "rsqrt"}[func]
    assert np.array_equal(host(ops.sfu(func, cu(g["x"].view(F)))).view(np.uint32), g[name])


def test_silu_gate_bit_exact():
    x = np.random.default_rng(9).uniform(-120, 120, 1 << 18).astype(F)
    ok, _ = same_bits(host(ops.sfu(ops.SFU_SILU, cu(x))), N.silu_gate(x, np.ones_like(x)))
    assert ok


def same_bits_nan(got, want):
    """Bit-exact, except that a NaN equals any NaN: a NaN made by an invalid
    operation (-inf * 0, NaN inputs) carries the hardware's default pattern
    (x86 0xFFC00000, the GPU's canonical one), not a value of the algorithm."""
    g, w = np.asarray(got, F).ravel(), np.asarray(want, F).ravel()
    gn, wn = np.isnan(g), np.isnan(w)
    bad = np.flatnonzero((gn != wn) | (~gn & (g.view(np.uint32) != w.view(np.uint32))))
    return bad.size == 0, bad[:5]


def test_gelu_gate_bit_exact_with_reference():
    """GELU-tanh (SaGELUTanh under the device SFU, gelu.npz) on the device,
    and the oracle's restatement on random bit patterns."""
    g = golden("gelu.npz")
    ok, bad = same_bits_nan(host(ops.sfu(ops.SFU_GELU, cu(g["x"]))), g["y"])
    assert ok, bad
    x = np.random.default_rng(4).integers(0, 2**32, 1 << 18, dtype=np.uint64).astype(np.uint32).view(F)
    ok, bad = same_bits_nan(host(ops.sfu(ops.SFU_GELU, cu(x))), N.gelu_gate(x, np.ones_like(x)))
    assert ok, bad


# ------------------------------------------------------------ vector ops
@pytest.mark.parametrize("k", [48, 288, 1024, 3072, 100])
def test_quant_act_and_rmsnorm(k):
    rng = np.random.default_rng(k)
    x = (rng.standard_normal((5, k)) * np.exp(rng.uniform(-8, 8, (5, 1)))).astype(F)
    x[3] = 0.0                                                    # amax 0: s = 0, q = 0
    x[4, :7] = -0.0
    xq, s = ops.quant_act(cu(x))
    wq, ws = N.quant_act(x)
    assert np.array_equal(host(xq), wq) and same_bits(host(s), ws)[0]
    g = (1 + 0.1 * rng.standard_normal(k)).astype(F)
    ok, _ = same_bits(host(ops.rmsnorm(cu(x[:3]), cu(g), 1e-5)), N.rmsnorm(x[:3], g, 1e-5))
    assert ok


def test_embed_and_argmax():
    rng = np.random.default_rng(4)
    q, s = quantize_rows(rng.standard_normal((300, 64)).astype(F))
    toks = np.array([0, 299, 17, 17], np.int32)
    x = host(ops.embed(cu(toks), cu(q), cu(s)))
    assert same_bits(x, (q[toks].astype(F) * s[toks][:, None]).astype(F))[0]
    lg = rng.standard_normal((3, 5000)).astype(F)
    lg[1, [10, 4000]] = 50.0                                       # ties: the first index wins
    assert list(host(ops.argmax(cu(lg)))) == [int(np.argmax(r)) for r in lg]


# ----------------------------------------------------------------- linear
LIN_SHAPES = [(864, 288), (1024, 2048), (6144, 1024), (2048, 8192), (9000, 576), (16, 4080), (64, 4096),
              (48, 4112)]


@pytest.mark.parametrize("n,k", LIN_SHAPES)
@pytest.mark.parametrize("m", [1, 3, 16])
def test_linear_bit_exact(n, k, m):
    rng = np.random.default_rng(n * 31 + k + m)
    w, sw = quantize_rows(rng.standard_normal((n, k)).astype(F))
    x = rng.standard_normal((m, k)).astype(F)
    xq, sx = N.quant_act(x)
    acc = torch.zeros(m, n, dtype=torch.int32, device=DEV)
    y = host(ops.linear(cu(xq), cu(sx), cu(w), cu(sw), acc=acc))
    wy, wacc = N.linear(xq, sx, w, sw)
    assert np.array_equal(host(acc), wacc)
    assert same_bits(y, wy)[0]


@pytest.mark.parametrize("k", [4080, 4096, 4112, 8192])
def test_linear_worst_case_accumulator(k):
    """|sum| = K * 127 * 127 (~K * 2^14), the reference's K-split worst case
    (`compiler/tests/test_gemv_ksplit.py`): exact int32."""
    n = 32
    w = np.full((n, k), 127, np.int8)
    w[1::2] = -127
    xq = np.full((1, k), 127, np.int8)
    acc = torch.zeros(1, n, dtype=torch.int32, device=DEV)
    ops.linear(cu(xq), cu(np.ones(1, F)), cu(w), cu(np.ones(n, F)), acc=acc)
    want = np.where(np.arange(n) % 2 == 0, k * 16129, -k * 16129)
    assert np.array_equal(host(acc)[0], want)


@pytest.mark.parametrize("n,k", [(151936, 1024), (128256, 2048)])
def test_linear_classifier_shape_sampled_rows(n, k):
    """The C2 and C3 classifiers (151936 x 1024: two streaming CTAs per SM;
    128256 x 2048: one CTA with the deeper ring): every output bit-exact,
    checked against the oracle on a sample of rows; one row and four."""
    rng = np.random.default_rng(11)
    w, sw = quantize_rows((rng.standard_normal((n, k)) * 0.02).astype(F))
    rows = np.concatenate([np.arange(64), rng.integers(0, n, 2000), np.arange(n - 64, n)])
    wd, swd = cu(w), cu(sw)
    for m in (1, 4):
        x = rng.standard_normal((m, k)).astype(F)
        xq, sx = N.quant_act(x)
        y = host(ops.linear(cu(xq), cu(sx), wd, swd))
        wy, _ = N.linear(xq, sx, w[rows], sw[rows])
        assert same_bits(y[:, rows], wy)[0], m


@pytest.mark.parametrize("m", [1, 16])
@pytest.mark.parametrize("norm", [True, False])
def test_linear_fused_prologues(m, norm):
    rng = np.random.default_rng(m + 2 * norm)
    n, k = 4096, 1024
    w, sw = quantize_rows(rng.standard_normal((n, k)).astype(F))
    x = rng.standard_normal((m, k)).astype(F)
    g = (1 + 0.1 * rng.standard_normal(k)).astype(F)
    resid = rng.standard_normal((m, n)).astype(F)
    sx = torch.zeros(m, device=DEV)
    if norm:
        y = host(ops.linear_fused(cu(x), cu(w), cu(sw), norm_g=cu(g), eps=1e-6, s_x_out=sx))
        xq, s = N.quant_act(N.rmsnorm(x, g, 1e-6))
        want = N.linear(xq, s, w, sw)[0]
    else:
        y = host(ops.linear_fused(cu(x), cu(w), cu(sw), resid=cu(resid), s_x_out=sx))
        xq, s = N.quant_act(x)
        want = (resid + N.linear(xq, s, w, sw)[0]).astype(F)
    assert same_bits(host(sx), s)[0]
    assert same_bits(y, want)[0]


def test_linear_int8_in_place_residual():
    rng = np.random.default_rng(5)
    n, k = 1024, 3072
    w, sw = quantize_rows(rng.standard_normal((n, k)).astype(F))
    hq, sh = N.quant_act(rng.standard_normal((1, k)).astype(F))
    x = rng.standard_normal((1, n)).astype(F)
    xt = cu(x)
    ops.linear(cu(hq), cu(sh), cu(w), cu(sw), out=xt, resid=xt)
    assert same_bits(host(xt), (x + N.linear(hq, sh, w, sw)[0]).astype(F))[0]


# ----------------------------------------------------------------- SwiGLU
@pytest.mark.parametrize("m,hidden,k", [(1, 3072, 1024), (1, 768, 288), (16, 1536, 576), (4, 8192, 2048)])
def test_ffn_swiglu_bit_exact_twice(m, hidden, k):
    rng = np.random.default_rng(hidden + m)
    wg, sg = quantize_rows((rng.standard_normal((hidden, k)) * 0.05).astype(F))
    wu, su = quantize_rows((rng.standard_normal((hidden, k)) * 0.05).astype(F))
    g = (1 + 0.1 * rng.standard_normal(k)).astype(F)
    scratch = ops.ffn_scratch(m, DEV)
    for it in range(2):                                          # the scratch is left zeroed for the next call
        x = rng.standard_normal((m, k)).astype(F)
        h, hq, sh = ops.ffn_swiglu(cu(x), cu(g), 1e-5, cu(wg), cu(sg), cu(wu), cu(su), scratch)
        xq, sx = N.quant_act(N.rmsnorm(x, g, 1e-5))
        want_h = N.silu_gate(N.linear(xq, sx, wg, sg)[0], N.linear(xq, sx, wu, su)[0])
        want_q, want_s = N.quant_act(want_h)
        assert same_bits(host(h), want_h)[0], it
        assert np.array_equal(host(hq), want_q) and same_bits(host(sh), want_s)[0], it
    assert not host(scratch).any()


# -------------------------------------------------------------- attention
ATT_CASES = [
    # heads, kv_heads, head_dim, seq_len, variant, qk_norm, positions (one call's rows)
    (6, 6, 48, 256, "norm", False, [0]),
    (6, 6, 48, 256, "norm", False, [200]),
    (16, 8, 128, 2048, "qsum", True, [2047]),
    (16, 8, 128, 2048, "qsum", True, [127]),
    (16, 8, 128, 2048, "qsum", True, [128]),
    (16, 8, 128, 2048, "norm", True, [1500]),
    (9, 3, 64, 2048, "qsum", False, [1000]),
    (32, 8, 64, 2048, "qsum", False, list(range(1016, 1032))),      # a 16-row chunk across a chunk boundary
    (16, 8, 128, 2048, "qsum", True, list(range(2032, 2048))),
    (16, 8, 128, 2048, "norm", True, list(range(0, 16))),
    (4, 2, 16, 48, "norm", False, list(range(5, 12))),
]


@pytest.mark.parametrize("case", ATT_CASES)
def test_attention_bit_exact(case):
    H, Hk, hd, T, variant, qkn, pos = case
    cfg = C.ModelConfig("att", 64, 64, 1, H, Hk, hd, 64, T, theta=1e6, eps=1e-6, qk_norm=qkn, attn=variant,
                        rope="hf")
    rng = np.random.default_rng(hd + len(pos) + pos[0])
    M = len(pos)
    qkv = (rng.standard_normal((M, cfg.qkv_dim)) * 2).astype(F)
    n0 = min(pos)
    kc = np.zeros((T, cfg.kv_dim), np.int8)
    vc = np.zeros((T, cfg.kv_dim), np.int8)
    kc[:n0] = rng.integers(-127, 128, (n0, cfg.kv_dim))         # earlier positions' rows
    vc[:n0] = rng.integers(-127, 128, (n0, cfg.kv_dim))
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(F) if qkn else None
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(F) if qkn else None
    cos, sin = rope_tables(cfg)
    consts = kv_consts(F(0.05), F(0.03), hd)
    # device: cache [Hk, T, hd]
    dk = cu(kc.reshape(T, Hk, hd).transpose(1, 0, 2))                  # [Hk, T, hd]
    dv = cu(vc.reshape(T, Hk, hd).transpose(1, 2, 0))                  # [Hk, hd, T]
    att = torch.zeros(M, cfg.q_dim, device=DEV)
    scratch = ops.attn_scratch(M, H, Hk, hd, T, DEV)
    dpos, dqkv, dcos, dsin = cu(np.array(pos, np.int32)), cu(qkv), cu(cos), cu(sin)
    dqn, dkn = (cu(qn), cu(kn)) if qkn else (None, None)
    args = ops.attn_args(cfg, M, dpos, dqkv, dk, dv, att, consts, dcos, dsin, scratch, dqn, dkn)
    ops.attn(args)
    got = host(att)
    want = OM.attn_layer(cfg, qkv, pos, kc, vc, consts, cos, sin, qn, kn)
    gk = host(dk).transpose(1, 0, 2).reshape(T, -1)
    gv = host(dv).transpose(2, 0, 1).reshape(T, -1)
    assert np.array_equal(gk, kc) and np.array_equal(gv, vc), "KV rows"
    ok, bad = same_bits(got, want)
    assert ok, (bad, got.ravel()[bad], want.ravel()[bad])
    ops.attn(args)                                               # again: the scratch counters were reset
    assert same_bits(host(att), want)[0]


PREFILL_CASES = [
    (16, 8, 128, 2048, "qsum", True, list(range(100, 145))),      # 16 + 16 + 13 rows
    (32, 8, 64, 2048, "qsum", False, list(range(1000, 1070))),     # across 128-position chunk boundaries
    (6, 6, 48, 256, "norm", False, list(range(0, 40))),
    (16, 8, 128, 2048, "norm", True, list(range(1990, 2048))),
]


@pytest.mark.parametrize("case", PREFILL_CASES)
def test_prefill_attention_groups_bit_exact(case):
    """A prefill chunk of more than 16 rows: every row's K/V appended
    (w8a8_kv_append), then one attention launch in 16-row groups
    (w8a8_attn_prefill): the outputs and the cache equal the oracle's (which
    writes the chunk's rows before attending, as the reference's chunks do)."""
    H, Hk, hd, T, variant, qkn, pos = case
    cfg = C.ModelConfig("att", 64, 64, 1, H, Hk, hd, 64, T, theta=1e6, eps=1e-6, qk_norm=qkn, attn=variant,
                        rope="hf")
    rng = np.random.default_rng(hd + len(pos))
    M, n0 = len(pos), min(pos)
    qkv = (rng.standard_normal((M, cfg.qkv_dim)) * 2).astype(F)
    kc = np.zeros((T, cfg.kv_dim), np.int8)
    vc = np.zeros((T, cfg.kv_dim), np.int8)
    kc[:n0] = rng.integers(-127, 128, (n0, cfg.kv_dim))
    vc[:n0] = rng.integers(-127, 128, (n0, cfg.kv_dim))
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(F) if qkn else None
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(F) if qkn else None
    cos, sin = rope_tables(cfg)
    consts = kv_consts(F(0.05), F(0.03), hd)
    dk = cu(kc.reshape(T, Hk, hd).transpose(1, 0, 2))
    dv = cu(vc.reshape(T, Hk, hd).transpose(1, 2, 0))
    att = torch.zeros(M, cfg.q_dim, device=DEV)
    scratch = ops.attn_scratch(16, H, Hk, hd, T, DEV)
    dqn, dkn = (cu(qn), cu(kn)) if qkn else (None, None)
    args = ops.attn_args(cfg, M, cu(np.array(pos, np.int32)), cu(qkv), dk, dv, att, consts, cu(cos), cu(sin),
                         scratch, dqn, dkn)
    ops.kv_append(args)
    ops.attn_prefill(args)
    want = OM.attn_layer(cfg, qkv, pos, kc, vc, consts, cos, sin, qn, kn)
    gk = host(dk).transpose(1, 0, 2).reshape(T, -1)
    gv = host(dv).transpose(2, 0, 1).reshape(T, -1)
    assert np.array_equal(gk, kc) and np.array_equal(gv, vc), "KV rows"
    ok, bad = same_bits(host(att), want)
    assert ok, bad
    assert ops.error_flags() == 0


def test_embed_out_of_range_token_sets_error_flag():
    """The embedding kernel's bounds check: a token outside the table reads
    nothing, writes a zero row and raises the device error flag."""
    rng = np.random.default_rng(12)
    q, s = quantize_rows(rng.standard_normal((50, 32)).astype(F))
    assert ops.error_flags() == 0
    x = host(ops.embed(cu(np.array([3, 50, -1, 7], np.int32)), cu(q), cu(s)))
    assert not x[1].any() and not x[2].any() and x[0].any() and x[3].any()
    assert ops.error_flags() == 1
    assert ops.error_flags() == 0                                # read and cleared


@pytest.mark.parametrize("m", [1, 4])
def test_classifier_fused_argmax(m):
    """Final rmsnorm + quant + classifier with the greedy argmax in the epilogue:
    logits bit-exact, the packed key's index = np.argmax (first maximum on ties)."""
    rng = np.random.default_rng(m)
    n, k = 32000, 288
    w, sw = quantize_rows((rng.standard_normal((n, k)) * 0.02).astype(F))
    w[7777] = w[123]                                            # a tie: the lower index must win
    sw[7777] = sw[123]
    w[123] *= 0
    w[123] += 127
    w[7777] = w[123]
    x = rng.standard_normal((m, k)).astype(F)
    x[:, :] = np.abs(x)
    g = (1 + 0.1 * rng.standard_normal(k)).astype(F)
    key = torch.zeros(m, dtype=torch.int64, device=DEV)
    y = host(ops.classifier(cu(x), cu(w), cu(sw), cu(g), 1e-5, argmax_key=key))
    xq, s = N.quant_act(N.rmsnorm(x, g, 1e-5))
    want = N.linear(xq, s, w, sw)[0]
    assert same_bits(y, want)[0]
    assert [ops.key_token(v) for v in host(key)] == [int(np.argmax(r)) for r in want]


def test_ffn_swiglu_without_requant_then_fused_down_projection():
    """The decode chain's split: the SwiGLU kernel stops at h, the down
    projection's prologue does quant_act(h): the same bytes as the full
    dispatch followed by the int8 linear."""
    rng = np.random.default_rng(31)
    k, hidden, n = 1024, 3072, 1024
    wg, sg = quantize_rows((rng.standard_normal((hidden, k)) * 0.05).astype(F))
    wu, su = quantize_rows((rng.standard_normal((hidden, k)) * 0.05).astype(F))
    wd, sd = quantize_rows((rng.standard_normal((n, hidden)) * 0.05).astype(F))
    g = (1 + 0.1 * rng.standard_normal(k)).astype(F)
    x = rng.standard_normal((1, k)).astype(F)
    resid = rng.standard_normal((1, n)).astype(F)
    h, hq, sh = ops.ffn_swiglu(cu(x), cu(g), 1e-6, cu(wg), cu(sg), cu(wu), cu(su), ops.ffn_scratch(1, DEV))
    y1 = host(ops.linear(hq, sh, cu(wd), cu(sd), resid=cu(resid)))
    h2, none_q, none_s = ops.ffn_swiglu(cu(x), cu(g), 1e-6, cu(wg), cu(sg), cu(wu), cu(su), None, requant=False)
    assert none_q is None and none_s is None
    y2 = host(ops.linear_fused(h2, cu(wd), cu(sd), resid=cu(resid)))
    assert same_bits(host(h), host(h2))[0] and same_bits(y1, y2)[0]
