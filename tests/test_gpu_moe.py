"""MoE FFN on the GPU through the C ABI against the reference's golden rows
(hf_generic.QMixtralMoe under the device SFU) and the oracle at the Granite
(C4) shape: routing (ids, weights) and outputs bit-exact."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import model as OM
from oracle import numerics as N
from torch2riscv_accelerator_b200 import config as C
from torch2riscv_accelerator_b200 import ops
from torch2riscv_accelerator_b200.weights import quantize_rows

pytestmark = pytest.mark.gpu
F = np.float32
DEV = "cuda"


def cu(a, dt=None):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=dt).to(DEV)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def bits(a):
    return np.asarray(a, F).view(np.uint32)


def run(x, t, top_k, norm_g=None, eps=1e-6, resid=None, inplace=False):
    m, dim = x.shape
    ih = t["e_gate"].shape[1]
    xd = cu(x)
    rd = cu(resid) if resid is not None else torch.zeros_like(xd)
    scratch = ops.moe_scratch(m, dim, top_k, ih, DEV)
    out = rd if inplace else None
    y, ids, w = ops.moe_ffn(xd, None if norm_g is None else cu(norm_g), eps, cu(t["router"]), cu(t["s_router"]),
                            top_k, cu(t["e_gate"]), cu(t["s_e_gate"]), cu(t["e_up"]), cu(t["s_e_up"]),
                            cu(t["e_down"]), cu(t["s_e_down"]), scratch, resid=rd, out=out)
    assert ops.error_flags() == 0
    return host(y), host(ids), host(w)


def test_moe_golden_rows_bit_exact():
    g = golden("moe.npz")
    top_k = int(g["top_k"])
    t = {"router": g["rq"], "s_router": g["rs"], "e_gate": g["gq"], "s_e_gate": g["gs"], "e_up": g["uq"],
         "s_e_up": g["us"], "e_down": g["dq"], "s_e_down": g["ds"]}
    x = g["x"].astype(F)
    y, ids, w = run(x, t, top_k)
    assert np.array_equal(ids, g["ids"].astype(np.int32))
    assert np.array_equal(bits(w), bits(g["w"]))
    assert np.array_equal(bits(y), bits(g["y"]))


def c4_tables(rng, E, dim, ih):
    q = lambda *s: quantize_rows((rng.standard_normal(s) * 0.05).astype(F).reshape(-1, s[-1]))
    t = {}
    t["router"], t["s_router"] = q(E, dim)
    for name, shape in (("e_gate", (E, ih, dim)), ("e_up", (E, ih, dim)), ("e_down", (E, dim, ih))):
        wq, ws = q(*shape)
        t[name], t["s_" + name] = wq.reshape(shape), ws.reshape(shape[:2])
    return t


@pytest.mark.parametrize("rows", [1, 5, 16])
def test_moe_c4_shape_against_oracle(rows):
    cfg = C.C4
    rng = np.random.default_rng(40 + rows)
    t = c4_tables(rng, cfg.experts, cfg.dim, cfg.expert_hidden)
    x = rng.standard_normal((rows, cfg.dim)).astype(F)
    g = (1 + 0.1 * rng.standard_normal(cfg.dim)).astype(F)
    resid = rng.standard_normal((rows, cfg.dim)).astype(F)
    y, ids, w = run(x, t, cfg.top_k, norm_g=g, eps=cfg.eps, resid=resid, inplace=True)
    xn = N.rmsnorm(x, g, cfg.eps)
    for m in range(rows):
        ym, idm, wm = OM.moe_ffn_row(xn[m], t, cfg)
        assert np.array_equal(ids[m], idm.astype(np.int32)), m
        assert np.array_equal(bits(w[m]), bits(wm)), m
        assert np.array_equal(bits(y[m]), bits((resid[m] + ym).astype(F))), m


def run_rows(x, t, top_k, norm_g, eps, resid=None, expert_lo=0, local=None):
    """The grouped entry (w8a8_moe_ffn_rows): y (resid given) or the terms of
    experts [expert_lo, expert_lo + local)."""
    m, dim = x.shape
    E, ih = t["e_gate"].shape[:2]
    local = E if local is None else local
    sl = slice(expert_lo, expert_lo + local)
    scratch = ops.moe_rows_scratch(m, dim, E, top_k, ih, DEV)
    wy = None if resid is not None else torch.full((m, top_k, dim), float("nan"), device=DEV)
    args = (cu(x), cu(norm_g), eps, cu(t["router"]), cu(t["s_router"]), top_k, cu(t["e_gate"][sl]),
            cu(t["s_e_gate"][sl]), cu(t["e_up"][sl]), cu(t["s_e_up"][sl]), cu(t["e_down"][sl]),
            cu(t["s_e_down"][sl]), scratch)
    if resid is not None:
        rd = cu(resid)
        y, ids, w = ops.moe_ffn_rows(*args, resid=rd, out=rd)
    else:
        y, ids, w = ops.moe_ffn_rows(*args, expert_lo=expert_lo, wy=wy)
    assert ops.error_flags() == 0
    return host(y), host(ids), host(w)


@pytest.mark.parametrize("rows", [17, 64, 203])
def test_moe_grouped_rows_equal_per_row_path(rows):
    """More than 16 rows grouped by expert (17 and 64: the CUDA-core kernels;
    203: the tensor-core path): the same routing and outputs, bit for bit, as
    the per-row kernels over 16-row groups; the first rows also against the
    oracle."""
    cfg = C.C4
    rng = np.random.default_rng(70 + rows)
    t = c4_tables(rng, cfg.experts, cfg.dim, cfg.expert_hidden)
    x = rng.standard_normal((rows, cfg.dim)).astype(F)
    g = (1 + 0.1 * rng.standard_normal(cfg.dim)).astype(F)
    resid = rng.standard_normal((rows, cfg.dim)).astype(F)
    y, ids, w = run_rows(x, t, cfg.top_k, g, cfg.eps, resid=resid)
    for j in range(0, rows, 16):
        yj, idj, wj = run(x[j:j + 16], t, cfg.top_k, norm_g=g, eps=cfg.eps, resid=resid[j:j + 16])
        assert np.array_equal(ids[j:j + 16], idj), j
        assert np.array_equal(bits(w[j:j + 16]), bits(wj)), j
        assert np.array_equal(bits(y[j:j + 16]), bits(yj)), j
    xn = N.rmsnorm(x, g, cfg.eps)
    for m in range(3):
        ym, _, _ = OM.moe_ffn_row(xn[m], t, cfg)
        assert np.array_equal(bits(y[m]), bits((resid[m] + ym).astype(F))), m


@pytest.mark.parametrize("ranks,rows", [(2, 40), (4, 40), (2, 150)])
def test_moe_grouped_rows_expert_parallel_terms(ranks, rows):
    """Expert parallelism through the grouped entry (40 rows: the CUDA-core
    kernels; 150: the tensor-core path, two slab tiles per expert): each
    rank's terms are w_j * y_j for its experts and +0 elsewhere, their sum
    folded by w8a8_moe_combine equals the one-GPU result bit for bit."""
    cfg = C.C4
    rng = np.random.default_rng(90 + ranks + rows)
    t = c4_tables(rng, cfg.experts, cfg.dim, cfg.expert_hidden)
    x = rng.standard_normal((rows, cfg.dim)).astype(F)
    g = (1 + 0.1 * rng.standard_normal(cfg.dim)).astype(F)
    resid = rng.standard_normal((rows, cfg.dim)).astype(F)
    y, ids, w = run_rows(x, t, cfg.top_k, g, cfg.eps, resid=resid)
    n = cfg.experts // ranks
    total = np.zeros((rows, cfg.top_k, cfg.dim), F)
    for r in range(ranks):
        wy, idr, wr = run_rows(x, t, cfg.top_k, g, cfg.eps, expert_lo=r * n, local=n)
        assert np.array_equal(idr, ids) and np.array_equal(bits(wr), bits(w))
        mine = (idr >= r * n) & (idr < (r + 1) * n)
        assert not np.isnan(wy).any()
        assert np.all(bits(wy[~mine]) == 0)                       # +0 for other ranks' experts
        total = (total + wy).astype(F)
    out = ops.moe_combine(cu(total), cu(resid), torch.empty(rows, cfg.dim, device=DEV))
    assert np.array_equal(bits(host(out)), bits(y))


def skewed_case(rows, seed):
    """C4 tables and rows whose routing piles onto a few experts: every row
    shares one direction that router row 5 (and partly 9) follows, so expert 5
    is in every row's Top-k (rows pairs: ceil(rows / 128) slab tiles) and a
    few others in most."""
    cfg = C.C4
    rng = np.random.default_rng(seed)
    t = c4_tables(rng, cfg.experts, cfg.dim, cfg.expert_hidden)
    common = rng.standard_normal(cfg.dim).astype(F)
    r = (rng.standard_normal((cfg.experts, cfg.dim)) * 0.05).astype(F)
    r[5] = common * 0.05
    r[9] = common * 0.04 + r[9] * 0.2
    t["router"], t["s_router"] = quantize_rows(r)
    x = (rng.standard_normal((rows, cfg.dim)) * 0.3 + common).astype(F)
    g = (1 + 0.1 * rng.standard_normal(cfg.dim)).astype(F)
    resid = rng.standard_normal((rows, cfg.dim)).astype(F)
    return cfg, t, x, g, resid


@pytest.mark.parametrize("rows", [300])
def test_moe_grouped_rows_several_slab_tiles(rows):
    """Experts with more than 128 and more than 256 pairs (the grouped
    GEMMs' second and third slab tiles hold valid rows): bit-exact with the
    per-row kernels over 16-row groups, and the expert-parallel terms of 2
    ranks summed equal the one-GPU result."""
    cfg, t, x, g, resid = skewed_case(rows, 123)
    y, ids, w = run_rows(x, t, cfg.top_k, g, cfg.eps, resid=resid)
    counts = np.bincount(ids.ravel(), minlength=cfg.experts)
    assert counts[5] == rows and counts.max() > 256 and (counts > 128).sum() >= 3
    for j in range(0, rows, 16):
        yj, idj, wj = run(x[j:j + 16], t, cfg.top_k, norm_g=g, eps=cfg.eps, resid=resid[j:j + 16])
        assert np.array_equal(ids[j:j + 16], idj), j
        assert np.array_equal(bits(w[j:j + 16]), bits(wj)), j
        assert np.array_equal(bits(y[j:j + 16]), bits(yj)), j
    n = cfg.experts // 2
    total = np.zeros((rows, cfg.top_k, cfg.dim), F)
    for r in range(2):
        wy, idr, _ = run_rows(x, t, cfg.top_k, g, cfg.eps, expert_lo=r * n, local=n)
        assert np.array_equal(idr, ids)
        total = (total + wy).astype(F)
    out = ops.moe_combine(cu(total), cu(resid), torch.empty(rows, cfg.dim, device=DEV))
    assert np.array_equal(bits(host(out)), bits(y))


def test_moe_router_tie_goes_to_the_lower_expert():
    """Router rows duplicated so that experts' scores tie exactly: Top-k keeps
    the lower expert id first (docs/moe_native_lowering_design.md:340-345),
    on the GPU as in the oracle, through the per-row and the grouped entries."""
    cfg = C.C4
    rng = np.random.default_rng(321)
    t = c4_tables(rng, cfg.experts, cfg.dim, cfg.expert_hidden)
    rq, rs = t["router"].copy(), t["s_router"].copy()
    for dst, src in ((20, 3), (7, 3), (30, 11), (12, 11), (25, 0)):
        rq[dst], rs[dst] = rq[src], rs[src]
    t["router"], t["s_router"] = rq, rs
    x = rng.standard_normal((40, cfg.dim)).astype(F)
    g = (1 + 0.1 * rng.standard_normal(cfg.dim)).astype(F)
    resid = rng.standard_normal((40, cfg.dim)).astype(F)
    y, ids, w = run(x[:16], t, cfg.top_k, norm_g=g, eps=cfg.eps, resid=resid[:16])
    xn = N.rmsnorm(x, g, cfg.eps)
    tied = 0
    for m in range(16):
        ym, idm, wm = OM.moe_ffn_row(xn[m], t, cfg)
        assert np.array_equal(ids[m], idm.astype(np.int32)), m
        assert np.array_equal(bits(y[m]), bits((resid[m] + ym).astype(F))), m
        for a, b in ((3, 7), (3, 20), (11, 12), (11, 30), (0, 25)):
            if a in ids[m] and b in ids[m]:
                tied += 1
                assert list(ids[m]).index(min(a, b)) < list(ids[m]).index(max(a, b))
    assert tied > 0
    y2, ids2, w2 = run_rows(x, t, cfg.top_k, g, cfg.eps, resid=resid)
    assert np.array_equal(ids2[:16], ids) and np.array_equal(bits(y2[:16]), bits(y))
