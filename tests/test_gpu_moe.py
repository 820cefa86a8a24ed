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
