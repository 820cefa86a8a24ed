"""Tensor-core GEMM (tcgen05 kind::i8) and the row quantizer through the C ABI:
bit-exact with the oracle and with the GEMV path (same arithmetic after the
exact int32 sums)."""
import numpy as np
import pytest
import torch

from oracle import numerics as N
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


@pytest.mark.parametrize("m,n,k", [(128, 4096, 1024), (200, 1024, 2048), (33, 1024, 3072), (300, 576, 576),
                                   (17, 1000, 288), (256, 3072, 1024)])
def test_gemm_bit_exact_with_oracle(m, n, k):
    rng = np.random.default_rng(m * 7 + n + k)
    w, sw = quantize_rows((rng.standard_normal((n, k)) * 0.05).astype(F))
    x = rng.standard_normal((m, k)).astype(F)
    xq, sx = N.quant_act(x)
    acc = torch.zeros(m, n, dtype=torch.int32, device=DEV)
    y = host(ops.gemm(cu(xq), cu(sx), cu(w), cu(sw), acc=acc))
    wy, wacc = N.linear(xq, sx, w, sw)
    assert np.array_equal(host(acc), wacc)
    assert np.array_equal(bits(y), bits(wy))
    assert ops.error_flags() == 0


@pytest.mark.parametrize("m", [1, 4, 16])
def test_gemm_equals_gemv_path(m):
    """Decode-sized rows: the tensor-core GEMM and the bulk-copy GEMV give the
    same bits (in place residual included)."""
    rng = np.random.default_rng(90 + m)
    n, k = 4096, 1024
    w, sw = quantize_rows((rng.standard_normal((n, k)) * 0.05).astype(F))
    xq, sx = N.quant_act(rng.standard_normal((m, k)).astype(F))
    resid = rng.standard_normal((m, n)).astype(F)
    a, b = cu(resid), cu(resid)
    ops.gemm(cu(xq), cu(sx), cu(w), cu(sw), out=a, resid=a)
    ops.linear(cu(xq), cu(sx), cu(w), cu(sw), out=b, resid=b)
    assert np.array_equal(bits(host(a)), bits(host(b)))


@pytest.mark.parametrize("m,hidden,k", [(128, 3072, 1024), (40, 512, 1024), (200, 1536, 576)])
def test_gemm_swiglu_bit_exact(m, hidden, k):
    rng = np.random.default_rng(m + hidden)
    wg, sg = quantize_rows((rng.standard_normal((hidden, k)) * 0.05).astype(F))
    wu, su = quantize_rows((rng.standard_normal((hidden, k)) * 0.05).astype(F))
    xq, sx = N.quant_act(rng.standard_normal((m, k)).astype(F))
    h = host(ops.gemm_swiglu(cu(xq), cu(sx), cu(wg), cu(sg), cu(wu), cu(su)))
    want = N.silu_gate(N.linear(xq, sx, wg, sg)[0], N.linear(xq, sx, wu, su)[0])
    assert np.array_equal(bits(h), bits(want))


@pytest.mark.parametrize("norm", [False, True])
def test_quant_rows_bit_exact(norm):
    rng = np.random.default_rng(3 + norm)
    m, k = 77, 1024
    x = rng.standard_normal((m, k)).astype(F)
    g = (1 + 0.1 * rng.standard_normal(k)).astype(F)
    xq, sx = ops.quant_rows(cu(x), cu(g) if norm else None, 1e-6)
    want_q, want_s = N.quant_act(N.rmsnorm(x, g, 1e-6) if norm else x)
    assert np.array_equal(host(xq), want_q)
    assert np.array_equal(bits(host(sx)), bits(want_s))
