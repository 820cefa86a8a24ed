"""w8a8_ffn_swiglu_noalloc: the SwiGLU dispatch with its scratch in the
library's static device memory. Called through the C ABI and compared with
w8a8_ffn_swiglu (caller-provided scratch) on two calls in a row. The file name
sorts last so that the test also runs after every other test in one session."""
import ctypes as C

import numpy as np
import pytest

from torch2riscv_accelerator_b200 import _lib
from torch2riscv_accelerator_b200.weights import quantize_rows

F = np.float32


def test_noalloc_rejects_before_any_launch(lib):
    """Argument errors return a status before anything touches a device."""
    big = _lib.load().w8a8_ffn_swiglu_noalloc(16, 16, C.c_float(1e-5), 17, 64, 16, 16, 16, 16, 64, 16, 16, 16,
                                              None)
    assert big == _lib.W8A8_ESCRATCH
    assert lib.w8a8_status_string(big) == b"scratch buffer too small"
    no_hq = lib.w8a8_ffn_swiglu_noalloc(16, 16, C.c_float(1e-5), 1, 64, 16, 16, 16, 16, 64, 16, None, None, None)
    assert no_hq == _lib.W8A8_EINVAL
    odd_k = lib.w8a8_ffn_swiglu_noalloc(16, 16, C.c_float(1e-5), 1, 40, 16, 16, 16, 16, 64, 16, 16, 16, None)
    assert odd_k == _lib.W8A8_EALIGN


@pytest.mark.gpu
@pytest.mark.parametrize("m", [1, 3, 16])
def test_noalloc_matches_caller_scratch_entry_twice(lib, m):
    import torch

    dev = "cuda"
    k, hidden = 1024, 3072
    rng = np.random.default_rng(500 + m)
    wg, sg = quantize_rows((rng.standard_normal((hidden, k)) * 0.05).astype(F))
    wu, su = quantize_rows((rng.standard_normal((hidden, k)) * 0.05).astype(F))
    g = (1 + 0.1 * rng.standard_normal(k)).astype(F)
    t = lambda a: torch.as_tensor(np.ascontiguousarray(a)).to(dev)
    wg_d, sg_d, wu_d, su_d, g_d = t(wg), t(sg), t(wu), t(su), t(g)
    scratch = torch.zeros(lib.w8a8_ffn_scratch_bytes(m), dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream().cuda_stream

    def outputs():
        return (torch.empty((m, hidden), dtype=torch.float32, device=dev),
                torch.empty((m, hidden), dtype=torch.int8, device=dev),
                torch.empty(m, dtype=torch.float32, device=dev))

    for it in range(2):                                  # two calls in a row: the static scratch is reused
        x = t(rng.standard_normal((m, k)).astype(F))
        h1, q1, s1 = outputs()
        rc = lib.w8a8_ffn_swiglu(x.data_ptr(), g_d.data_ptr(), C.c_float(1e-6), m, k, wg_d.data_ptr(),
                                 sg_d.data_ptr(), wu_d.data_ptr(), su_d.data_ptr(), hidden, h1.data_ptr(),
                                 q1.data_ptr(), s1.data_ptr(), scratch.data_ptr(), scratch.numel(), st)
        assert rc == 0, lib.w8a8_status_string(rc)
        h2, q2, s2 = outputs()
        rc = lib.w8a8_ffn_swiglu_noalloc(x.data_ptr(), g_d.data_ptr(), C.c_float(1e-6), m, k, wg_d.data_ptr(),
                                         sg_d.data_ptr(), wu_d.data_ptr(), su_d.data_ptr(), hidden,
                                         h2.data_ptr(), q2.data_ptr(), s2.data_ptr(), st)
        assert rc == 0, lib.w8a8_status_string(rc)
        torch.cuda.synchronize()
        a, b = h1.cpu().numpy(), h2.cpu().numpy()
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), it
        assert torch.equal(q1, q2), it
        assert np.array_equal(s1.cpu().numpy().view(np.uint32), s2.cpu().numpy().view(np.uint32)), it
        assert int(q2.abs().max()) == 127, it           # the requantization ran
    flags = C.c_uint32(0)
    assert lib.w8a8_error_flags(C.byref(flags)) == 0 and flags.value == 0
