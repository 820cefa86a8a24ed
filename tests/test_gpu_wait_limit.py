"""A tensor-parallel exchange wait that runs out, on one GPU.

The reference's host gives a submitted list a timeout and reports a status
instead of hanging (driver/pynq_matmul.py:983-998 Device.wait; the funcsim's
SaError, llm/sa_funcsim.py:62-66). Here the decode kernels poll exchange words
with a bounded spin. This test builds a 2-rank exchange whose second rank's
region is a buffer on this GPU that nothing writes, so the linear's wait for
that rank's row maxima gives up: the call returns, the outputs are zeros, error
bit 5 is set, and the context stays usable (a normal call right after is
exact). No fault is involved: the kernel only polls memory of its own GPU.
"""
import ctypes

import numpy as np
import pytest
import torch

from torch2riscv_accelerator_b200 import _lib, ops
from torch2riscv_accelerator_b200.weights import quantize_rows

pytestmark = pytest.mark.gpu


def test_exchange_wait_gives_up_with_error_bit_5():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    assert ops.error_flags() == 0
    nbytes = 1 << 20
    regions = []
    for _ in range(2):                        # this rank's region, and the silent "peer" (local memory)
        p = ctypes.c_void_p()
        _lib.check("w8a8_tp_alloc", lib.w8a8_tp_alloc(nbytes, ctypes.byref(p)))
        regions.append(p.value)
    try:
        comm = _lib.W8A8TpComm(0, 2, nbytes, (ctypes.c_void_p * _lib.TP_MAX_RANKS)(*regions))
        rng = np.random.default_rng(5)
        k, n, vocab = 1024, 256, 64
        emb_q, emb_s = quantize_rows(rng.standard_normal((vocab, k)).astype(np.float32))
        emb_q, emb_s = torch.as_tensor(emb_q).to(dev), torch.as_tensor(emb_s).to(dev)
        tok = torch.tensor([3], dtype=torch.int32, device=dev)
        x = torch.empty(1, k, device=dev)
        ops.tp_embed(comm, tok, emb_q, emb_s, x)          # a new step: epoch 1 (no word of either region has it)
        wq, ws = quantize_rows((rng.standard_normal((n, k)) * 0.05).astype(np.float32))
        wq, ws = torch.as_tensor(wq).to(dev), torch.as_tensor(ws).to(dev)
        y = torch.full((1, n), float("nan"), device=dev)
        amax_block = regions[0] + _lib.TP_HEADER                   # this step's max|x| words: never posted
        a = _lib.W8A8TpLinearArgs()
        a.comm = ctypes.pointer(comm)
        a.rows, a.k, a.n = 1, k, n
        a.x, a.amax_in, a.w, a.s_w = x.data_ptr(), amax_block, wq.data_ptr(), ws.data_ptr()
        a.epilogue, a.y = _lib.TP_STORE, y.data_ptr()
        ops.tp_linear(a)                                            # returns: the wait is bounded
        torch.cuda.synchronize()
        flags = ops.error_flags()
        assert flags & 32, flags                                    # bit 5: an exchange wait gave up
        assert torch.count_nonzero(y).item() == 0                   # nothing from the missing maxima
        # the context is still usable: a plain one-GPU linear right after is exact
        xq, sx = ops.quant_act(x)
        out = ops.linear(xq, sx, wq, ws)
        acc = xq.cpu().numpy().astype(np.int64) @ wq.cpu().numpy().astype(np.int64).T
        ref = ((acc.astype(np.float32) * ws.cpu().numpy()) * sx.cpu().numpy()[:, None]).astype(np.float32)
        assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))
        assert ops.error_flags() == 0
    finally:
        torch.cuda.synchronize()
        for p in regions:
            lib.w8a8_tp_free(ctypes.c_void_p(p))
