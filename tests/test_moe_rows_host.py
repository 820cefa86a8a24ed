"""Host side of the MoE over many rows, without a GPU: which entry the
decoders call for a row count and model width (the ops are recorded instead
of launched), and the kernel count the batched step claims. More than 16
rows go to the grouped entry (w8a8_moe_ffn_rows) when dim is a multiple of
32 (its 32-row down tiles); otherwise, and up to 16 rows, 16-row groups go to
the per-row kernels (w8a8_moe_ffn)."""
import numpy as np
import pytest
import torch

from torch2riscv_accelerator_b200 import config as C
from torch2riscv_accelerator_b200 import ops
from torch2riscv_accelerator_b200 import weights as W
from torch2riscv_accelerator_b200.model import CHUNK, BatchDecoder, DeviceDecoder


def _model(dim, heads):
    cfg = C.tiny(dim=dim, heads=heads, kv_heads=heads, experts=4, top_k=2, expert_hidden=32)
    qw = W.QuantWeights(cfg, seed=1, calib_tokens=np.arange(4))
    return cfg, qw


@pytest.fixture
def calls(monkeypatch):
    log = []
    monkeypatch.setattr(ops, "moe_ffn", lambda x, *a, **k: log.append(("per-row", x.shape[0])))
    monkeypatch.setattr(ops, "moe_ffn_rows", lambda x, *a, **k: log.append(("grouped", x.shape[0])))
    return log


@pytest.mark.parametrize("rows", [1, 16, 17, 40])
def test_moe_entry_by_row_count(calls, rows):
    cfg, qw = _model(64, 4)
    dec = DeviceDecoder(cfg, qw, qw.kv_scales, device="cpu", prefill_rows=64)
    dec._moe_rows(0, torch.zeros(rows, cfg.dim))
    assert calls == ([("per-row", rows)] if rows <= CHUNK else [("grouped", rows)])


def test_moe_width_not_multiple_of_32_keeps_16_row_groups(calls):
    cfg, qw = _model(48, 3)
    dec = DeviceDecoder(cfg, qw, qw.kv_scales, device="cpu", prefill_rows=64)
    assert dec.moe_rows_scratch is None
    dec._moe_rows(0, torch.zeros(40, cfg.dim))
    assert calls == [("per-row", 16), ("per-row", 16), ("per-row", 8)]


def test_batched_step_launch_count():
    """Per layer: row quantizer, qkv GEMM, attention, quantizer, o GEMM, then
    the grouped MoE's router, gate/up, down and combine (or 3 per 16-row group)."""
    cfg, qw = _model(64, 4)
    dec = BatchDecoder(cfg, qw, qw.kv_scales, 20, device="cpu")
    assert dec.kernel_launches() == 1 + cfg.layers * (5 + 4) + 2
    cfg, qw = _model(48, 3)
    dec = BatchDecoder(cfg, qw, qw.kv_scales, 20, device="cpu")
    assert dec.kernel_launches() == 1 + cfg.layers * (5 + 3 * 2) + 2
