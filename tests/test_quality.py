"""Quality evaluation (`llm/eval_quant.py`'s measures): the measures
themselves, and the evaluation pipeline with the oracle standing in for the
device (on the GPU the device gives the oracle's logits bit for bit, so the
same numbers: tests/test_gpu_quality.py)."""
import numpy as np
import pytest

from oracle import model as OM
from torch2riscv_accelerator_b200 import config as C
from torch2riscv_accelerator_b200 import quality as Q
from torch2riscv_accelerator_b200 import weights as W

CFG = C.tiny("quality", heads=4, kv_heads=2, vocab=96, seq_len=48, attn="qsum", rope="hf", qk_norm=True, tied=True)


class OracleDevice:
    """The LlamaDevice surface (reset, forward) over the oracle."""

    def __init__(self, cfg, w, kv):
        self.dec = OM.OracleDecoder(cfg, OM.quantize_model(cfg, w), kv)
        self.pos = 0

    def reset(self):
        self.dec.reset()
        self.pos = 0

    def forward(self, t):
        lg = self.dec.forward(int(t), self.pos)
        self.pos += 1
        return lg


def test_measures():
    rng = np.random.default_rng(0)
    a = rng.standard_normal((20, 50)).astype(np.float32)
    r = Q.compare(a, a)
    assert r["top1"] == 1.0 and r["top5"] == 1.0 and abs(r["kl_mean"]) < 1e-12
    b = a.copy()
    b[:, 0] += 100                                                    # every top-1 moves to 0
    r = Q.compare(a, b)
    assert r["top1"] == np.mean(a.argmax(-1) == 0) and r["kl_mean"] > 1
    assert Q.first_divergence([1, 2, 3], [1, 2, 4]) == 2 and Q.first_divergence([1, 2], [1, 2, 5]) == 2


@pytest.mark.parametrize("channel", ["", "kv"])
def test_evaluate_with_the_oracle_device(channel):
    w = W.fp32_model(CFG, 3, gains="random", std=0.3)
    kv = W.calibrate_kv(CFG, w, [np.arange(10), np.arange(20, 34)], channel=channel)
    prompts = [np.array([5, 17, 40]), np.array([1, 2])]
    r = Q.evaluate(CFG, w, kv, prompts, 16, lambda k: OracleDevice(CFG, w, k))
    assert r["positions"] == 32 and 0 <= r["top1"] <= r["top5"] <= 1 and r["kl_mean"] >= -1e-9
    assert all(0 <= d <= 16 for d in r["first_divergence"])
    assert r["top1"] > 0.5                                    # W8A8 stays close to fp32 on this model
