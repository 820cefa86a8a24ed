"""Quality evaluation on the GPU: the device's teacher-forced logits equal the
oracle's bit for bit, so every measure equals the oracle-device evaluation's."""
import numpy as np
import pytest

from test_quality import CFG, OracleDevice
from torch2riscv_accelerator_b200 import quality as Q
from torch2riscv_accelerator_b200 import weights as W
from torch2riscv_accelerator_b200.runtime import LlamaDevice

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("channel", ["", "kv"])
def test_device_quality_equals_oracle_quality(channel):
    w = W.fp32_model(CFG, 3, gains="random", std=0.3)
    kv = W.calibrate_kv(CFG, w, [np.arange(10), np.arange(20, 34)], channel=channel)
    prompts = [np.array([5, 17, 40]), np.array([1, 2])]
    qw = W.from_fp32(CFG, w)
    got = Q.evaluate(CFG, w, kv, prompts, 16, lambda k: LlamaDevice((CFG, qw, k)))
    want = Q.evaluate(CFG, w, kv, prompts, 16, lambda k: OracleDevice(CFG, w, k))
    assert got == want
