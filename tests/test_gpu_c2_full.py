"""The full C2 (Qwen3-0.6B shape) decoder at the benchmark's own state: all 28
layers, vocabulary 151936, the seeded weights and prompt of bench.py, prefilled
to position 2023 on the GPU; then two decode steps from the GPU's own KV cache
against the oracle, logits bit for bit (and so the greedy tokens)."""
import numpy as np
import pytest

from oracle import model as OM
from torch2riscv_accelerator_b200 import config as C
from torch2riscv_accelerator_b200.model import DeviceDecoder
from torch2riscv_accelerator_b200.runtime import LlamaDevice
from torch2riscv_accelerator_b200.weights import QuantWeights

pytestmark = pytest.mark.gpu


class _NoCache(dict):
    """The oracle keeps float64 copies of the weights it has used; at this size
    (4.8 GB) convert per use instead."""

    def __setitem__(self, k, v):
        pass


def test_full_c2_two_steps_bit_exact_with_the_oracle():
    cfg = C.C2
    qw = QuantWeights(cfg, seed=0, calib_tokens=np.random.default_rng(1).integers(0, cfg.vocab, 16))
    dev = LlamaDevice(DeviceDecoder(cfg, qw, qw.kv_scales))
    P = 2023
    dev.prefill(np.random.default_rng(3).integers(0, cfg.vocab, P))
    ora = OM.OracleDecoder(cfg, qw, qw.kv_scales)
    ora._w64 = _NoCache()
    for l in range(cfg.layers):
        ora.kc[l], ora.vc[l] = dev.dec.kv_rows(l, cfg.seq_len)
    toks = np.random.default_rng(5).integers(0, cfg.vocab, 2)
    for i, t in enumerate(toks):
        want = np.asarray(ora.forward(int(t), P + i), np.float32)
        got = dev.forward(int(t))
        assert got.tobytes() == want.tobytes(), f"step {i}"
        assert int(np.argmax(got)) == int(np.argmax(want))
    k, v = dev.dec.kv_rows(cfg.layers - 1, P + 2)
    assert np.array_equal(k, ora.kc[cfg.layers - 1, :P + 2]) and np.array_equal(v, ora.vc[cfg.layers - 1, :P + 2])
