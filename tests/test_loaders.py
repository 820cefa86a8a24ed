"""Model files: the reference's .w8a8 device format and llama2.c checkpoints
(fixtures written by the reference's own exporter and checked against its
reader in tests/golden/make_golden.py)."""
import os

import numpy as np
import pytest

from conftest import GOLDEN, golden
from oracle import model as OM
from torch2riscv_accelerator_b200 import weights as W
from torch2riscv_accelerator_b200.loaders import load_llama2c, read_w8a8, write_w8a8

F = np.float32
W8A8_FILE = os.path.join(GOLDEN, "tiny_a_d8.w8a8")
BIN_FILE = os.path.join(GOLDEN, "tiny_a.bin")


def _logits_of(cfg, qw, kv, tokens):
    ora = OM.OracleDecoder(cfg, qw, kv)
    return np.stack([ora.forward(int(t), p) for p, t in enumerate(tokens)]), ora


def test_w8a8_file_reproduces_reference_logits_and_kv():
    """The reference's .w8a8 export of tiny model "a" (D = 8), read into this
    runtime's layout: every token's logits and the int8 KV cache equal the
    reference DeviceModel's."""
    g = golden("dm_tiny.npz")
    cfg, m, kv = read_w8a8(W8A8_FILE)
    assert (cfg.dim, cfg.hidden, cfg.layers, cfg.heads, cfg.vocab, cfg.seq_len) == tuple(
        int(v) for v in g["a_cfg"][[0, 1, 2, 3, 5, 6]])
    assert np.array_equal(kv, g["a_kv"])
    lg, ora = _logits_of(cfg, m, kv, g["tokens"])
    assert lg.tobytes() == g["a_logits"].tobytes()
    n = len(g["tokens"])
    assert np.array_equal(ora.kc[:, :n], g["a_kc"][:, :n]) and np.array_equal(ora.vc[:, :n], g["a_vc"][:, :n])


def test_w8a8_writer_is_byte_identical_to_the_reference_exporter(tmp_path):
    cfg, m, kv = read_w8a8(W8A8_FILE)
    out = str(tmp_path / "again.w8a8")
    write_w8a8(out, cfg, m, kv, d=8)
    assert open(out, "rb").read() == open(W8A8_FILE, "rb").read()


def test_w8a8_rejects_foreign_bytes():
    with pytest.raises(ValueError):
        read_w8a8(b"\0" * 128)
    raw = bytearray(open(W8A8_FILE, "rb").read())
    raw[8] = 7                                                       # version
    with pytest.raises(ValueError):
        read_w8a8(bytes(raw))


def test_llama2c_checkpoint_roundtrip_and_logits():
    """llama2.c legacy checkpoint of the same model: the fp32 tensors come back
    exactly; quantized here, the oracle's logits equal the reference's."""
    g = golden("dm_tiny.npz")
    cfg, w = load_llama2c(BIN_FILE)
    for k in ("tok", "wq", "wk", "wv", "wo", "w1", "w2", "w3", "rms_att", "rms_ffn", "rms_final", "wcls"):
        assert np.array_equal(w[k], g[f"a_w_{k}"]), k
    lg, _ = _logits_of(cfg, W.from_fp32(cfg, w), g["a_kv"], g["tokens"])
    assert lg.tobytes() == g["a_logits"].tobytes()


def test_llama2c_rejects_a_truncated_file(tmp_path):
    data = open(BIN_FILE, "rb").read()
    p = tmp_path / "cut.bin"
    p.write_bytes(data[:-4])
    with pytest.raises(ValueError):
        load_llama2c(str(p))


@pytest.mark.gpu
def test_w8a8_file_on_the_gpu():
    from torch2riscv_accelerator_b200.runtime import LlamaDevice
    g = golden("dm_tiny.npz")
    cfg, m, kv = read_w8a8(W8A8_FILE)
    dev = LlamaDevice((cfg, m, kv))
    for p, t in enumerate(g["tokens"]):
        assert dev.forward(int(t)).tobytes() == g["a_logits"][p].tobytes(), p
