"""Batched decode (BatchLlamaDevice, `llm/runtime.py:155-241`): D slots with
their own caches and positions, one tensor-core GEMM per linear over the D
rows, one attention launch over all slots. Every slot's logits equal the
one-sequence runtime's (itself bit-exact with the reference) bit for bit."""
import numpy as np
import pytest

from conftest import golden
from torch2riscv_accelerator_b200 import config as C
from torch2riscv_accelerator_b200 import weights as W
from torch2riscv_accelerator_b200.runtime import BatchLlamaDevice, LlamaDevice

pytestmark = pytest.mark.gpu
F = np.float32


def _single(model, toks):
    """Logits of each position of one sequence through the one-sequence runtime."""
    dev = LlamaDevice(model)
    return [dev.forward(int(t)) for t in toks]


@pytest.mark.parametrize("graphs", [True, False])
def test_batch_generate_slots_equal_single_sequences(graphs):
    g = golden("dm_tiny.npz")
    dim, hidden, layers, heads, kv_heads, vocab, seq = [int(v) for v in g["a_cfg"]]
    cfg = C.ModelConfig("tiny-a", dim, hidden, layers, heads, kv_heads, dim // heads, vocab, seq,
                        theta=10000.0, eps=1e-5, tied=False, attn="norm", rope="llama2c")
    w = {n[4:]: g[n] for n in g.files if n.startswith("a_w_")}
    qw = W.from_fp32(cfg, w)
    kv = np.asarray(g["a_kv"], F) if "a_kv" in g.files else np.full((layers, 2), 0.05, F)
    rng = np.random.default_rng(9)
    prompts = [list(rng.integers(0, vocab, n)) for n in (5, 9, 3)]
    seen = {}
    dev = BatchLlamaDevice((cfg, qw, kv), slots=4, graphs=graphs)    # one slot stays idle (dummy rows)
    out = dev.generate(prompts, steps=12, stagger=2, on_logits=lambda b, p, lg: seen.__setitem__((b, p), lg))
    for b, toks in enumerate(out):
        ref = _single((cfg, qw, kv), toks)
        for p in range(12):
            assert seen[(b, p)].tobytes() == ref[p].tobytes(), (b, p)


@pytest.mark.parametrize("name,channel", [("C2", ""), ("C4", ""), ("C2", "kv"), ("C1", "")])
def test_batch_step_full_dims_mixed_positions(name, channel):
    """C2 (dense, QK-norm, 128-dim heads), C4 (MoE; 64-dim heads, 6 ring
    stages) or C1 (3 query heads per KV head, 5 ring stages) dimensions, 2
    layers, 20 slots (GEMMs of 20 rows, the MoE grouped by expert), each slot at
    its own position after a slot-specific history; C2 also with per-channel KV
    scales (the batched stream kernel's per-channel path)."""
    cfg = getattr(C, name).with_(layers=2, vocab=4096)
    qw = W.QuantWeights(cfg, seed=7, gains="random", calib_tokens=np.arange(8), kv_channel=channel)
    kv = qw.kv_scales                                               # (per cache channel with "kv")
    D, steps = 20, 4
    rng = np.random.default_rng(11)
    seqs = [list(rng.integers(0, cfg.vocab, steps)) for _ in range(D)]
    offs = rng.integers(0, 40, D)                                   # slot b runs positions offs[b] ...
    dev = BatchLlamaDevice((cfg, qw, kv), slots=D)
    got = [[None] * steps for _ in range(D)]
    for s in range(steps):
        lg = dev.step([int(offs[b]) + s for b in range(D)], [int(seqs[b][s]) for b in range(D)])
        for b in range(D):
            got[b][s] = lg[b]
    for b in (0, 7, 15, 16, 19):
        single = LlamaDevice((cfg, qw, kv))
        single.pos = int(offs[b])                                   # the same (empty) history before offs[b]
        for s in range(steps):
            assert single.forward(int(seqs[b][s])).tobytes() == got[b][s].tobytes(), (b, s)
