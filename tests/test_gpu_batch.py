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


@pytest.mark.parametrize("name,channel", [("C2", ""), ("C4", ""), ("C2", "kv"), ("C1", ""), ("C3", "")])
def test_batch_step_full_dims_mixed_positions(name, channel):
    """C2 (dense, QK-norm, 128-dim heads), C4 (MoE; 64-dim heads, 6 ring
    stages), C1 (3 query heads per KV head, 5 ring stages) or C3 (4 query heads
    per KV head, 64-dim heads, dim 2048, hidden 8192) dimensions, 2
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


def test_batch_step_against_the_oracle():
    """Batched decode checked against the oracle directly (not only against the
    one-sequence GPU runtime): C3 dimensions (32 / 8 heads of 64), 2 layers, 18
    slots at their own positions after their own histories; slots 0, 9 and 17
    re-run on the oracle from the same tokens, logits bit for bit."""
    from oracle import model as OM
    cfg = C.C3.with_(layers=2, vocab=2048)
    qw = W.QuantWeights(cfg, seed=3, gains="random", calib_tokens=np.arange(8))
    kv = qw.kv_scales
    D, steps = 18, 3
    rng = np.random.default_rng(21)
    hist = [list(rng.integers(0, cfg.vocab, int(n))) for n in rng.integers(1, 12, D)]
    dev = BatchLlamaDevice((cfg, qw, kv), slots=D)
    for b in range(D):
        dev.clear_slot(b)
    L = max(len(h) for h in hist)
    last = [None] * D
    for s in range(L):                                              # each slot's own history, then stops
        live = [s < len(hist[b]) for b in range(D)]
        lg = dev.step([s if live[b] else 0 for b in range(D)], [hist[b][s] if live[b] else 0 for b in range(D)])
        for b in range(D):
            if live[b] and s == len(hist[b]) - 1:
                last[b] = lg[b].copy()
    for b in (0, 9, 17):
        ora = OM.OracleDecoder(cfg, qw, kv)
        for p, t in enumerate(hist[b]):
            want = np.asarray(ora.forward(int(t), p), np.float32)
        assert want.tobytes() == last[b].tobytes(), b
