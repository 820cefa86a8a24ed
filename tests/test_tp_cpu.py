"""Tensor parallelism's host side on the CPU: the shards tile the model, and the
sharded program (tests/tp_sim.py: the oracle over one rank's shard, with gloo
collectives for the exchanges) equals the unsharded oracle bit for bit on 2 and
4 ranks, rows of a chunk and single rows alike, KV cache included."""
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import model as OM
from torch2riscv_accelerator_b200 import config as C
from torch2riscv_accelerator_b200 import weights as W
from torch2riscv_accelerator_b200.tp import check_split, local_config, shard

CFG_NORM = C.tiny("tp-norm", heads=8, kv_heads=4, hidden=128, vocab=96)
CFG_QSUM = C.tiny("tp-qsum", heads=8, kv_heads=4, hidden=128, vocab=96, qk_norm=True, attn="qsum", rope="hf",
                  theta=1e6, eps=1e-6, tied=True)


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, ranks, port, cfg, seed):
    from tp_sim import TpOracle
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=ranks)
    try:
        qw = W.QuantWeights(cfg, seed=seed, gains="random", calib_tokens=np.arange(8))
        ref = OM.OracleDecoder(cfg, qw, qw.kv_scales)
        tp = TpOracle(cfg, qw, qw.kv_scales, rank, ranks)
        toks = np.random.default_rng(seed).integers(0, cfg.vocab, 12)
        a = tp.forward_rows(toks[:7], np.arange(7), all_logits=True)
        b = ref.forward_rows(toks[:7], np.arange(7), all_logits=True)
        assert a.tobytes() == b.tobytes(), "chunk logits"
        for p in range(7, 12):
            assert tp.forward(int(toks[p]), p).tobytes() == ref.forward(int(toks[p]), p).tobytes(), p
        w = cfg.kv_heads // ranks * cfg.head_dim
        assert np.array_equal(tp.kc[:, :12], ref.kc[:, :12, rank * w:(rank + 1) * w])
        assert np.array_equal(tp.vc[:, :12], ref.vc[:, :12, rank * w:(rank + 1) * w])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("cfg,ranks", [(CFG_NORM, 2), (CFG_QSUM, 2), (CFG_QSUM, 4)])
def test_sharded_oracle_equals_oracle(cfg, ranks):
    mp.spawn(_worker, args=(ranks, _port(), cfg, 5), nprocs=ranks, join=True)


@pytest.mark.parametrize("ranks", [2, 4])
def test_shards_tile_the_model(ranks):
    cfg = CFG_QSUM
    qw = W.QuantWeights(cfg, seed=2, gains="random")
    sh = [shard(cfg, qw, r, ranks) for r in range(ranks)]
    qd, kd = cfg.q_dim, cfg.kv_dim
    lc = local_config(cfg, ranks)
    for l, t in enumerate(qw.layers):
        u = [s.layers[l] for s in sh]
        q = np.concatenate([x["wqkv"][:lc.q_dim] for x in u])
        k = np.concatenate([x["wqkv"][lc.q_dim:lc.q_dim + lc.kv_dim] for x in u])
        v = np.concatenate([x["wqkv"][lc.q_dim + lc.kv_dim:] for x in u])
        assert np.array_equal(np.concatenate([q, k, v]), t["wqkv"])
        assert np.array_equal(np.concatenate([x["s_wqkv"][:lc.q_dim] for x in u]), t["s_wqkv"][:qd])
        assert np.array_equal(np.concatenate([x["wo"] for x in u], axis=1), t["wo"])
        assert np.array_equal(np.concatenate([x["w1"] for x in u]), t["w1"])
        assert np.array_equal(np.concatenate([x["w3"] for x in u]), t["w3"])
        assert np.array_equal(np.concatenate([x["w2"] for x in u], axis=1), t["w2"])
        assert all(x["s_wo"] is t["s_wo"] and x["s_w2"] is t["s_w2"] for x in u)
        assert kd == ranks * lc.kv_dim
    assert np.array_equal(np.concatenate([s.cls_q for s in sh]), qw.cls_q)
    assert [s.vocab_offset for s in sh] == [r * cfg.vocab // ranks for r in range(ranks)]


def test_split_rejects_what_does_not_divide():
    with pytest.raises(ValueError):
        check_split(C.C1, 2)                       # 3 KV heads
    with pytest.raises(ValueError):
        check_split(C.C4, 2)                       # MoE: split by expert instead
    with pytest.raises(ValueError):
        check_split(C.C2, 16)                      # more ranks than the exchange holds
    for r in (2, 4, 8):
        check_split(C.C2, r)
        check_split(C.C3, r)
