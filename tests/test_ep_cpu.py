"""Expert parallelism's algebra on the CPU: the router whole on every rank,
each rank's experts' terms w_j * y_j (zeros elsewhere) summed over gloo ranks,
then the k-order fold, equals the one-device MoE FFN (the oracle's
moe_ffn_row) bit for bit; the expert shards tile the experts."""
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import model as OM
from torch2riscv_accelerator_b200 import config as C
from torch2riscv_accelerator_b200 import weights as W
from torch2riscv_accelerator_b200.ep import EXPERT_KEYS, check_ep, shard_experts

CFG = C.tiny("ep", experts=8, top_k=3, expert_hidden=32, rope="hf", attn="qsum", theta=1e6, tied=True)


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, ranks, port):
    from tp_sim import moe_ep_row
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=ranks)
    try:
        qw = W.QuantWeights(CFG, seed=4, gains="random")
        n = CFG.experts // ranks
        rng = np.random.default_rng(6)
        for l, t in enumerate(qw.layers):
            for _ in range(6):
                x = (rng.standard_normal(CFG.dim) * 0.5).astype(np.float32)
                y = moe_ep_row(x, t, CFG, rank * n, n)
                want, _, _ = OM.moe_ffn_row(x, t, CFG)
                assert y.tobytes() == want.tobytes(), l
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("ranks", [2, 4])
def test_expert_parallel_terms_equal_moe(ranks):
    mp.spawn(_worker, args=(ranks, _port()), nprocs=ranks, join=True)


def test_expert_shards_tile_the_experts():
    qw = W.QuantWeights(CFG, seed=4, gains="random")
    sh = [shard_experts(CFG, qw, r, 4) for r in range(4)]
    for l, t in enumerate(qw.layers):
        for k in EXPERT_KEYS:
            assert np.array_equal(np.concatenate([s.layers[l][k] for s in sh]), t[k])
        assert all(s.layers[l]["router"] is t["router"] for s in sh)
    assert [s.expert_lo for s in sh] == [0, 2, 4, 6]
    with pytest.raises(ValueError):
        check_ep(CFG, 3)
    with pytest.raises(ValueError):
        check_ep(C.C2, 2)
