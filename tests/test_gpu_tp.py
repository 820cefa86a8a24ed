"""Tensor parallelism on 2+ GPUs (one process per GPU, NCCL): every rank's
logits and greedy tokens equal the one-GPU decoder's (itself bit-exact with the
reference) bit for bit, through the prefill GEMM path (NCCL collectives), the
decode rows' in-kernel NVLink exchange, and the captured on-device greedy loop.
Skipped with fewer than 2 GPUs (ranks must be on distinct GPUs)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from torch2riscv_accelerator_b200 import config as C
from torch2riscv_accelerator_b200 import weights as W

pytestmark = pytest.mark.gpu
PREFILL, CHUNK2, FWD, STEPS = 40, 10, 5, 6


CFG = C.C2.with_(layers=2, vocab=4096)


def _model(kv=None, act="silu", channel=""):
    """The test model: the quantized weights are elementwise functions of the
    seed (identical in every process); the KV scales come from one fp32
    calibration run (BLAS sums), made once in the parent and handed to the ranks."""
    cfg = CFG.with_(act=act)
    if kv is None:
        qw = W.QuantWeights(cfg, seed=7, gains="random", calib_tokens=np.arange(8), kv_channel=channel)
        kv = qw.kv_scales
    else:
        qw = W.QuantWeights(cfg, seed=7, gains="random")
    toks = np.random.default_rng(3).integers(0, cfg.vocab, PREFILL + CHUNK2 + FWD)
    return cfg, qw, np.asarray(kv, np.float32), toks


def _run(dev, toks):
    """prefill (a 40-row and a 10-row chunk), FWD single-token forwards, then
    STEPS replays of the captured greedy step: logits and tokens of each."""
    out = {"p1": dev.prefill(toks[:PREFILL]), "p2": dev.prefill(toks[PREFILL:PREFILL + CHUNK2])}
    out["fwd"] = np.stack([dev.forward(int(t)) for t in toks[PREFILL + CHUNK2:]])
    dec = dev.dec
    g = dec.capture_decode_step(int(np.argmax(out["fwd"][-1])), dev.pos - 1)
    tok, lg = [], []
    for _ in range(STEPS):
        g.replay()
        tok.append(int(dec.next_token[0].item()))
        full = dec.gather_logits(1)[0] if hasattr(dec, "gather_logits") else dec.logits[0]
        lg.append(full.cpu().numpy())
    out["loop_tok"], out["loop_lg"] = np.array(tok), np.stack(lg)
    return out


def _worker(rank, ranks, port, path, kv, act):
    from torch2riscv_accelerator_b200 import ops
    from torch2riscv_accelerator_b200.tp import TpLlamaDevice
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=ranks,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    dev = None
    try:
        cfg, qw, kv, toks = _model(kv, act)
        dev = TpLlamaDevice((cfg, qw, kv))
        out = _run(dev, toks)
        torch.cuda.synchronize()
        out["flags"] = np.array(ops.error_flags())
        np.savez(f"{path}.{rank}.npz", **out)
    finally:
        if dev is not None:
            dev.close()
        dist.destroy_process_group()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("ranks,act,channel", [(2, "silu", ""), (2, "gelu_tanh", ""), (2, "silu", "kv"),
                                               (4, "silu", ""), (8, "silu", "kv")])
def test_tp_equals_one_gpu(ranks, act, channel, tmp_path):
    """channel "kv": per-channel KV scales, each rank holding its KV heads' channels."""
    if torch.cuda.device_count() < ranks:
        pytest.skip(f"needs {ranks} GPUs")
    from torch2riscv_accelerator_b200.runtime import LlamaDevice
    path = str(tmp_path / "tp")
    cfg, qw, kv, toks = _model(act=act, channel=channel)
    mp.spawn(_worker, args=(ranks, _port(), path, kv, act), nprocs=ranks, join=True)
    ref = _run(LlamaDevice((cfg, qw, kv)), toks)
    for r in range(ranks):
        got = np.load(f"{path}.{r}.npz")
        assert int(got["flags"]) == 0, (r, int(got["flags"]))
        for k in ("p1", "p2", "fwd", "loop_tok", "loop_lg"):
            assert got[k].tobytes() == ref[k].tobytes(), (r, k)


BATCH, BSTEPS = 20, 4


def _batch_inputs():
    rng = np.random.default_rng(11)
    seqs = rng.integers(0, CFG.vocab, (BSTEPS, BATCH))
    offs = rng.integers(0, 40, BATCH)                       # slot b runs positions offs[b] ...
    return seqs, offs


def _batch_worker(rank, ranks, port, path, kv, graphs):
    from torch2riscv_accelerator_b200 import ops
    from torch2riscv_accelerator_b200.tp import TpBatchLlamaDevice
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=ranks,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    dev = None
    try:
        cfg, qw, kv, _ = _model(kv)
        dev = TpBatchLlamaDevice((cfg, qw, kv), slots=BATCH, graphs=graphs)
        seqs, offs = _batch_inputs()
        lg = np.stack([dev.step([int(o) + s for o in offs], [int(t) for t in seqs[s]]) for s in range(BSTEPS)])
        torch.cuda.synchronize()
        np.savez(f"{path}.{rank}.npz", lg=lg, flags=np.array(ops.error_flags()))
    finally:
        if dev is not None:
            dev.close()                                # its graph holds NCCL work: released first
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("graphs", [False, True])
@pytest.mark.parametrize("ranks", [2, 4, 8])
def test_tp_batch_equals_one_gpu(ranks, graphs, tmp_path):
    """Batched decode (20 slots at their own positions) over `ranks` GPUs, the
    step launched eagerly or replayed as one CUDA graph with its NCCL
    all-reduces: the full [D, vocab] logits of every step equal the one-GPU
    BatchDecoder's."""
    if torch.cuda.device_count() < ranks:
        pytest.skip(f"needs {ranks} GPUs")
    from torch2riscv_accelerator_b200.runtime import BatchLlamaDevice
    path = str(tmp_path / "tpb")
    cfg, qw, kv, _ = _model()
    mp.spawn(_batch_worker, args=(ranks, _port(), path, kv, graphs), nprocs=ranks, join=True)
    dev = BatchLlamaDevice((cfg, qw, kv), slots=BATCH)
    seqs, offs = _batch_inputs()
    ref = np.stack([dev.step([int(o) + s for o in offs], [int(t) for t in seqs[s]]) for s in range(BSTEPS)])
    for r in range(ranks):
        got = np.load(f"{path}.{r}.npz")
        assert int(got["flags"]) == 0
        assert got["lg"].tobytes() == ref.tobytes(), r

