"""Expert parallelism on 2+ GPUs (one process per GPU, NCCL): the MoE decoder
with 1/ranks of the experts per rank gives the one-GPU decoder's logits and
greedy tokens bit for bit (prefill chunks, single-token forwards, the on-device
greedy loop, batched decode). Skipped with fewer than 2 GPUs."""
import datetime
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from torch2riscv_accelerator_b200 import config as C
from torch2riscv_accelerator_b200 import weights as W

pytestmark = pytest.mark.gpu
CFG = C.C4.with_(layers=2, vocab=4096)
PREFILL, FWD, STEPS, BATCH = 40, 4, 5, 20


def _model(kv=None):
    """Weights are elementwise functions of the seed; the KV scales (one fp32
    calibration run) are made once in the parent and handed to the ranks."""
    if kv is None:
        qw = W.QuantWeights(CFG, seed=9, gains="random", calib_tokens=np.arange(8))
        kv = qw.kv_scales
    else:
        qw = W.QuantWeights(CFG, seed=9, gains="random")
    return CFG, qw, np.asarray(kv, np.float32)


def _run(dev):
    """prefill (NCCL path), forwards (the exchange, captured), then the
    captured greedy step replayed STEPS times."""
    toks = np.random.default_rng(3).integers(0, CFG.vocab, PREFILL + FWD)
    out = {"p": dev.prefill(toks[:PREFILL])}
    out["fwd"] = np.stack([dev.forward(int(t)) for t in toks[PREFILL:]])
    dec = dev.dec
    g = dec.capture_decode_step(int(np.argmax(out["fwd"][-1])), dev.pos - 1)
    tok, lg = [], []
    for _ in range(STEPS):
        g.replay()
        tok.append(int(dec.next_token[0].item()))
        lg.append(dec.logits[0].cpu().numpy())
    out["loop_tok"], out["loop_lg"] = np.array(tok), np.stack(lg)
    rng = np.random.default_rng(11)
    return out, rng.integers(0, CFG.vocab, (3, BATCH)), rng.integers(0, 40, BATCH)


def _batch(dev, seqs, offs):
    return np.stack([dev.step([int(o) + s for o in offs], [int(t) for t in seqs[s]]) for s in range(len(seqs))])


def _worker(rank, ranks, port, path, kv):
    from torch2riscv_accelerator_b200 import ops
    from torch2riscv_accelerator_b200.ep import EpBatchLlamaDevice, EpLlamaDevice
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=ranks,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    try:
        model = _model(kv)
        dev = EpLlamaDevice(model)
        out, seqs, offs = _run(dev)
        dev.close()
        out["batch"] = _batch(EpBatchLlamaDevice(model, slots=BATCH), seqs, offs)
        torch.cuda.synchronize()
        out["flags"] = np.array(ops.error_flags())
        np.savez(f"{path}.{rank}.npz", **out)
    finally:
        dist.destroy_process_group()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("ranks", [2, 4, 8])
def test_ep_equals_one_gpu(ranks, tmp_path):
    if torch.cuda.device_count() < ranks:
        pytest.skip(f"needs {ranks} GPUs")
    from torch2riscv_accelerator_b200.runtime import BatchLlamaDevice, LlamaDevice
    path = str(tmp_path / "ep")
    model = _model()
    mp.spawn(_worker, args=(ranks, _port(), path, model[2]), nprocs=ranks, join=True)
    ref, seqs, offs = _run(LlamaDevice(model))
    ref["batch"] = _batch(BatchLlamaDevice(model, slots=BATCH), seqs, offs)
    for r in range(ranks):
        got = np.load(f"{path}.{r}.npz")
        assert int(got["flags"]) == 0, (r, int(got["flags"]))
        for k in ("p", "fwd", "loop_tok", "loop_lg", "batch"):
            assert got[k].tobytes() == ref[k].tobytes(), (r, k)
