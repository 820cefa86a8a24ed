"""The reference-facing surface on the GPU: LlamaDevice built from a .w8a8 path
(the reference's constructor, llm/runtime.py:75-97), DeviceRig in the place of
the functional simulator's test rig (llm/test_l4.py:58-85 over
llm/sa_funcsim.py:420), and torch.ops.w8a8.* giving the ops.py results bit for
bit. The tiny model "a" of dm_tiny.npz (DeviceModel(SfuExact) logits and KV)
and its .w8a8 file from the reference's exporter pin the results."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden
from torch2riscv_accelerator_b200 import ops
from torch2riscv_accelerator_b200.loaders import read_w8a8
from torch2riscv_accelerator_b200.runtime import DeviceRig, LlamaDevice

pytestmark = pytest.mark.gpu
W8A8_FILE = os.path.join(GOLDEN, "tiny_a_d8.w8a8")


def test_llamadevice_from_a_model_path():
    g = golden("dm_tiny.npz")
    for dev in (LlamaDevice(W8A8_FILE), LlamaDevice.from_w8a8(W8A8_FILE, tokenizer_path=None)):
        for p, t in enumerate(g["tokens"]):
            assert dev.forward(int(t)).tobytes() == g["a_logits"][p].tobytes(), p


def test_device_rig_runs_the_program_like_the_funcsim_rig():
    g = golden("dm_tiny.npz")
    rig = DeviceRig(W8A8_FILE)
    prog = rig.program()
    toks = g["tokens"]
    for p, t in enumerate(toks):
        n = rig.run(prog, p, int(t))
        assert n == rig.dec.kernel_launches(1)
        assert rig.logits().tobytes() == g["a_logits"][p].tobytes(), p
    kv = rig.kv_cache()
    n = len(toks)
    assert np.array_equal(kv[:, 0, :n], g["a_kc"][:, :n]) and np.array_equal(kv[:, 1, :n], g["a_vc"][:, :n])
    with pytest.raises(RuntimeError):                     # a token outside the vocabulary: the error flag
        rig.run(prog, 0, rig.cfg.vocab + 5)


def test_torch_ops_equal_the_c_abi_bindings():
    import torch2riscv_accelerator_b200.torch_ops  # noqa: F401  (registers torch.ops.w8a8)
    cfg, m, kv = read_w8a8(W8A8_FILE)
    dev = torch.device("cuda")
    rng = np.random.default_rng(4)
    x = torch.as_tensor(rng.standard_normal((3, cfg.dim)).astype(np.float32), device=dev)
    t = {k: torch.as_tensor(v, device=dev) for k, v in m.layers[0].items()}
    bits = lambda a: a.cpu().numpy().tobytes()
    xq, sx = torch.ops.w8a8.quant_act(x)
    xq2, sx2 = ops.quant_act(x)
    assert bits(xq) == bits(xq2) and bits(sx) == bits(sx2)
    assert bits(torch.ops.w8a8.linear(xq, sx, t["wo"], t["s_wo"])) == bits(ops.linear(xq, sx, t["wo"], t["s_wo"]))
    assert bits(torch.ops.w8a8.gemm(xq, sx, t["wo"], t["s_wo"])) == bits(ops.linear(xq, sx, t["wo"], t["s_wo"]))
    assert bits(torch.ops.w8a8.rmsnorm(x, t["rms_att"], 1e-5)) == bits(ops.rmsnorm(x, t["rms_att"], 1e-5))
    assert bits(torch.ops.w8a8.linear_fused(x, t["wqkv"], t["s_wqkv"], t["rms_att"], 1e-5)) == \
        bits(ops.linear_fused(x, t["wqkv"], t["s_wqkv"], norm_g=t["rms_att"], eps=1e-5))
    h, hq, sh = torch.ops.w8a8.ffn_swiglu(x, t["rms_ffn"], 1e-5, t["w1"], t["s_w1"], t["w3"], t["s_w3"])
    h2, hq2, sh2 = ops.ffn_swiglu(x, t["rms_ffn"], 1e-5, t["w1"], t["s_w1"], t["w3"], t["s_w3"],
                                  ops.ffn_scratch(3, dev))
    assert bits(h) == bits(h2) and bits(hq) == bits(hq2) and bits(sh) == bits(sh2)
    tok = torch.tensor([1, 5, 7], dtype=torch.int32, device=dev)
    eq, es = torch.as_tensor(m.emb_q, device=dev), torch.as_tensor(m.emb_s, device=dev)
    assert bits(torch.ops.w8a8.embed(tok, eq, es)) == bits(ops.embed(tok, eq, es))
    cq, cs, rf = (torch.as_tensor(a, device=dev) for a in (m.cls_q, m.cls_s, m.rms_final))
    assert bits(torch.ops.w8a8.classifier(x, cq, cs, rf, 1e-5)) == bits(ops.classifier(x, cq, cs, rf, 1e-5))
    assert bits(torch.ops.w8a8.sfu(0, x)) == bits(ops.sfu(0, x))
    assert ops.error_flags() == 0
