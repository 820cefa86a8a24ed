"""torch.ops.w8a8.*: registered through torch.library with the schemas of the
C ABI's operators, and fake (meta) implementations that give the output shapes
and dtypes without a GPU."""
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import torch2riscv_accelerator_b200.torch_ops as T


def test_every_op_is_registered():
    for name in T.OPS:
        assert hasattr(torch.ops.w8a8, name), name
    assert str(torch.ops.w8a8.linear.default._schema) == \
        "w8a8::linear(Tensor xq, Tensor s_x, Tensor w, Tensor s_w) -> Tensor"


def test_fake_shapes():
    with FakeTensorMode():
        x = torch.empty(3, 64)
        w = torch.empty(32, 64, dtype=torch.int8)
        s = torch.empty(32)
        xq, sx = torch.ops.w8a8.quant_act(x)
        assert xq.shape == (3, 64) and xq.dtype == torch.int8 and sx.shape == (3,)
        assert torch.ops.w8a8.linear(xq, sx, w, s).shape == (3, 32)
        assert torch.ops.w8a8.linear_fused(x, w, s, None, 1e-5).shape == (3, 32)
        h, hq, sh = torch.ops.w8a8.ffn_swiglu(x, torch.empty(64), 1e-5, w, s, w, s)
        assert h.shape == (3, 32) and hq.dtype == torch.int8 and sh.shape == (3,)
        tok = torch.empty(5, dtype=torch.int32)
        assert torch.ops.w8a8.embed(tok, torch.empty(100, 64, dtype=torch.int8), torch.empty(100)).shape == (5, 64)
