"""`torch.ops.w8a8.*`: the main operators of the C ABI registered with
torch.library, for callers that hold torch tensors (the host side of the
reference's `llm/compile_model.py` dispatches: quant_act, the W8A8 linear,
RMSNorm, the fused SwiGLU, embedding, the classifier; `llm/sa_funcsim.py`'s
SFU). Each op allocates its outputs and calls the same C entry point as
`ops.py` on the current stream; a fake (meta) implementation gives the output
shapes for tracing. Importing this module registers them:

    import torch2riscv_accelerator_b200.torch_ops
    xq, s_x = torch.ops.w8a8.quant_act(x)
    y = torch.ops.w8a8.linear(xq, s_x, w, s_w)

There is no CPU kernel: on a CPU tensor the C ABI refuses the call.
"""
import torch

from . import ops

_LIB = "w8a8"


@torch.library.custom_op(f"{_LIB}::quant_act", mutates_args=())
def quant_act(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """x [rows, k] fp32 -> (int8 rows, scales [rows]) (llm/ref_model.py:191-196)."""
    return ops.quant_act(x)


@quant_act.register_fake
def _(x):
    return torch.empty(x.shape, dtype=torch.int8, device=x.device), x.new_empty(x.shape[0])


@torch.library.custom_op(f"{_LIB}::rmsnorm", mutates_args=())
def rmsnorm(x: torch.Tensor, g: torch.Tensor, eps: float) -> torch.Tensor:
    """(x * RSQRT(red_sum16(x * x) / n + eps)) * g per row (llm/ref_model.py:204-207)."""
    return ops.rmsnorm(x, g, eps)


@rmsnorm.register_fake
def _(x, g, eps):
    return torch.empty_like(x)


@torch.library.custom_op(f"{_LIB}::linear", mutates_args=())
def linear(xq: torch.Tensor, s_x: torch.Tensor, w: torch.Tensor, s_w: torch.Tensor) -> torch.Tensor:
    """(f32(xq . W^T) * s_w) * s_x on int8 rows, up to 16 of them (llm/ref_model.py:198-202)."""
    return ops.linear(xq, s_x, w, s_w)


@linear.register_fake
def _(xq, s_x, w, s_w):
    return xq.new_empty((xq.shape[0], w.shape[0]), dtype=torch.float32)


@torch.library.custom_op(f"{_LIB}::gemm", mutates_args=())
def gemm(xq: torch.Tensor, s_x: torch.Tensor, w: torch.Tensor, s_w: torch.Tensor) -> torch.Tensor:
    """The same linear for any row count on the tensor cores (tcgen05 kind::i8)."""
    return ops.gemm(xq, s_x, w, s_w)


@gemm.register_fake
def _(xq, s_x, w, s_w):
    return xq.new_empty((xq.shape[0], w.shape[0]), dtype=torch.float32)


@torch.library.custom_op(f"{_LIB}::linear_fused", mutates_args=())
def linear_fused(x: torch.Tensor, w: torch.Tensor, s_w: torch.Tensor, norm_g: torch.Tensor | None,
                 eps: float) -> torch.Tensor:
    """[rmsnorm ->] quant_act -> linear on fp32 rows (the decode GEMV with its fused prologue)."""
    return ops.linear_fused(x, w, s_w, norm_g=norm_g, eps=eps)


@linear_fused.register_fake
def _(x, w, s_w, norm_g, eps):
    return x.new_empty((x.shape[0], w.shape[0]))


@torch.library.custom_op(f"{_LIB}::ffn_swiglu", mutates_args=())
def ffn_swiglu(x: torch.Tensor, norm_g: torch.Tensor, eps: float, w_gate: torch.Tensor, s_gate: torch.Tensor,
               w_up: torch.Tensor, s_up: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Decode's fused SwiGLU dispatch: (h, int8 h, its scales) (llm/compile_model.py:295-328)."""
    scratch = ops.ffn_scratch(x.shape[0], x.device)
    h, hq, sh = ops.ffn_swiglu(x, norm_g, eps, w_gate, s_gate, w_up, s_up, scratch)
    return h, hq, sh


@ffn_swiglu.register_fake
def _(x, norm_g, eps, w_gate, s_gate, w_up, s_up):
    m, n = x.shape[0], w_gate.shape[0]
    return (x.new_empty((m, n)), torch.empty((m, n), dtype=torch.int8, device=x.device), x.new_empty(m))


@torch.library.custom_op(f"{_LIB}::embed", mutates_args=())
def embed(tokens: torch.Tensor, emb_q: torch.Tensor, emb_s: torch.Tensor) -> torch.Tensor:
    """f32(emb_q[token]) * emb_s[token] per token (llm/compile_model.py:192-201)."""
    return ops.embed(tokens, emb_q, emb_s)


@embed.register_fake
def _(tokens, emb_q, emb_s):
    return emb_s.new_empty((tokens.numel(), emb_q.shape[1]))


@torch.library.custom_op(f"{_LIB}::classifier", mutates_args=())
def classifier(x: torch.Tensor, w: torch.Tensor, s_w: torch.Tensor, norm_g: torch.Tensor, eps: float) -> torch.Tensor:
    """Final rmsnorm -> quant_act -> classifier GEMV (llm/compile_model.py:347-349)."""
    return ops.classifier(x, w, s_w, norm_g, eps)


@classifier.register_fake
def _(x, w, s_w, norm_g, eps):
    return x.new_empty((x.shape[0], w.shape[0]))


@torch.library.custom_op(f"{_LIB}::sfu", mutates_args=())
def sfu(func: int, x: torch.Tensor) -> torch.Tensor:
    """The overlay's table SFU elementwise: 0 EXP, 1 RECIP, 2 RSQRT, 3 SiLU, 4 GELU-tanh (llm/sfu.py)."""
    return ops.sfu(func, x)


@sfu.register_fake
def _(func, x):
    return torch.empty_like(x)


OPS = ("quant_act", "rmsnorm", "linear", "gemm", "linear_fused", "ffn_swiglu", "embed", "classifier", "sfu")
