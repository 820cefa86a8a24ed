"""Model configurations of the W8A8 decode path.

Field meanings follow the reference's two config types: `llm/checkpoint.py:15-30`
(llama2.c: dim, hidden, layers, heads, kv_heads, vocab, seq_len) and
`compiler/frontend/qhf.py:97-121` (HFConfig: decoupled head_dim, QK-norm, RoPE
theta, eps, tied embeddings), plus the Mixtral-style MoE block of
`compiler/frontend/hf_generic.py:602-663` (experts, top_k, expert_hidden).

`attn` picks the attention numerics:
- "norm": p = e*RECIP(red_sum(e)), pq = i8(127p), out = f32(pq.V)*a_v
  (`llm/ref_model.py:233-243`, `qhf.QModel.attention` :304-319);
- "qsum": eq = i8(127e), out = (f32(eq.V)*(RECIP(sum eq)*127))*a_v
  (`compiler/frontend/hf_generic.py:281-292`).
`rope` picks how the cos / sin tables are computed on the host: "llama2c"
(`llm/ref_model.py:34-41`, float32 powers, theta fixed in the reference, taken
from `theta` here) or "hf" (`compiler/frontend/qhf.py:183-189`, float64).
"""
from dataclasses import dataclass, replace


@dataclass(frozen=True)
class ModelConfig:
    name: str
    dim: int
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    seq_len: int
    theta: float = 10000.0
    eps: float = 1e-5
    tied: bool = True
    qk_norm: bool = False
    attn: str = "norm"
    rope: str = "llama2c"
    experts: int = 0
    top_k: int = 0
    expert_hidden: int = 0
    act: str = "silu"                  # the gated MLP's activation: "silu" or "gelu_tanh" (Gemma-class)

    @property
    def q_dim(self):
        return self.heads * self.head_dim

    @property
    def kv_dim(self):
        return self.kv_heads * self.head_dim

    @property
    def qkv_dim(self):
        return self.q_dim + 2 * self.kv_dim

    @property
    def group(self):
        return self.heads // self.kv_heads

    @property
    def moe(self):
        return self.experts > 0

    def with_(self, **kw):
        return replace(self, **kw)

    def validate(self):
        if self.heads % self.kv_heads:
            raise ValueError(f"{self.name}: heads {self.heads} not a multiple of kv_heads {self.kv_heads}")
        if self.head_dim % 8 or self.head_dim > 256:
            raise ValueError(f"{self.name}: head_dim {self.head_dim} must be a multiple of 8, at most 256")
        if self.dim % 16 or self.hidden % 16:
            raise ValueError(f"{self.name}: dim / hidden must be multiples of 16")
        if self.attn not in ("norm", "qsum") or self.rope not in ("llama2c", "hf"):
            raise ValueError(f"{self.name}: attn {self.attn!r} / rope {self.rope!r}")
        if self.moe and not (1 <= self.top_k <= self.experts <= 64 and self.expert_hidden % 16 == 0):
            raise ValueError(f"{self.name}: MoE experts {self.experts} top_k {self.top_k}")
        if self.act not in ("silu", "gelu_tanh") or (self.moe and self.act != "silu"):
            raise ValueError(f"{self.name}: activation {self.act!r} (MoE experts: silu)")
        return self


# BASELINE.json configs. Theta of C2 / C4 is not given there: the real
# checkpoints' value (1e6) is used and stated here.
C0 = ModelConfig("stories15M", dim=288, hidden=768, layers=6, heads=6, kv_heads=6, head_dim=48, vocab=32000,
                 seq_len=256, theta=10000.0, eps=1e-5, tied=True, attn="norm", rope="llama2c")
C1 = ModelConfig("SmolLM2-135M", dim=576, hidden=1536, layers=30, heads=9, kv_heads=3, head_dim=64, vocab=49152,
                 seq_len=2048, theta=1e5, eps=1e-5, tied=True, attn="qsum", rope="hf")
C2 = ModelConfig("Qwen3-0.6B", dim=1024, hidden=3072, layers=28, heads=16, kv_heads=8, head_dim=128, vocab=151936,
                 seq_len=2048, theta=1e6, eps=1e-6, tied=True, qk_norm=True, attn="qsum", rope="hf")
C3 = ModelConfig("Llama-3.2-1B", dim=2048, hidden=8192, layers=16, heads=32, kv_heads=8, head_dim=64, vocab=128256,
                 seq_len=2048, theta=5e5, eps=1e-5, tied=True, attn="qsum", rope="hf")
C4 = ModelConfig("Granite-3.1-1B-A400M", dim=1024, hidden=512, layers=24, heads=16, kv_heads=8, head_dim=64,
                 vocab=49155, seq_len=2048, theta=1e6, eps=1e-6, tied=True, attn="qsum", rope="hf",
                 experts=32, top_k=8, expert_hidden=512)
CONFIGS = {c.name: c for c in (C0, C1, C2, C3, C4)}


def tiny(seed_name="tiny", **kw):
    """A small model for tests (the shape of `llm/test_l4.tiny_model`, :41-55,
    with D = 16 head sizes)."""
    base = dict(name=seed_name, dim=64, hidden=128, layers=2, heads=4, kv_heads=2, head_dim=16, vocab=96,
                seq_len=48, theta=10000.0, eps=1e-5, tied=False, attn="norm", rope="llama2c")
    base.update(kw)
    return ModelConfig(**base).validate()
