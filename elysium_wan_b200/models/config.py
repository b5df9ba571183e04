"""GPT configuration, presets and precision recipes.

Field names follow the reference's GPTConfig (src/wantrain/model/gpt.py:47-253)
so a job JSON written for wantrain loads unchanged; knobs of the reference that
this engine does not build (hf / user archs, MoE, LoRA) are accepted in the
JSON and refused with a clear message at build time.
"""

from __future__ import annotations

import dataclasses
from dataclasses import dataclass, field

# Precision recipes (reference: src/wantrain/model/precision.py:18-162).
COMPUTE_DTYPES = ("fp32", "bf16")
BOUNDARY_DTYPES = ("fp32", "bf16", "fp8_e4m3_b128")
RECIPE_BYTES = {"fp32": 4, "bf16": 2, "fp8_e4m3_b128": 1}


@dataclass
class GPTConfig:
    vocab_size: int = 256
    n_layer: int = 6
    n_head: int = 4
    d_model: int = 128
    seq_len: int = 64
    # compute_dtype: what the block math runs in (bf16 on the GPU kernels, fp32
    # on the CPU plumbing path). boundary_dtype: what crosses every block
    # boundary (and so every stage cut). fp8_e4m3_b128 = e4m3 with one
    # power-of-two scale per 128 elements of a row; gradients stay bf16.
    compute_dtype: str = "fp32"
    boundary_dtype: str = "fp32"
    attn_impl: str = "sdpa"  # naive | sdpa: both map to the same causal kernel here
    sdpa_backend: str = "auto"
    arch: str = "builtin"
    d_ff: int | None = None
    norm: str = "layernorm"
    mlp: str = "gelu"
    pos: str = "learned"
    bias: bool = True
    tie_embeddings: bool = False
    init_scheme: str = "gpt2"  # gpt2 | torch_default
    init_std: float = 0.02
    ln_eps: float = 1e-5
    n_kv_head: int | None = None
    lora_rank: int = 0
    moe_experts: int = 0
    extras: dict = field(default_factory=dict)

    @property
    def ff(self) -> int:
        return self.d_ff or 4 * self.d_model

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_head

    @property
    def n_entries(self) -> int:
        """Length of the flat layer list [Embed, Block x n_layer, Head]."""
        return self.n_layer + 2

    def fp8_boundary(self) -> bool:
        return self.boundary_dtype == "fp8_e4m3_b128"

    def validate(self) -> "GPTConfig":
        if self.compute_dtype not in COMPUTE_DTYPES:
            raise ValueError(f"compute_dtype {self.compute_dtype!r} not in {COMPUTE_DTYPES}")
        if self.boundary_dtype not in BOUNDARY_DTYPES:
            raise ValueError(f"boundary_dtype {self.boundary_dtype!r} not in {BOUNDARY_DTYPES}")
        if self.d_model % self.n_head:
            raise ValueError("d_model must be divisible by n_head")
        if self.arch != "builtin":
            raise NotImplementedError(
                f"arch {self.arch!r}: only the built-in dense GPT is implemented in this engine")
        if self.moe_experts or self.lora_rank:
            raise NotImplementedError("MoE and LoRA are not implemented in this engine")
        if (self.norm, self.mlp, self.pos, self.tie_embeddings) != ("layernorm", "gelu", "learned", False):
            raise NotImplementedError("only LayerNorm / GELU / learned positions / untied head")
        if self.n_kv_head not in (None, self.n_head):
            raise NotImplementedError("GQA is not implemented")
        if self.fp8_boundary() and self.d_model % 128:
            raise ValueError("fp8_e4m3_b128 boundaries need d_model % 128 == 0")
        return self

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)

    @classmethod
    def from_dict(cls, d: dict) -> "GPTConfig":
        known = {f.name for f in dataclasses.fields(cls)}
        kw = {k: v for k, v in d.items() if k in known}
        extras = {k: v for k, v in d.items() if k not in known}
        cfg = cls(**kw)
        cfg.extras.update(extras)
        return cfg

    def n_params(self) -> int:
        d, V, S, f = self.d_model, self.vocab_size, self.seq_len, self.ff
        block = 4 * d + 3 * d * d + 3 * d + d * d + d + d * f + f + f * d + d
        return V * d + S * d + self.n_layer * block + 2 * d + V * d


# Reference presets (gpt.py:258-268) plus the BASELINE shapes.
PRESETS: dict[str, dict] = {
    "toy": dict(),
    "gpt124m": dict(vocab_size=32768, n_layer=12, n_head=12, d_model=768, seq_len=512),
    "gpt350m": dict(vocab_size=32768, n_layer=24, n_head=16, d_model=1024, seq_len=512),
    "gpt760m": dict(vocab_size=32768, n_layer=24, n_head=16, d_model=1536, seq_len=512),
    "gpt1_5b": dict(vocab_size=32768, n_layer=48, n_head=25, d_model=1600, seq_len=512),
    "gpt4_4b": dict(vocab_size=32768, n_layer=34, n_head=25, d_model=3200, seq_len=1024),
    # CPU/gloo plumbing run.
    "cpu_plumbing": dict(vocab_size=50257, n_layer=8, n_head=4, d_model=256, seq_len=128),
    # BASELINE configs 2-5 (bf16 on the GPU).
    "gpt0_6b": dict(vocab_size=50257, n_layer=20, n_head=12, d_model=1536, seq_len=2048,
                    compute_dtype="bf16", boundary_dtype="bf16"),
    "gpt2_8b": dict(vocab_size=50257, n_layer=32, n_head=32, d_model=2560, seq_len=2048,
                    compute_dtype="bf16", boundary_dtype="bf16"),
    "gpt15b": dict(vocab_size=50257, n_layer=48, n_head=40, d_model=5120, seq_len=2048,
                   compute_dtype="bf16", boundary_dtype="fp8_e4m3_b128"),
    "gpt25b": dict(vocab_size=50257, n_layer=60, n_head=46, d_model=5888, d_ff=23552,
                   seq_len=2048, compute_dtype="bf16", boundary_dtype="fp8_e4m3_b128"),
}


def make_config(preset: str, **overrides) -> GPTConfig:
    if preset not in PRESETS:
        raise KeyError(f"unknown preset {preset!r}; known: {sorted(PRESETS)}")
    d = dict(PRESETS[preset])
    d.update(overrides)
    return GPTConfig(**d).validate()
