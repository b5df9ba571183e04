"""GPT configuration, presets and precision recipes.

Field names follow the reference's GPTConfig (src/wantrain/model/gpt.py:47-253)
so a job JSON written for wantrain loads unchanged. The block is the reference's
generalized decoder (src/wantrain/model/arch.py): norm layernorm | rmsnorm,
mlp gelu | swiglu, pos learned | rope, grouped-query attention (n_kv_head),
bias on/off, tied embeddings, and the exact MoE block (moe_* fields). User
models (arch "user": the operator's own flat layer list, models/user.py) run
on the host path. Arch "hf" (transformers module trees) is accepted in the
JSON and refused with a clear message at build time.
"""

from __future__ import annotations

import dataclasses
import math
from dataclasses import dataclass, field

# Precision recipes (reference: src/wantrain/model/precision.py:18-162; the
# table with classification and capability gates is models/precision.py).
COMPUTE_DTYPES = ("fp32", "bf16")
BOUNDARY_DTYPES = ("fp32", "bf16", "fp16", "fp8_e5m2_b128", "fp8_e4m3_b128")
RECIPE_BYTES = {"fp32": 4, "bf16": 2, "fp16": 2, "fp8_e5m2_b128": 1, "fp8_e4m3_b128": 1}
# The reference's fp8 boundary names scale per token; this engine scales the
# same formats per 1x128 block of a row (a finer scale, the layout the fused
# GEMM epilogue writes), and reads the reference's names as these.
BOUNDARY_ALIASES = {"fp8_e4m3": "fp8_e4m3_b128", "fp8_e5m2": "fp8_e5m2_b128"}


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
    rope_theta: float = 10000.0
    rms_eps: float = 1e-6
    lora_rank: int = 0
    lora_alpha: float = 16.0
    lora_targets: str = "attn"  # attn | attn_mlp | all
    # Mixture of experts (reference arch.py:279-763); 0 experts = dense.
    moe_experts: int = 0
    moe_top_k: int = 1
    moe_d_ff: int | None = None
    moe_shared_d_ff: int = 0
    moe_shared_gate: str = "sigmoid"  # sigmoid | none
    # arch "user": a Python file defining build(cfg) -> n_layer + 2 modules
    # (token ids -> ... -> logits), pinned by its sha256
    user_model: str = ""
    user_model_sha256: str = ""
    moe_layers: list | None = None  # 0-based block indices; None = every block
    moe_router_dtype: str = "compute"  # compute | fp32
    moe_router_bias: bool = False
    moe_score: str = "softmax"  # softmax | softmax_k | sigmoid
    moe_select: str = "score"  # score | logit | score_bias
    moe_groups: int = 1
    moe_topk_groups: int = 1
    moe_norm: bool = False
    moe_norm_eps: float = 0.0
    moe_scale: float = 1.0
    moe_apply: str = "output"  # output | input (k = 1)
    moe_expert: str = "swiglu"  # swiglu | swiglu_clamped
    moe_limit: float = 7.0
    moe_alpha: float = 1.702
    moe_lbl_coef: float = 0.0
    moe_lbl_scope: str = "layer"  # layer | sequence
    moe_z_coef: float = 0.0
    moe_bias_rate: float = 0.0
    extras: dict = field(default_factory=dict)

    @property
    def ff(self) -> int:
        """MLP width: 4 d for GELU, 8/3 d rounded up to a multiple of 256 for
        SwiGLU (three matrices at about the parameter count of two)."""
        if self.d_ff:
            return self.d_ff
        if self.mlp == "gelu":
            return 4 * self.d_model
        return int(math.ceil(8 * self.d_model / 3 / 256) * 256)

    @property
    def kv_heads(self) -> int:
        return self.n_kv_head or self.n_head

    @property
    def qkv_width(self) -> int:
        """Columns of the fused projection: q (n_head) + k, v (kv_heads)."""
        return self.d_model + 2 * self.kv_heads * self.head_dim

    @property
    def norm_eps(self) -> float:
        return self.ln_eps if self.norm == "layernorm" else self.rms_eps

    @property
    def moe_width(self) -> int:
        return self.moe_d_ff or self.d_ff or int(math.ceil(8 * self.d_model / 3 / 256) * 256)

    def is_moe_layer(self, entry: int) -> bool:
        """Flat-list entry `entry` (block i is entry i + 1) is an MoE block."""
        if self.moe_experts <= 0 or entry < 1 or entry > self.n_layer:
            return False
        return self.moe_layers is None or (entry - 1) in self.moe_layers

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_head

    @property
    def n_entries(self) -> int:
        """Length of the flat layer list [Embed, Block x n_layer, Head]."""
        return self.n_layer + 2

    def fp8_boundary(self) -> bool:
        return self.boundary_dtype in ("fp8_e4m3_b128", "fp8_e5m2_b128")

    def validate(self) -> "GPTConfig":
        self.boundary_dtype = BOUNDARY_ALIASES.get(self.boundary_dtype, self.boundary_dtype)
        if self.compute_dtype not in COMPUTE_DTYPES:
            raise ValueError(f"compute_dtype {self.compute_dtype!r} not in {COMPUTE_DTYPES}")
        if self.boundary_dtype not in BOUNDARY_DTYPES:
            raise ValueError(f"boundary_dtype {self.boundary_dtype!r} not in {BOUNDARY_DTYPES}")
        if self.d_model % self.n_head:
            raise ValueError("d_model must be divisible by n_head")
        if self.arch == "user":
            if not self.user_model:
                raise ValueError("arch 'user' needs user_model (a Python file defining build(cfg))")
            if self.compute_dtype != "fp32" or self.boundary_dtype != "fp32":
                raise ValueError("user models run in fp32 with fp32 boundaries (the host path)")
            if self.lora_rank or self.moe_experts or self.tie_embeddings:
                raise ValueError("LoRA, MoE and tied embeddings are built-in decoder knobs")
        elif self.arch != "builtin":
            raise NotImplementedError(
                f"arch {self.arch!r}: this engine builds the built-in decoder family and user "
                f"models (arch 'user'); HF module trees are not built")
        for name, allowed in (("norm", ("layernorm", "rmsnorm")), ("mlp", ("gelu", "swiglu")),
                              ("pos", ("learned", "rope")),
                              ("lora_targets", ("attn", "attn_mlp", "all"))):
            if getattr(self, name) not in allowed:
                raise ValueError(f"{name}={getattr(self, name)!r} is not one of {allowed}")
        if self.n_kv_head is not None and (self.n_kv_head < 1 or self.n_head % self.n_kv_head):
            raise ValueError("n_head must be a multiple of n_kv_head")
        if self.pos == "rope" and self.head_dim % 2:
            raise ValueError("rope needs an even head_dim")
        if self.tie_embeddings and self.init_scheme != "gpt2":
            raise ValueError("tie_embeddings requires init_scheme='gpt2' (one scale for both uses)")
        if self.lora_rank < 0:
            raise ValueError("lora_rank must be >= 0")
        if self.fp8_boundary() and self.d_model % 128:
            raise ValueError(f"{self.boundary_dtype} boundaries need d_model % 128 == 0")
        check_moe(self)
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
        b = 1 if self.bias else 0
        nrm = d * (2 if self.norm == "layernorm" else 1)
        attn = self.qkv_width * d + b * self.qkv_width + d * d + b * d
        mats = 3 if self.mlp == "swiglu" else 2
        dense_mlp = mats * d * f + b * ((mats - 1) * f + d)
        E = self.moe_experts
        moe_mlp = (d * E + (E if self.moe_router_bias else 0)
                   + E * 3 * d * self.moe_width
                   + (3 * d * self.moe_shared_d_ff if self.moe_shared_d_ff else 0)
                   + (d if self.moe_shared_d_ff and self.moe_shared_gate == "sigmoid" else 0))
        total = V * d + (S * d if self.pos == "learned" else 0) + nrm
        for e in range(1, self.n_layer + 1):
            total += 2 * nrm + attn + (moe_mlp if self.is_moe_layer(e) else dense_mlp)
        return total + (0 if self.tie_embeddings else V * d)


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
    # Llama-style decoders (RMSNorm, SwiGLU, RoPE, GQA, no bias).
    "llama_tiny": dict(vocab_size=512, n_layer=4, n_head=4, n_kv_head=2, d_model=256, seq_len=128,
                       norm="rmsnorm", mlp="swiglu", pos="rope", bias=False, init_scheme="gpt2"),
    "llama1b": dict(vocab_size=32768, n_layer=16, n_head=32, n_kv_head=8, d_model=2048,
                    seq_len=2048, norm="rmsnorm", mlp="swiglu", pos="rope", bias=False,
                    rope_theta=500000.0, init_scheme="gpt2", compute_dtype="bf16",
                    boundary_dtype="bf16"),
    "llama8b": dict(vocab_size=128256, n_layer=32, n_head=32, n_kv_head=8, d_model=4096,
                    d_ff=14336, seq_len=2048, norm="rmsnorm", mlp="swiglu", pos="rope",
                    bias=False, rope_theta=500000.0, init_scheme="gpt2", compute_dtype="bf16",
                    boundary_dtype="bf16"),
    # A small mixture-of-experts decoder (8 experts, top-2, shared expert).
    "moe_tiny": dict(vocab_size=512, n_layer=4, n_head=4, n_kv_head=2, d_model=256, seq_len=128,
                     norm="rmsnorm", mlp="swiglu", pos="rope", bias=False, init_scheme="gpt2",
                     moe_experts=8, moe_top_k=2, moe_d_ff=256, moe_shared_d_ff=256,
                     moe_lbl_coef=0.01, moe_z_coef=0.001),
}


def check_moe(cfg) -> None:
    """The MoE construction rules (reference arch.py:338-391); each refusal
    names the field."""
    E, k = cfg.moe_experts, cfg.moe_top_k
    if E < 0:
        raise ValueError(f"moe_experts={E} must be >= 0")
    if E == 0:
        return
    if not 1 <= k <= E:
        raise ValueError(f"moe_top_k={k} must satisfy 1 <= moe_top_k <= moe_experts={E}")
    for name, allowed in (("moe_router_dtype", ("compute", "fp32")),
                          ("moe_score", ("softmax", "softmax_k", "sigmoid")),
                          ("moe_select", ("score", "logit", "score_bias")),
                          ("moe_shared_gate", ("sigmoid", "none")),
                          ("moe_apply", ("output", "input")),
                          ("moe_expert", ("swiglu", "swiglu_clamped")),
                          ("moe_lbl_scope", ("layer", "sequence"))):
        if getattr(cfg, name) not in allowed:
            raise ValueError(f"{name}={getattr(cfg, name)!r} is not one of {allowed}")
    if cfg.moe_apply == "input" and k != 1:
        raise ValueError(f"moe_apply='input' requires moe_top_k=1, got moe_top_k={k}")
    G, Gt = cfg.moe_groups, cfg.moe_topk_groups
    if G < 1:
        raise ValueError(f"moe_groups={G} must be >= 1")
    if G > 1:
        if E % G:
            raise ValueError(f"moe_groups={G} must divide moe_experts={E}")
        if E // G < 2:
            raise ValueError(f"moe_groups={G}: moe_experts/moe_groups={E // G} must be >= 2")
        if not 1 <= Gt <= G:
            raise ValueError(f"moe_topk_groups={Gt} must satisfy 1 <= moe_topk_groups <= {G}")
        if k > Gt * (E // G):
            raise ValueError(f"moe_top_k={k} exceeds moe_topk_groups*moe_experts/moe_groups="
                             f"{Gt * (E // G)}")
    elif Gt != 1:
        raise ValueError(f"moe_topk_groups={Gt} requires moe_groups > 1")
    if cfg.moe_d_ff is not None and cfg.moe_d_ff < 1:
        raise ValueError(f"moe_d_ff={cfg.moe_d_ff} must be >= 1")
    if cfg.moe_shared_d_ff < 0:
        raise ValueError(f"moe_shared_d_ff={cfg.moe_shared_d_ff} must be >= 0")
    if cfg.moe_bias_rate < 0:
        raise ValueError(f"moe_bias_rate={cfg.moe_bias_rate} must be >= 0")
    if cfg.moe_lbl_coef < 0 or cfg.moe_z_coef < 0:
        raise ValueError("moe_lbl_coef and moe_z_coef must be >= 0")


def make_config(preset: str, **overrides) -> GPTConfig:
    if preset not in PRESETS:
        raise KeyError(f"unknown preset {preset!r}; known: {sorted(PRESETS)}")
    d = dict(PRESETS[preset])
    d.update(overrides)
    return GPTConfig(**d).validate()
