"""Precision recipes as data: the number formats a run computes in and sends
across entry boundaries, what each pair of them claims, and where each runs.

Reference behaviour (src/wantrain/model/precision.py:18-162, semantics only):
precision is part of the recipe, never of the transport; a boundary format
is "native" when the wire carries the compute tensor's whole information and
"wire-quantized" otherwise; each rung has a wire size, a scale requirement
and a minimum device capability; a planner walks the rungs widest first.

This engine's own model of it:

* A format is described by its bit fields (exponent and mantissa bits), its
  storage size and whether it carries a block scale. The fp8 rungs scale one
  power of two per 1x128 block of a row (e4m3: 2^(e-8), e5m2: 2^(e-15) for
  amax = f 2^e), the layout the fused GEMM epilogue writes; their wire cost
  is one byte plus 4/128 bytes of scale per value.
* "native" is decided by representability, not by width: a boundary is
  native for a compute dtype when every finite compute value is exactly a
  boundary value, i.e. at least as many exponent and mantissa bits and no
  shared scale. So fp32 and bf16 are native for bf16 compute while fp16 is
  not (its 5-bit exponent cannot hold bf16's range below 2^-24 or above
  65504), which is stricter than a width comparison.
* Capability: compute runs on this engine's tcgen05 kernels (sm_100a) in
  bf16, or on the host path in fp32. fp16 compute is not built: on B200 bf16
  runs at the fp16 tensor rate with fp32's exponent range, and fp16 compute
  would also need a loss scale. Every boundary format runs wherever its
  compute dtype does (the casts are fused into the GEMM epilogues, the
  LayerNorm prologue and the embedding).
"""

from __future__ import annotations

from dataclasses import dataclass

from elysium_wan_b200.models.config import BOUNDARY_ALIASES


@dataclass(frozen=True)
class Format:
    name: str
    storage_bits: int
    exp_bits: int
    man_bits: int
    block_scale: bool  # one fp32 power-of-two scale per 128 values of a row
    max_finite: float
    min_normal: float

    @property
    def wire_bytes(self) -> float:
        """Bytes per value on the wire before any codec."""
        return self.storage_bits / 8 + (4.0 / 128 if self.block_scale else 0.0)

    @property
    def needs_scale(self) -> bool:
        """Whether activation gradients / activations underflow without a scale."""
        return self.block_scale


FORMATS = {
    "fp32": Format("fp32", 32, 8, 23, False, 3.4028234663852886e38, 1.1754943508222875e-38),
    "bf16": Format("bf16", 16, 8, 7, False, 3.3895313892515355e38, 1.1754943508222875e-38),
    "fp16": Format("fp16", 16, 5, 10, False, 65504.0, 6.103515625e-05),
    "fp8_e5m2_b128": Format("fp8_e5m2_b128", 8, 5, 2, True, 57344.0, 6.103515625e-05),
    "fp8_e4m3_b128": Format("fp8_e4m3_b128", 8, 4, 3, True, 448.0, 0.015625),
}

# Boundary rungs, widest first (the admission ladder). Among rungs of one
# size the one with more mantissa bits comes first: with a scale per 128
# values, range is the scale's job, so e4m3 carries more of each value than
# e5m2 (fp16 follows bf16 because only bf16 holds every bf16 value).
LADDER = ["fp32", "bf16", "fp16", "fp8_e4m3_b128", "fp8_e5m2_b128"]

NATIVE, WIRE_QUANTIZED = "native", "wire-quantized"

# Where a compute dtype runs: (minimum CUDA capability of this engine's
# kernels, or None for the host path only). fp16 compute is not built.
COMPUTE_PATHS = {"bf16": (10, 0), "fp32": None}


def fmt(name: str) -> Format:
    name = BOUNDARY_ALIASES.get(name, name)
    if name not in FORMATS:
        raise ValueError(f"unknown precision {name!r}; choose from {sorted(FORMATS)}")
    return FORMATS[name]


def represents(boundary: str, compute: str) -> bool:
    """Every finite value of `compute` is exactly a value of `boundary`."""
    b, c = fmt(boundary), fmt(compute)
    return not b.block_scale and b.exp_bits >= c.exp_bits and b.man_bits >= c.man_bits


def classify(compute: str, boundary: str) -> dict:
    """The claim a (compute, boundary) pair earns."""
    b, c = fmt(boundary), fmt(compute)
    if represents(boundary, compute):
        return dict(level=NATIVE, lossless_vs_reference=True,
                    claim=f"boundary {b.name} holds every {c.name} value exactly: the run is "
                          f"lossless against the single-device {c.name} recipe")
    why = []
    if b.exp_bits < c.exp_bits:
        why.append(f"{b.exp_bits}-bit exponent vs {c.exp_bits}")
    if b.man_bits < c.man_bits:
        why.append(f"{b.man_bits} mantissa bits vs {c.man_bits}")
    if b.block_scale:
        why.append("one shared scale per 128 values")
    return dict(level=WIRE_QUANTIZED, lossless_vs_reference=False,
                claim=f"boundary {b.name} narrows {c.name} ({', '.join(why)}; "
                      f"{c.storage_bits // 8} -> {b.wire_bytes:g} bytes per value): the run is "
                      f"bit-reproducible and the oracle applies the same narrowing at the same "
                      f"points, but it is not lossless against the {c.name} recipe")


def compute_runnable(name: str, cap) -> bool:
    """Can a device of compute capability `cap` ((major, minor); None for the
    host / unknown) run block math in `name` on this engine?"""
    if name not in COMPUTE_PATHS:
        return False
    need = COMPUTE_PATHS[name]
    if need is None:  # host path
        return True
    return cap is None or tuple(cap) >= need


def describe(compute: str, boundary: str, d_model: int, wire_ratio: float = 1.0) -> dict:
    """The recipe's fingerprint: what was chosen and what it costs per token."""
    b = fmt(boundary)
    raw = b.wire_bytes * d_model
    return dict(compute=compute, boundary=b.name, bytes_per_value=b.wire_bytes,
                wire_bytes_per_token_raw=raw,
                wire_bytes_per_token_coded=round(raw / max(1e-9, wire_ratio), 1),
                needs_scale=b.needs_scale, **classify(compute, b.name))
