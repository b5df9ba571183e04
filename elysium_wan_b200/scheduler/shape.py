"""Shape advisor: the largest standard dense GPT a fleet runs with a priced
bubble under a target.

Parity: src/wantrain/scheduler/shape.py (`Shape` :30, `price` :48, `advise`
:91, `needed_mbps` :114). A stage computes about 8 x its parameters FLOPs per
token (forward, recomputed forward, backward), growing with d^2 x layers; its
boundary moves seq x d values per microbatch, growing with d alone. The stage
stalls whenever moving a microbatch takes longer than computing it; the priced
bubble is that stall combined with the pipeline's fill and drain
(stages - 1) / (microbatches + stages - 1). Candidates keep the width/depth
ratio in [20, 200] (Kaplan et al. 2020 found the loss within a few percent of
optimal there), d a multiple of 128 and 128-wide heads, so every candidate is
a standard decoder trained exactly.

B200 terms: `wire_ratio` 1.0 (NVLink carries raw bf16; over a WAN hop with
the planes codec pass the measured ratio), bytes per parameter 16 (fp32
master, gradient and device AdamW moments; 8 with adamw-host), activation
charge from this engine's saved-tensor model.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

VOCAB = 50257


@dataclass(frozen=True)
class Shape:
    d_model: int
    n_head: int
    layers_per_stage: int
    stages: int
    params: float
    compute_s: float
    transfer_s: float
    bubble: float
    stage_bytes: float

    @property
    def n_layer(self) -> int:
        return self.layers_per_stage * self.stages


def price(d: int, layers_per_stage: int, stages: int, *, tflops: float, link_mbps: float,
          seq: int = 2048, microbatches: int = 64, bytes_per_param: float = 16.0,
          wire_ratio: float = 1.0, act_bytes_per_layer_token: float | None = None,
          pending: int | None = None) -> Shape:
    """One candidate. tflops: the effective dense bf16 rate of a stage's GPU;
    link_mbps: the slowest hop's per-direction rate (megabits/s)."""
    per_layer = 12 * d * d
    stage_params = per_layer * layers_per_stage + VOCAB * d  # the heavy stage holds a table
    compute = 8.0 * stage_params * seq / (tflops * 1e12)
    transfer = seq * d * 2 * wire_ratio * 8 / (link_mbps * 1e6) if link_mbps > 0 else 0.0
    stall = 1.0 - compute / max(compute, transfer) if compute > 0 else 1.0
    fill = (stages - 1) / (microbatches + stages - 1)
    bubble = 1.0 - (1.0 - stall) * (1.0 - fill)
    # Saved bf16 activations per block per token (LN outs, qkv, attention out,
    # proj residual, fc1 pre/post GELU): about 14 d values at 2 bytes.
    act = act_bytes_per_layer_token if act_bytes_per_layer_token is not None else 28.0 * d
    live = stages if pending is None else pending + 1
    stage_bytes = stage_params * bytes_per_param + act * seq * layers_per_stage * live
    total = per_layer * layers_per_stage * stages + 2 * VOCAB * d
    return Shape(d_model=d, n_head=max(1, d // 128), layers_per_stage=layers_per_stage,
                 stages=stages, params=float(total), compute_s=compute, transfer_s=transfer,
                 bubble=bubble, stage_bytes=stage_bytes)


def advise(stages: int, memory_bytes: float, *, tflops: float, link_mbps: float,
           bubble_target: float = 0.2, d_choices: tuple = tuple(range(1024, 12288 + 1, 512)),
           max_layers_per_stage: int = 128, aspect: tuple = (20.0, 200.0), **kw) -> dict:
    """{"best": Shape, "fits": [...], "met_target": bool}: the shape with the
    most parameters whose heaviest stage fits `memory_bytes` with a priced
    bubble at most `bubble_target`, else the fitting shape with the least
    bubble."""
    fits = []
    for d in d_choices:
        for lps in range(1, max_layers_per_stage + 1):
            s = price(d, lps, stages, tflops=tflops, link_mbps=link_mbps, **kw)
            if s.stage_bytes > memory_bytes:
                break
            if aspect[0] <= d / s.n_layer <= aspect[1]:
                fits.append(s)
    if not fits:
        raise ValueError("no standard shape fits one stage's memory within the width/depth range")
    ok = [s for s in fits if s.bubble <= bubble_target]
    best = max(ok, key=lambda s: s.params) if ok else min(fits, key=lambda s: (s.bubble, -s.params))
    return {"best": best, "fits": fits, "met_target": bool(ok)}


def needed_mbps(d: int, layers_per_stage: int, *, tflops: float, seq: int = 2048,
                wire_ratio: float = 1.0) -> float:
    """The hop rate at which this stage stops waiting: one microbatch's
    boundary crosses in one microbatch's compute time."""
    s = price(d, layers_per_stage, 2, tflops=tflops, link_mbps=1e12, seq=seq, wire_ratio=wire_ratio)
    return seq * d * 2 * wire_ratio * 8 / s.compute_s / 1e6 if s.compute_s > 0 else math.inf
