"""Shape advisor: the largest standard dense GPT that a fleet of pipeline
stages trains with little waiting.

Reference behaviour (src/wantrain/scheduler/shape.py, SCHEDULER-I23):
compute per microbatch grows with d^2 x layers while the boundary a stage
sends grows with d alone, so on a slow hop small models wait; the advisor
recommends, among standard decoders (d a multiple of 128, 128-wide heads,
width/depth ratio d / n_layer inside [20, 200], the range in which Kaplan et
al. 2020 measured the loss within a few percent of optimal), the one with the
most parameters whose heaviest stage fits memory and whose priced bubble meets
a target, else the fitting one with the least bubble.

This advisor's own pricing and search:

* Cost model: this engine's. A block costs h(72h + 12s) FLOPs per token over
  its F, B and W passes (the partition model, scheduler/partition.py); the
  heaviest stage also holds the 6hV head. Memory: `bytes_per_param` of
  parameter state (16 with AdamW moments on the device, 10 with them in host
  memory) plus the saved activations of `in_flight` microbatches per block as
  the engine keeps them (scheduler/planner.py `act_bytes`).
* Link: the boundary a microbatch sends is seq x d elements of the boundary
  format (1 byte + one fp32 scale per 128 for fp8_e4m3_b128, 2 for bf16),
  divided by the codec's `wire_ratio`.
* Priced bubble: 1 - (1 - stall)(1 - fill), stall = max(0, 1 - compute /
  transfer) of the slowest hop, fill = (S - 1) / (M + S - 1).
* Search: for one width, more layers per stage only adds parameters and
  compute (the boundary does not grow), so the bubble never rises with depth;
  the best depth of a width is therefore the deepest that memory and the
  aspect range allow, found in closed form. `fits` lists that candidate for
  every width that has one, and the answer is chosen among them.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

VOCAB = 50257
BOUNDARY_BYTES = {"fp8_e4m3_b128": 1.0 + 4.0 / 128, "fp8_e5m2_b128": 1.0 + 4.0 / 128,
                  "fp16": 2.0, "bf16": 2.0, "fp32": 4.0}


@dataclass(frozen=True)
class Shape:
    d_model: int
    n_head: int
    layers_per_stage: int
    stages: int
    params: float
    compute_s: float  # one microbatch on the heaviest stage
    transfer_s: float  # one microbatch's boundary over the slowest hop
    bubble: float
    stage_bytes: float  # device memory of the heaviest stage

    @property
    def n_layer(self) -> int:
        return self.layers_per_stage * self.stages


def _block_flops_per_token(d: int, seq: int) -> float:
    return d * (72.0 * d + 12.0 * seq)


def _act_bytes_per_block(d: int, seq: int, mb_size: int) -> float:
    """Saved activations of one block for one microbatch (bf16), the engine's model."""
    from types import SimpleNamespace

    from elysium_wan_b200.scheduler.planner import act_bytes

    cfg = SimpleNamespace(seq_len=seq, d_model=d, ff=4 * d, n_head=max(1, d // 128),
                          boundary_dtype="bf16")
    m = act_bytes(cfg, mb_size, "cuda")
    return float(m["saved"] + m["w_keep"])


def price(d: int, layers_per_stage: int, stages: int, *, tflops: float, link_mbps: float,
          seq: int = 2048, mb_size: int = 1, microbatches: int = 64, bytes_per_param: float = 16.0,
          boundary: str = "bf16", wire_ratio: float = 1.0, in_flight: int | None = None) -> Shape:
    """Figures of one candidate. tflops: effective dense rate of a stage's
    GPU; link_mbps: the slowest hop's rate per direction (megabits/s, 0 =
    no limit)."""
    tokens = seq * mb_size
    stage_params = 12.0 * d * d * layers_per_stage + VOCAB * d
    flops = tokens * (_block_flops_per_token(d, seq) * layers_per_stage + 6.0 * d * VOCAB)
    compute = flops / (tflops * 1e12)
    sent = tokens * d * BOUNDARY_BYTES[boundary] / wire_ratio
    transfer = sent * 8.0 / (link_mbps * 1e6) if link_mbps > 0 else 0.0
    stall = max(0.0, 1.0 - compute / transfer) if transfer > 0 else 0.0
    fill = (stages - 1) / (microbatches + stages - 1)
    bubble = 1.0 - (1.0 - stall) * (1.0 - fill)
    live = stages if in_flight is None else in_flight
    stage_bytes = stage_params * bytes_per_param + \
        _act_bytes_per_block(d, seq, mb_size) * layers_per_stage * live
    params = 12.0 * d * d * layers_per_stage * stages + 2.0 * VOCAB * d
    return Shape(d_model=d, n_head=max(1, d // 128), layers_per_stage=layers_per_stage,
                 stages=stages, params=params, compute_s=compute, transfer_s=transfer,
                 bubble=bubble, stage_bytes=stage_bytes)


def deepest_fit(d: int, stages: int, memory_bytes: float, aspect=(20.0, 200.0),
                max_layers_per_stage: int = 256, **kw) -> Shape | None:
    """The deepest stage of width d that fits memory inside the aspect range
    (memory grows linearly with depth, so the bound is solved, not searched)."""
    lo = max(1, math.ceil(d / (aspect[1] * stages)))
    hi = min(max_layers_per_stage, math.floor(d / (aspect[0] * stages)))
    if hi < lo:
        return None
    one = price(d, 1, stages, **kw)
    two = price(d, 2, stages, **kw)
    per_layer = two.stage_bytes - one.stage_bytes
    base = one.stage_bytes - per_layer
    fit = math.floor((memory_bytes - base) / per_layer) if per_layer > 0 else hi
    L = min(hi, fit)
    return price(d, L, stages, **kw) if L >= lo else None


def advise(stages: int, memory_bytes: float, *, tflops: float, link_mbps: float,
           bubble_target: float = 0.2, d_choices: tuple = tuple(range(1024, 12288 + 1, 512)),
           aspect: tuple = (20.0, 200.0), **kw) -> dict:
    """{"best": Shape, "fits": [Shape per width], "met_target": bool}."""
    fits = [s for s in (deepest_fit(d, stages, memory_bytes, aspect, tflops=tflops,
                                    link_mbps=link_mbps, **kw) for d in d_choices) if s]
    if not fits:
        raise ValueError("no standard shape fits one stage's memory within the width/depth range")
    meets = [s for s in fits if s.bubble <= bubble_target]
    if meets:
        best = max(meets, key=lambda s: s.params)
    else:
        best = min(fits, key=lambda s: (s.bubble, -s.params))
    return {"best": best, "fits": fits, "met_target": bool(meets)}


def needed_mbps(d: int, layers_per_stage: int, *, tflops: float, seq: int = 2048,
                boundary: str = "bf16", wire_ratio: float = 1.0) -> float:
    """The hop rate at which a stage of this shape stops waiting (its
    boundary crosses the hop in its compute time)."""
    s = price(d, layers_per_stage, 2, tflops=tflops, link_mbps=0.0, seq=seq, boundary=boundary,
              wire_ratio=wire_ratio)
    sent = seq * d * BOUNDARY_BYTES[boundary] / wire_ratio
    return sent * 8.0 / s.compute_s / 1e6 if s.compute_s > 0 else math.inf
