"""Per-step telemetry summary (reference: src/wantrain/runtime/telemetry.py:38-98).

WT_TELEM {v, step, rank, peer, step_ms, ops{F,B,W:{n, med_ms}}, busy_ms,
busy_frac, hops{frames, bytes}} capped at 4096 bytes. Op durations are CUDA
event times on the compute stream; busy = union of op intervals.
"""

from __future__ import annotations

import json
import os
import statistics


def summarize_step(step, stage, peer, step_ms, op_times, bytes_sent, frames) -> dict:
    ops = {}
    for op in ("F", "B", "W"):
        ds = [d for o, _, _, d in op_times if o == op]
        if ds:
            ops[op] = {"n": len(ds), "med_ms": round(statistics.median(ds), 4)}
    busy = 0.0
    end = -1.0
    for _, _, s, d in sorted(op_times, key=lambda x: x[2]):
        e = s + d
        if s >= end:
            busy += d
        elif e > end:
            busy += e - end
        end = max(end, e)
    span = (max(s + d for _, _, s, d in op_times) - min(s for _, _, s, _ in op_times)) if op_times else 0.0
    out = {"v": 1, "step": step, "rank": stage, "peer": peer, "step_ms": round(step_ms, 3),
           "ops": ops, "busy_ms": round(busy, 3),
           "busy_frac": round(busy / span, 4) if span > 0 else None,
           "hops": {"frames": frames, "bytes": bytes_sent}}
    s = json.dumps(out)
    if len(s) > 4096:
        out.pop("ops")
    return out


def parse_sim_slow(value: str | None = None) -> dict:
    """WANTRAIN_SIM_SLOW="stage:factor[@from_step],...": a timing-only seam
    (moves when, never what): the stage's ops take `factor` x their time from
    `from_step` on (default 0). -> {stage: (factor, from_step)}."""
    value = value if value is not None else os.environ.get("WANTRAIN_SIM_SLOW", "")
    out = {}
    for part in filter(None, value.split(",")):
        k, _, v = part.partition(":")
        f, _, s = v.partition("@")
        out[int(k)] = (float(f), int(s) if s else 0)
    return out
