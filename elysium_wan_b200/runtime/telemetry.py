"""Per-step telemetry summary (reference: src/wantrain/runtime/telemetry.py:38-98).

WT_TELEM {v, step, rank, peer, step_ms, emit_us, ops{F,B,W[,OPT]:{n, med_ms}},
stall_ms, busy_ms, busy_frac, hops{frames, bytes}, recv{n, med_ms, max_ms}}
capped at 4096 bytes (the reference's keys; busy_ms / busy_frac are added).
Op durations are CUDA-event times (host clock on a CPU stage); W on a GPU
stage is bracketed on the side stream that runs it. busy = union of the op
intervals; stall_ms = the part of the ops' span with no op running; recv =
the gaps before F and B ops (each starts once its input has arrived).
"""

from __future__ import annotations

import json
import math
import os
import statistics


def summarize_step(step, stage, peer, step_ms, op_times, bytes_sent, frames,
                   opt_ms: float | None = None, links: dict | None = None) -> dict:
    """The per-step WT_TELEM summary. `links`: this step's per-link send
    statistics ({label: {"frames", "bytes", "busy_ms"}}, the TCP plane's),
    filed under "hops" next to the step's totals."""
    import time as _time

    t_emit = _time.perf_counter()
    ops = {}
    for op in ("F", "B", "W"):
        ds = [d for o, _, _, d in op_times if o == op]
        if ds:
            ops[op] = {"n": len(ds), "med_ms": round(statistics.median(ds), 4)}
    if opt_ms is not None:
        ops["OPT"] = {"n": 1, "med_ms": round(float(opt_ms), 4)}
    # waits for inputs: the gap before each F / B since the previous op ended
    gaps, last_end = [], None
    for o, _, s0, d in sorted(op_times, key=lambda x: x[2]):
        if last_end is not None and o in ("F", "B") and s0 > last_end:
            gaps.append(s0 - last_end)
        last_end = s0 + d if last_end is None else max(last_end, s0 + d)
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
           "emit_us": 0, "ops": ops, "stall_ms": round(max(0.0, span - busy), 3),
           "busy_ms": round(busy, 3),
           "busy_frac": round(busy / span, 4) if span > 0 else None,
           "hops": {"frames": frames, "bytes": bytes_sent, **(links or {})},
           "recv": {"n": len(gaps), "med_ms": round(statistics.median(gaps), 4) if gaps else 0.0,
                    "max_ms": round(max(gaps), 4) if gaps else 0.0}}
    out["emit_us"] = int((_time.perf_counter() - t_emit) * 1e6)
    s = json.dumps(out)
    if len(s) > 4096:
        out.pop("ops")
    return out


def parse_sim_slow(value: str | None = None) -> dict:
    """WANTRAIN_SIM_SLOW, a timing-only seam (moves when, never what): the
    named stage's ops take `factor` x their time from `from_step` on (default
    0). Comma-separated parts, each either "stage:factor[@from_step]" (every
    peer of the stage) or the reference's one-slot form
    "rank:peer:factor[:from_step]" (src/wantrain/runtime/telemetry.py:81).
    -> {stage or (stage, peer): (factor, from_step)}."""
    value = value if value is not None else os.environ.get("WANTRAIN_SIM_SLOW", "")
    out = {}
    for part in filter(None, value.split(",")):
        f = part.split(":")
        try:
            if len(f) == 2:
                fac, _, st = f[1].partition("@")
                key, factor, start = int(f[0]), float(fac), int(st) if st else 0
            elif len(f) in (3, 4):
                key, factor = (int(f[0]), int(f[1])), float(f[2])
                start = int(f[3]) if len(f) == 4 else 0
            else:
                raise ValueError
        except ValueError:
            raise ValueError(f"WANTRAIN_SIM_SLOW={value!r}: expected stage:factor[@from_step] "
                             "or rank:peer:factor[:from_step]") from None
        if not (math.isfinite(factor) and factor >= 1.0) or start < 0:
            raise ValueError(f"WANTRAIN_SIM_SLOW={value!r}: a finite factor >= 1, from_step >= 0")
        out[key] = (factor, start)
    return out
