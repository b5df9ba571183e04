"""Production defaults every planned spec starts from; explicit overrides win
and are listed as deviations in the run log.

Parity: src/wantrain/scheduler/production.py:14-49 (`PRODUCTION`,
`spec_fields`, `deviations`). The reference's defaults serve a TCP data plane
(lossless planes codec, 8 parallel flows); on one B200 box the boundary moves
over NVLink through NCCL, where a codec costs time and a flow count means
nothing, so the defaults here are the GPU ones: recompute on (it re-runs the
same kernels on the same inputs, so the bits do not change), raw wire, one
stream, the fused ZeRO-1 gradient path, and the NCCL backend.
"""

from __future__ import annotations

PRODUCTION = dict(recompute=True, wire_codec="raw", p2p_streams=1, backend="nccl")

# Applied when any stage is wider than one replica.
PRODUCTION_WIDE = dict(grad_sync="fused", shard="zero1")

# The CPU / WAN path (gloo or tcp backend): a lossless codec pays for itself
# on a slow hop.
PRODUCTION_WAN = dict(recompute=True, wire_codec="planes", p2p_streams=8)


def spec_fields(stage_widths=None, overrides: dict | None = None, wan: bool = False) -> dict:
    """Production JobSpec fields with operator overrides layered on top (an
    override of None means 'keep the default')."""
    out = dict(PRODUCTION_WAN if wan else PRODUCTION)
    if stage_widths and any(w > 1 for w in stage_widths):
        out.update(PRODUCTION_WIDE)
    for k, v in (overrides or {}).items():
        if v is not None:
            out[k] = v
    return out


def deviations(fields: dict, wan: bool = False) -> list:
    """The production flags a spec turned off, one line each, for the run log."""
    base = PRODUCTION_WAN if wan else PRODUCTION
    return [f"{k}={fields[k]!r} (production: {v!r})" for k, v in base.items()
            if k in fields and fields[k] != v]
