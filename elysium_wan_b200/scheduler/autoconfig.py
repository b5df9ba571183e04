"""Precision admission: which boundary dtype a fleet's links and memory admit.

Parity: src/wantrain/scheduler/autoconfig.py (`LADDER` :16,
`boundary_bytes_per_token` :33, `tokens_per_s_ceiling` :39, `floor_mbps` :48,
`stage_memory_bytes` :59, `evaluate` :131, `choose` :217, `report` :292,
`plan` :319). The boundary dtype is a decision variable: each rung, widest
first, is priced by the bandwidth one microbatch's boundary needs to cross a
hop inside one compute window (the floor), with a safety margin, and by the
stage's memory. Policies:

- "lossless": only rungs at least as wide as the compute dtype;
- "balanced": prefer lossless rungs, say so loudly when it falls back;
- "max_throughput": the rung with the highest wire ceiling that clears the
  margin.

Rungs are this engine's boundary formats (models/precision.py): fp32, bf16,
fp16 and the 1x128 block-scaled e5m2 and e4m3 (one byte per value plus one
fp32 scale per 128 values); "lossless" is the table's representability rule.
Memory is priced with this engine's model (`planner.act_bytes`: saved bf16
activations, deferred-W inputs and boundary buffers), not the reference's
fp32 autograd graph.
"""

from __future__ import annotations

from elysium_wan_b200.models import precision

# widest first
LADDER = list(precision.LADDER)
_BYTES = {name: f.wire_bytes for name, f in precision.FORMATS.items()}
BYTES_PER_PARAM_ADAM = 16
BYTES_PER_PARAM_HOST_ADAM = 8
BYTES_PER_PARAM_FROZEN = 2  # a frozen bf16 working copy (LoRA base)


def boundary_bytes_per_token(d_model: int, boundary: str, wire_ratio: float = 1.0) -> float:
    """Wire bytes per token per direction; `wire_ratio` is the codec's
    compression (1.0 raw over NVLink)."""
    return _BYTES[boundary] * d_model / max(1e-9, wire_ratio)


def tokens_per_s_ceiling(d_model: int, boundary: str, link_mbps: float,
                         wire_ratio: float = 1.0) -> float:
    """The wire's hard throughput ceiling per direction."""
    return (link_mbps * 1e6 / 8) / boundary_bytes_per_token(d_model, boundary, wire_ratio)


def floor_mbps(d_model: int, seq_len: int, mb_size: int, boundary: str, window_s: float,
               wire_ratio: float = 1.0) -> float:
    """Bandwidth at which one microbatch's boundary crosses in one window."""
    per_mb = boundary_bytes_per_token(d_model, boundary, wire_ratio) * mb_size * seq_len
    return per_mb * 8 / max(1e-12, window_s) / 1e6


def lossless(compute_dtype: str, boundary: str) -> bool:
    """The boundary holds every compute value exactly (a bf16 activation fits
    fp32 and bf16 bit for bit; fp16's exponent and the fp8 rungs do not)."""
    return precision.represents(boundary, compute_dtype)


def stage_memory_bytes(cfg, params_stage: int, n_layers_stage: int, mb_size: int,
                       live_graphs: int, boundary: str, recompute: bool, head_vocab: int = 0,
                       frozen_params_stage: int = 0, host_adam: bool = False,
                       extra_bytes: float = 0.0) -> dict:
    """One stage's device bytes at peak: optimizer state, boundary buffers,
    live activations of `live_graphs` microbatches (with recompute only the
    stage inputs stay live, plus one rebuilt graph), the deferred-W inputs of
    one microbatch, and the head's logits and their gradient."""
    from elysium_wan_b200.scheduler.planner import act_bytes

    T = mb_size * cfg.seq_len
    a = act_bytes(cfg, mb_size, "cuda")
    per_param = BYTES_PER_PARAM_HOST_ADAM if host_adam else BYTES_PER_PARAM_ADAM
    state = params_stage * per_param + frozen_params_stage * BYTES_PER_PARAM_FROZEN
    bnd = live_graphs * T * cfg.d_model * _BYTES[boundary] * 2
    if recompute:
        acts = live_graphs * a["boundary"] + n_layers_stage * (a["saved"] + a["w_keep"])
    else:
        acts = live_graphs * n_layers_stage * a["saved"] + n_layers_stage * a["w_keep"]
    head = 2 * T * head_vocab * 2 + T * head_vocab * 4 if head_vocab else 0
    total = state + bnd + acts + head + extra_bytes
    return dict(optimizer_state=state, boundary_buffers=bnd, activations=acts, head_logits=head,
                extra=extra_bytes, total=total)


def evaluate(cfg, params_stage: int, n_layers_stage: int, mb_size: int, live_graphs: int,
             link_mbps: float, window_s: float, mem_budget_bytes: float, margin: float = 2.0,
             compute_dtype: str = "bf16", head_vocab: int = 0, wire_ratio: float = 1.0,
             recompute: bool = True, host_adam: bool = False) -> list:
    """One row per rung, widest first."""
    rows = []
    for b in LADDER:
        fl = floor_mbps(cfg.d_model, cfg.seq_len, mb_size, b, window_s, wire_ratio)
        mem = stage_memory_bytes(cfg, params_stage, n_layers_stage, mb_size, live_graphs, b,
                                 recompute, head_vocab=head_vocab, host_adam=host_adam)
        rows.append(dict(
            boundary=b, lossless=lossless(compute_dtype, b),
            bytes_per_token=round(boundary_bytes_per_token(cfg.d_model, b, wire_ratio), 1),
            floor_mbps=round(fl, 1), needed_with_margin=round(fl * margin, 1),
            link_mbps=link_mbps, admissible=link_mbps >= fl, meets_margin=link_mbps >= fl * margin,
            tokens_per_s_ceiling=round(tokens_per_s_ceiling(cfg.d_model, b, link_mbps, wire_ratio)),
            stage_mem_gb=round(mem["total"] / 2**30, 2),
            fits_memory=mem["total"] <= mem_budget_bytes,
            needs_scale=precision.fmt(b).needs_scale))
    return rows


def _margin_note(r, margin):
    return (f"admissible WITHOUT the {margin:g}x margin: needs {r['needed_with_margin']:g} Mbps, "
            f"link is {r['link_mbps']:g} Mbps; expect residual stall")


def choose(rows: list, policy: str = "balanced", require_margin: bool = True,
           margin: float = 2.0):
    """(row, reason) under the policy; row None when nothing is admitted."""
    if policy not in ("lossless", "balanced", "max_throughput"):
        raise ValueError(f"unknown policy {policy!r}")
    fits = [r for r in rows if r["fits_memory"]]
    strong = [r for r in fits if r["meets_margin"]]
    weak = [r for r in fits if r["admissible"] and not r["meets_margin"]]
    if policy == "max_throughput":
        if strong:
            return max(strong, key=lambda r: r["tokens_per_s_ceiling"]), (
                f"highest-throughput rung clearing the {margin:g}x margin (boundary "
                f"approximation accepted)")
        if weak and not require_margin:
            r = max(weak, key=lambda r: r["tokens_per_s_ceiling"])
            return r, "highest-throughput admissible rung -- " + _margin_note(r, margin)
        return None, "nothing is admissible on this link at any precision"
    ll_strong = [r for r in strong if r["lossless"]]
    ll_weak = [r for r in weak if r["lossless"]]
    if ll_strong:
        return ll_strong[0], f"widest lossless rung clearing the {margin:g}x margin"
    if policy == "lossless":
        if ll_weak and not require_margin:
            return ll_weak[0], "widest lossless rung -- " + _margin_note(ll_weak[0], margin)
        need = [r["needed_with_margin"] for r in rows if r["lossless"]]
        return None, ("no lossless boundary clears this link (the widest needs "
                      f"{need[0] if need else float('nan'):g} Mbps with the margin): add "
                      "bandwidth, widen the compute window (more layers per stage, longer "
                      "sequences), run at the floor, or accept policy='balanced'")
    if ll_weak:
        return ll_weak[0], "widest lossless rung -- " + _margin_note(ll_weak[0], margin)
    pool = strong if require_margin else strong + weak
    if pool:
        return pool[0], ("NO LOSSLESS RUNG FITS: widest admissible approximate boundary; this "
                         "run is not lossless against the compute dtype")
    if weak:
        return weak[0], ("NO LOSSLESS RUNG FITS and nothing clears the margin: widest "
                         "approximate boundary -- " + _margin_note(weak[0], margin))
    return None, "nothing is admissible on this link at any precision"


def report(rows: list, chosen, reason: str) -> str:
    """The rationale table printed before a run starts."""
    hdr = (f"{'boundary':14s} {'lossless':>8s} {'B/token':>8s} {'floor':>9s} {'need':>9s} "
           f"{'admit':>6s} {'margin':>7s} {'tok/s':>10s} {'mem GB':>8s} {'fits':>5s}")
    out = [hdr, "-" * len(hdr)]
    for r in rows:
        mark = "  <-- chosen" if chosen is not None and r is chosen else ""
        out.append(f"{r['boundary']:14s} {str(r['lossless']):>8s} {r['bytes_per_token']:8.0f} "
                   f"{r['floor_mbps']:9.1f} {r['needed_with_margin']:9.1f} "
                   f"{str(r['admissible']):>6s} {str(r['meets_margin']):>7s} "
                   f"{r['tokens_per_s_ceiling']:10.0f} {r['stage_mem_gb']:8.2f} "
                   f"{str(r['fits_memory']):>5s}{mark}")
    out += ["", f"decision: {reason}"]
    return "\n".join(out)


def plan(cfg, params_stage: int, n_layers_stage: int, link_mbps: float, window_s: float,
         mem_budget_bytes: float, mb_size: int = 1, live_graphs: int = 2, margin: float = 2.0,
         policy: str = "balanced", compute_dtype: str = "bf16", require_margin: bool = True,
         boundary_override: str | None = None, head_vocab: int = 0, wire_ratio: float = 1.0,
         recompute: bool = True, host_adam: bool = False) -> dict:
    """{rows, chosen, reason, report}. An override skips the choice and
    reports what it costs."""
    if boundary_override is not None and boundary_override not in LADDER:
        raise ValueError(f"boundary {boundary_override!r} is not one of {LADDER}")
    rows = evaluate(cfg, params_stage, n_layers_stage, mb_size, live_graphs, link_mbps, window_s,
                    mem_budget_bytes, margin, compute_dtype, head_vocab, wire_ratio, recompute,
                    host_adam)
    if boundary_override:
        chosen = next(r for r in rows if r["boundary"] == boundary_override)
        reason = f"boundary_dtype pinned to {boundary_override} by the operator"
        if not chosen["meets_margin"]:
            reason += " -- WARNING: " + _margin_note(chosen, margin)
        if not chosen["fits_memory"]:
            reason += (f" -- WARNING: {chosen['stage_mem_gb']} GB per stage exceeds the "
                       f"{mem_budget_bytes / 2**30:.1f} GB budget")
    else:
        chosen, reason = choose(rows, policy, require_margin, margin)
    return dict(rows=rows, chosen=chosen, reason=reason, report=report(rows, chosen, reason))
