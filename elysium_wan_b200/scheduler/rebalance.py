"""Rebalance from telemetry: re-cut a running job's chain from the stage costs it
measures, and spot a slot that has become slow.

Reference behaviour: src/wantrain/coordinator/coordinator.py (`_maybe_rebalance`
:2194, `_maybe_recut` :2299, `_watch_slow` :2406, `refined_partition` :3046,
`recut_refusal` :3068, `stage_compute_ms` :3085, `slow_slots` :3091) and
src/wantrain/scheduler/zero_bubble.py (`profiles_from_telemetry` :1008).

Inputs are the per-step WT_TELEM summaries a stage prints
(runtime/telemetry.summarize_step: {"ops": {"F"|"B"|"W": {"n", "med_ms"}}, ...}),
collected per slot by the coordinator into a window of recent steps.

- `profiles_from_telemetry(spec, windows)`: per stage and peer, the median over
  the window of each op's per-step median, in seconds.
- `refined_partition(spec, profiles, fits, min_gain)`: every stage's measured
  rate (microbatches per second, summed over its peers) turns the model's
  per-entry cost into that stage's speed (cost units per second); the exact
  min-max partition DP (partition.assign_layers) then re-cuts the chain for
  those speeds. The result is taken only when it shortens the slowest stage's
  time per microbatch by at least `min_gain`.
- `recut_pays(...)`: the saving over the remaining steps against the cost of a
  restart.
- `slow_slots(hist, base, ratio, runs)`: slots whose last `runs` compute
  samples all exceed `ratio` x their own baseline.
"""

from __future__ import annotations

import math
import statistics

from elysium_wan_b200.scheduler.partition import assign_layers, layer_costs

OPS = ("F", "B", "W")


def stage_compute_ms(summary: dict) -> float:
    """A slot's compute per microbatch in one summary: F + B + W medians (ms)."""
    ops = summary.get("ops") or {}
    return float(sum((ops.get(k) or {}).get("med_ms", 0.0) for k in OPS))


def profiles_from_telemetry(spec, windows: dict) -> list:
    """profiles[stage][peer] = {"t_f", "t_b", "t_w"} in seconds. windows:
    {(stage, peer): [summary, ...]}. A W that runs inside B (no W op of its
    own in a summary) counts as 0. Raises ValueError naming a slot without F
    or B samples."""
    out = []
    for r in range(spec.stages):
        row = []
        for q in range(spec.stage_widths[r]):
            win = windows.get((r, q)) or []
            prof = {}
            for op in OPS:
                xs = [float(s["ops"][op]["med_ms"]) for s in win
                      if (s.get("ops") or {}).get(op, {}).get("n", 0) > 0]
                if not xs:
                    if op == "W":
                        prof["t_w"] = 0.0
                        continue
                    raise ValueError(f"no {op} sample in the telemetry of slot ({r}, {q})")
                if not all(math.isfinite(x) and x >= 0 for x in xs):
                    raise ValueError(f"{op} med_ms of slot ({r}, {q}) must be finite and >= 0")
                prof["t_" + op.lower()] = statistics.median(xs) / 1e3
            row.append(prof)
        out.append(row)
    return out


def stage_rates(profiles: list) -> list:
    """Microbatches per second of each stage: its peers' rates added."""
    return [sum(1.0 / max(1e-9, p["t_f"] + p["t_b"] + p["t_w"]) for p in row) for row in profiles]


def refined_partition(spec, profiles: list, fits=None, min_gain: float = 0.05):
    """-> (new partition, slowest stage before, after) in seconds per
    microbatch, or None when the DP returns the same cut, nothing fits, or the
    slowest stage shrinks by less than `min_gain`. fits(stage, lo, hi) -> bool."""
    costs = layer_costs(spec.model)
    rate = stage_rates(profiles)
    speed = [sum(costs[a:b]) * r for (a, b), r in zip(spec.partition, rate)]
    try:
        new = [list(x) for x in assign_layers(costs, speed, fits)]
    except ValueError:
        return None
    before = max(1.0 / r for r in rate)
    after = max(sum(costs[a:b]) / s for (a, b), s in zip(new, speed))
    if new == [list(x) for x in spec.partition] or after > (1.0 - min_gain) * before:
        return None
    return new, before, after


def recut_pays(before_s: float, after_s: float, microbatches: int, remaining_steps: int,
               cost_s: float) -> tuple[bool, float]:
    """(worth it, seconds saved): the slowest stage sets the pipeline's pace, so
    each remaining step saves (before - after) per microbatch."""
    saving = (before_s - after_s) * microbatches * max(0, remaining_steps)
    return saving > cost_s, saving


def recut_refusal(spec) -> str | None:
    """Why a running job cannot be re-cut, or None. The waves are converted
    through the logical form (fault_tolerance/logical.py), which handles widths
    and ZeRO-1 / pieces; it does not move a tied table between stages or MoE
    routing state."""
    if spec.stages < 2:
        return "one stage"
    if getattr(spec.model, "tie_embeddings", False):
        return "a tied embedding"
    if getattr(spec.model, "moe_experts", 0):
        return "an MoE model"
    return None


def slow_slots(hist: dict, base: dict, ratio: float = 1.3, runs: int = 3) -> list:
    """[(slot, latest / baseline)] for the slots whose last `runs` samples all
    exceed `ratio` x their baseline. hist: slot -> [ms, ...]; base: slot -> ms."""
    out = []
    for slot, xs in hist.items():
        b = base.get(slot)
        tail = xs[len(xs) - runs:] if len(xs) >= runs else []
        if b and tail and all(x > ratio * b for x in tail):
            out.append((slot, round(xs[-1] / b, 3)))
    return out


def stage_costs_from_profiles(profiles: list, peer_weights: list | None = None) -> list:
    """[F, B, W] seconds per stage: each peer's measured ops weighted by its
    share of the stage's microbatches (its ownership weight)."""
    out = []
    for r, row in enumerate(profiles):
        wr = (peer_weights[r] if peer_weights else None) or [1.0] * len(row)
        tot = sum(wr)
        out.append([sum(p[k] * w for p, w in zip(row, wr)) / tot / len(row)
                    for k in ("t_f", "t_b", "t_w")])
    return out


def replan_schedule(spec, profiles: list, min_gain: float = 0.10, hops: list | None = None):
    """Re-solve the zero-bubble order from measured costs (reference:
    scheduler/zero_bubble.py:1079 `replan`, its order half). Ownership and
    the cut stay, so the run's bits do not change. -> (new schedule_order,
    predicted s/step now, predicted after) when the new order is at least
    `min_gain` shorter under the same measured costs, else None."""
    import copy

    from elysium_wan_b200.scheduler.planner import default_schedule, zb_config
    from elysium_wan_b200.scheduler.zero_bubble import simulate_slots

    s2 = copy.deepcopy(spec)
    s2.stage_costs = stage_costs_from_profiles(profiles, spec.peer_weights)
    cfg = _measured_comm(zb_config(s2), hops)

    def makespan(order):
        slots = [[[(op, int(mb)) for op, mb in o] for o in per_stage] for per_stage in order]
        return simulate_slots(cfg, slots, spec.peer_weights)[1]

    cur = makespan(spec.schedule_order)
    new_order = default_schedule(s2)
    new = makespan(new_order)
    if new > (1.0 - min_gain) * cur:
        return None
    return new_order, cur, new


def measured_model(profiles: list) -> tuple[list, list]:
    """(speeds, costs) of a window: speeds[stage][peer] is the peer's measured
    rate (microbatches per second over F + B + W), costs[stage] the [F, B, W]
    seconds under which `simulate_slots` gives peer q of a stage an op time of
    cost x sum(speeds) / speeds[q], the peer's measured time (exactly so when
    a stage's peers differ by one factor; otherwise the op mix is averaged)."""
    speeds, costs = [], []
    for row in profiles:
        w = [1.0 / max(1e-9, p["t_f"] + p["t_b"] + p["t_w"]) for p in row]
        speeds.append(w)
        costs.append([sum(p[k] * wq for p, wq in zip(row, w)) / len(row) / sum(w)
                      for k in ("t_f", "t_b", "t_w")])
    return speeds, costs


def _with_one_each(n: int, weights: list) -> list:
    """Weights under which IWRR leaves no peer without a microbatch: a peer
    that gets none has its weight doubled until it does."""
    from elysium_wan_b200.scheduler.zero_bubble import iwrr

    w = list(weights)
    for _ in range(64):
        got = set(iwrr(n, w))
        if len(got) == len(w):
            return w
        for q in range(len(w)):
            if q not in got:
                w[q] *= 2.0
    raise ValueError("cannot give every peer a microbatch")


def replan_ownership(spec, profiles: list, min_gain: float = 0.10, hops: list | None = None) -> dict:
    """Re-solve a job's ownership and order from measured per-peer costs
    (reference: scheduler/zero_bubble.py:1079 `replan`, both halves). Each
    wide stage's peer weights become its peers' measured rates (every peer
    keeps at least one microbatch, so the next window measures it again), the
    microbatches are re-dealt by IWRR and the zero-bubble order re-solved.
    Both predictions run the same measured model (`measured_model`, and the
    hops' measured transfer times when given: `hops_from_telemetry`), so a
    bias of the profile cancels. Only peer_weights, mb_owner and
    schedule_order change. Unlike the reference's per-microbatch fold, this
    engine's declared `dp_tree` fold sums each replica's own microbatches
    first, so moving microbatches moves bits: the caller records the old table
    in the spec's `ownership_log` from the resume step on, and the oracle
    follows it.

    -> {"decision", "pred_cur_s", "pred_new_s", "peer_weights", "mb_owner",
    "schedule_order", "stage_costs", "owner_changed", "why"}."""
    import copy

    from elysium_wan_b200.scheduler.planner import zb_config
    from elysium_wan_b200.scheduler.zero_bubble import simulate_slots

    if not 0.0 <= min_gain < 1.0:
        raise ValueError(f"min_gain must be in [0, 1), got {min_gain}")
    speeds, costs = measured_model(profiles)
    cur = copy.deepcopy(spec)
    cur.stage_costs = costs
    cfg = _measured_comm(zb_config(cur), hops)

    def predict(order):
        slots = [[[(op, int(mb)) for op, mb in o] for o in per_stage] for per_stage in order]
        return simulate_slots(cfg, slots, speeds)[1]

    pred_cur = predict(spec.schedule_order)
    new = copy.deepcopy(spec)
    new.stage_costs = costs
    new.peer_weights = [[round(x / max(row), 4) for x in _with_one_each(spec.microbatches, row)]
                        if len(row) > 1 else [1.0] for row in speeds]
    new.mb_owner, new.schedule_order = None, None
    new.finalize()
    pred_new = predict(new.schedule_order)
    owner_changed = new.mb_owner != spec.mb_owner
    order_changed = new.schedule_order != spec.schedule_order
    gain_ok = pred_new <= (1.0 - min_gain) * pred_cur
    decision = gain_ok and (owner_changed or order_changed)
    if decision:
        why = f"predicted {pred_cur:.6g} s -> {pred_new:.6g} s per step"
    elif not (owner_changed or order_changed):
        why = "the re-solve gives the current ownership and order"
    else:
        why = (f"predicted {pred_cur:.6g} s -> {pred_new:.6g} s per step, below the "
               f"{min_gain:.0%} threshold")
    return {"decision": decision, "pred_cur_s": pred_cur, "pred_new_s": pred_new,
            "peer_weights": new.peer_weights, "mb_owner": new.mb_owner,
            "schedule_order": new.schedule_order, "stage_costs": costs,
            "owner_changed": owner_changed, "why": why}


# ------------------------------------------------------------- fit feedback
def order_peak(order, deltas: dict) -> float:
    """Peak activation bytes an order holds (F adds deltas["F"], B and W
    their own, usually negative, deltas)."""
    m = peak = 0.0
    for op, _mb in order:
        m += deltas[op]
        peak = max(peak, m)
    return peak


def calibrated_budget(spec, stage: int, peak: float, budget: float, base: float,
                      oom: bool = False, feedback: float = 1.25) -> float:
    """The activation budget, in the memory model's bytes, under which
    `stage`'s schedule fits after a measured overshoot (reference behaviour:
    `calibrated_budget`, src/wantrain/coordinator/coordinator.py:3100-3136).
    The fit held `peak` bytes of which `base` were resident before any
    microbatch; the model expected the order's in-flight peak. The ratio of
    the two activation figures (times `feedback` again for an out-of-memory
    fit, whose demand is unknown) scales the room the budget leaves. Never
    below one microbatch's F and B."""
    from elysium_wan_b200.scheduler.planner import stage_memory_model

    mf, mb, mw = stage_memory_model(spec, stage)
    modeled = max(order_peak(o, {"F": mf, "B": mb, "W": mw}) for o in spec.schedule_order[stage])
    factor = max(1.0, (peak - base) / max(1.0, modeled)) * (feedback if oom else 1.0)
    return max(mf, mf + mb, (budget - base) / factor)


def budget_list(spec, caps: dict) -> list:
    """Per-stage schedule budgets: the calibrated caps, no cap elsewhere."""
    return [float(caps.get(r, math.inf)) for r in range(spec.stages)]


def memory_partition(spec, budgets: list) -> list | None:
    """A cut that every stage's memory allows: the min-max cost partition
    (the model's per-entry costs; a wide stage's replicas add their weights'
    throughput) among the cuts in which each stage's resident state (its
    layout's parameters, gradients and moments) plus the zero-bubble warm-up's
    (stages - r) microbatches of F activations fits `budgets[r]`. None when no
    cut fits or the answer is the current cut."""
    import copy

    from elysium_wan_b200.scheduler import admission as ad
    from elysium_wan_b200.scheduler.planner import stage_memory_model

    costs = layer_costs(spec.model)
    host = spec.optimizer == "adamw-host"
    need: dict = {}

    def fits(r, lo, hi):
        if (r, lo, hi) not in need:
            s2 = copy.copy(spec)
            s2.partition = [list(x) for x in spec.partition]
            s2.partition[r] = [lo, hi]
            mf, _, _ = stage_memory_model(s2, r)
            t = ad.stage_terms(s2, r)
            need[(r, lo, hi)] = ad.device_bytes(t, spec.stage_widths[r], spec.shard, 0, host) + \
                max(1, spec.stages - r) * max(0.0, mf)
        return need[(r, lo, hi)] <= budgets[r]

    speed = [float(sum(w)) for w in spec.peer_weights]
    try:
        new = [list(x) for x in assign_layers(costs, speed, fits)]
    except ValueError:
        return None
    return None if new == [list(x) for x in spec.partition] else new


def hops_from_telemetry(spec, windows: dict) -> list:
    """Per hop j -> j + 1, the seconds a sender spends per boundary transfer,
    measured: the median over the window of busy_ms / frames of every link
    across the hop (stage j's next<q> links, stage j + 1's prev<p> links), or
    None for a hop nothing was measured on (a plane without per-link
    statistics). A frame counts once however many fragments and flows carry
    it (reference: `hops_from_telemetry`, src/wantrain/scheduler/
    zero_bubble.py:1030, semantics only)."""
    out = []
    for j in range(spec.stages - 1):
        xs = []
        for r, head in ((j, "next"), (j + 1, "prev")):
            for q in range(spec.stage_widths[r]):
                for summ in windows.get((r, q)) or []:
                    for label, h in (summ.get("hops") or {}).items():
                        if not isinstance(h, dict) or label.rstrip("0123456789") != head:
                            continue
                        if h.get("frames", 0) > 0:
                            xs.append(float(h["busy_ms"]) / 1e3 / h["frames"])
        out.append(statistics.median(xs) if xs else None)
    return out


def _measured_comm(cfg, hops):
    """cfg with each hop's modelled transfer replaced by its measured one."""
    if hops:
        cfg.comm = [c if m is None else float(m) for c, m in zip(cfg.comm, hops)]
    return cfg
