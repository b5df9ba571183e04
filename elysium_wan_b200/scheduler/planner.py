"""Spec-level planning: analytic stage costs and memory model, and the
zero-bubble order a JobSpec runs when it names none.

Reference: default_schedule / schedule_for_spec / stage_memory_model in
src/wantrain/scheduler/zero_bubble.py:540-1000. The memory model here counts
the bytes the B200 kernels actually keep: F's saved activations per block,
the W inputs (dY, X pairs) that B hands over, and the boundary tensor.
"""

from __future__ import annotations

from elysium_wan_b200.scheduler import partition as part
from elysium_wan_b200.scheduler.zero_bubble import (ZBConfig, comm_seconds, simulate_slots,
                                                    slot_orders, stage_peak, zero_bubble)

_BOUNDARY_BYTES = {"fp32": 4, "bf16": 2, "fp16": 2, "fp8_e5m2_b128": 1, "fp8_e4m3_b128": 1}


def act_bytes(cfg, spec_mb_size: int, device: str) -> dict:
    """Per-microbatch bytes of one block: saved activations (F), kept W inputs
    (after B), and the boundary tensor."""
    T = spec_mb_size * cfg.seq_len
    d, f = cfg.d_model, cfg.ff
    e = 2 if device.startswith("cuda") else 4
    saved = T * e * (d + 3 * d + d + d + d + 2 * f) + T * cfg.n_head * 4
    w_keep = T * e * (8 * d + 2 * f)
    nb = _BOUNDARY_BYTES[cfg.boundary_dtype]
    boundary = T * d * nb + (T * (d // 128) * 4 if nb == 1 else 0)
    return dict(saved=saved, w_keep=w_keep, boundary=boundary)


def stage_memory_model(spec, stage: int) -> tuple[float, float, float]:
    """(mem_f, mem_b, mem_w) bytes of one microbatch on `stage` (sum zero)."""
    a, b = spec.partition[stage]
    cfg = spec.model
    blocks = sum(1 for e in range(a, b) if 1 <= e <= cfg.n_layer)
    m = act_bytes(cfg, spec.mb_size, spec.device_for(stage))
    T = spec.mb_size * cfg.seq_len
    head = b == cfg.n_entries
    head_keep = T * ((cfg.vocab_size + 7) // 8 * 8) * 2 + T * cfg.d_model * 2 if head else 0
    keep = blocks * m["w_keep"] + head_keep
    if spec.recomputes(stage):
        mem_f = blocks * m["boundary"] + m["boundary"] + head_keep
    else:
        mem_f = blocks * (m["saved"] + m["boundary"]) + m["boundary"] + head_keep
    mem_b = keep - mem_f
    mem_w = -keep
    return float(mem_f), float(mem_b), float(mem_w)


def analytic_costs(spec) -> tuple[list, list, list]:
    """Per-stage F/B/W costs from the FLOP model (seconds up to a constant):
    F, B and W each carry one GEMM pass; B adds attention's backward."""
    c = part.layer_costs(spec.model)
    fs, bs, ws = [], [], []
    for r, (a, b) in enumerate(spec.partition):
        tot = sum(c[a:b]) / sum(spec.peer_weights[r])
        rec = 1.0 if spec.recomputes(r) else 0.0
        fs.append(tot)
        bs.append(tot * (1.1 + rec))
        ws.append(tot * 0.9)
    return fs, bs, ws


def zb_config(spec, budget_bytes: list | None = None) -> ZBConfig:
    if spec.stage_costs:
        fs = [float(x[0]) for x in spec.stage_costs]
        bs = [float(x[1]) for x in spec.stage_costs]
        ws = [float(x[2]) for x in spec.stage_costs]
    else:
        fs, bs, ws = analytic_costs(spec)
    comm = []
    for j in range(spec.stages - 1):
        link = spec.links[j] if j < len(spec.links) else {}
        m = act_bytes(spec.model, spec.mb_size, spec.device_for(j))
        t = comm_seconds(m["boundary"], link.get("bw_mbps", 0.0), 2 * link.get("latency_ms", 0.0))
        # Express communication in the cost unit of the analytic model.
        comm.append(t * (sum(fs) / max(1e-12, len(fs))) if not spec.stage_costs else t)
    mems = [stage_memory_model(spec, r) for r in range(spec.stages)]
    cfg = ZBConfig(spec.stages, spec.microbatches, fs, bs, ws, comm,
                   [m[0] for m in mems], [m[1] for m in mems], [m[2] for m in mems],
                   max_mem=budget_bytes)
    return cfg


def default_schedule(spec, budget_bytes: list | None = None) -> list:
    """schedule_order[stage][peer] for the spec: the zero-bubble solve on the
    aggregate stage, split over the stage's peers by microbatch ownership."""
    mode = spec.zb_mem_mode
    cfg = zb_config(spec, budget_bytes)
    if mode == "auto":
        if budget_bytes is None:
            mode = "2p"
        else:
            unit = max(max(cfg.mem_f), max(f + b for f, b in zip(cfg.mem_f, cfg.mem_b)))
            two_p = [2 * spec.stages * unit] * spec.stages
            cfg = cfg.with_budget([min(a, b) for a, b in zip(budget_bytes, two_p)])
            mode = "given"
    mode = mode if mode in ("1p", "2p", "given") else "2p"
    sched = zero_bubble(cfg, mode)
    split = [slot_orders(sched.orders[r], spec.mb_owner[r], spec.stage_widths[r])
             for r in range(spec.stages)]
    if any(w > 1 for w in spec.stage_widths):
        lanes = lane_orders(spec, cfg, mode, budget_bytes)
        if lanes:
            mixed = [lanes.get(r, split[r]) for r in range(spec.stages)]
            try:
                _, ms_split = simulate_slots(cfg, split, spec.peer_weights)
                _, ms_lanes = simulate_slots(cfg, mixed, spec.peer_weights)
            except ValueError:  # a lane waits on an op another slot orders later
                ms_lanes = ms_split = 0.0
            if ms_lanes < ms_split * (1.0 - 1e-9):
                split = mixed
    return [[[[op, mb] for op, mb in o] for o in orders] for orders in split]


def lane_orders(spec, cfg: ZBConfig, mode: str, budget_bytes: list | None = None) -> dict:
    """{stage: [order per peer]} for the wide stages, each peer's order solved
    as a pipeline of its own (reference: _lane_orders / bridge_orders,
    src/wantrain/scheduler/zero_bubble.py:715-870, semantics only).

    A peer of a wide stage runs whole microbatches, the ones it owns. Seen
    from those microbatches the job is a pipeline in which every stage gives
    them the peer's share of its throughput, so each op costs the aggregate
    stage cost x (sum of the stage's weights / the peer's weight); the
    zero-bubble solve of that lane, mapped onto the owned microbatches, is the
    peer's order. Each solve keeps the device budget of one GPU, which the
    stage-level solve has to share among all the stage's microbatches. A
    stage whose lanes cannot all be solved, or whose lane order would not fit
    its budget, keeps the stage-level split. default_schedule keeps the lanes
    only when the slot simulation finds them faster."""
    out = {}
    for s in range(spec.stages):
        weights = spec.peer_weights[s]
        if len(weights) == 1:
            continue
        total = float(sum(weights))
        per: list | None = []
        for q, wq in enumerate(weights):
            own = [mb for mb, o in enumerate(spec.mb_owner[s]) if o == q]
            if not own:
                per.append([])
                continue
            k = total / wq
            lane = ZBConfig(cfg.n_stages, len(own), [c * k for c in cfg.cost_f],
                            [c * k for c in cfg.cost_b], [c * k for c in cfg.cost_w], cfg.comm,
                            cfg.mem_f, cfg.mem_b, cfg.mem_w, max_mem=cfg.max_mem)
            try:
                lane_sched = zero_bubble(lane, mode)
            except ValueError:
                per = None
                break
            order = [(op, own[i]) for op, i in lane_sched.orders[s]]
            if budget_bytes and stage_peak(cfg, s, order) > budget_bytes[s] * (1 + 1e-9):
                per = None
                break
            per.append(order)
        if per is not None:
            out[s] = per
    return out
