"""{plan, stages} job description -> JobSpec (reference:
src/wantrain/scheduler/fleetplan.py:45-335, keeps the job JSON schema).

A plan names the model (a preset and/or GPTConfig fields: MODEL_KEYS) and job
keys (microbatches, mb_size, steps, lr, seeds, dataset, recompute, precision,
ckpt_every, optimizer via `extras`). The stage count comes from "stages";
the cut is the compute-balanced partition over the fleet's device speeds.
"""

from __future__ import annotations

from elysium_wan_b200.models.config import GPTConfig, make_config
from elysium_wan_b200.runtime.spec import JobSpec
from elysium_wan_b200.scheduler import partition as part

MODEL_KEYS = ("preset", "vocab_size", "n_layer", "n_head", "d_model", "seq_len", "d_ff",
              "compute_dtype", "boundary_dtype", "attn_impl", "init_scheme", "init_std")
JOB_KEYS = ("microbatches", "mb_size", "steps", "lr", "init_seed", "data_seed", "dataset_path",
            "data_shards", "recompute", "ckpt_every", "optimizer", "tag", "stage_widths",
            "zb_mem_mode", "backend")


def model_config(plan: dict) -> GPTConfig:
    kw = {k: plan[k] for k in MODEL_KEYS if k in plan and k != "preset"}
    if "precision" in plan:
        p = plan["precision"]
        kw.setdefault("compute_dtype", p.get("compute", "bf16"))
        kw.setdefault("boundary_dtype", p.get("boundary", kw["compute_dtype"]))
    if "preset" in plan:
        return make_config(plan["preset"], **kw)
    return GPTConfig(**kw).validate()


def build_spec(plan: dict, stages: int | None, fleet: list | None = None) -> JobSpec:
    plan = dict(plan)
    cfg = model_config(plan)
    stages = int(stages or plan.get("stages", 1))
    job = {k: plan[k] for k in JOB_KEYS if k in plan}
    job.update(plan.get("extras", {}))
    dev = "cuda" if fleet and all(n.device.startswith("cuda") for n in fleet) else "cpu"
    if dev == "cuda":
        job.setdefault("backend", "nccl")
    spec = JobSpec(model=cfg, stages=stages, device=dev, **job)
    speeds = [1.0] * stages
    if fleet and len(fleet) >= stages and all(n.tflops_bf16 for n in fleet[:stages]):
        speeds = [float(n.tflops_bf16) for n in fleet[:stages]]
    try:
        spec.partition = part.even_blocks_partition(cfg, stages) if len(set(speeds)) == 1 else None
    except ValueError:
        spec.partition = None
    if spec.partition is None:
        spec.partition = part.proportional_partition(cfg, speeds)
    return spec


# ---------------------------------------------------------------- plan mode
# Rates the pricing assumes when a node states none.
_EFF = 0.55  # achieved fraction of a device's dense rate over a whole step
_HBM_BPS = 6.5e12
_PCIE_BPS = 50e9
_LINK_BPS = 770e9  # NVLink through NVSwitch, per direction (measured)


def largest_mb_size(spec, stage_fit, cap: int = 64) -> int:
    """The biggest power-of-two microbatch (<= cap) for which `stage_fit(spec)`
    holds, 0 if not even one sequence fits (reference: largest_mb_size,
    src/wantrain/scheduler/planner.py:178)."""
    best, mb = 0, 1
    while mb <= cap:
        spec.mb_size = mb
        if not stage_fit(spec):
            break
        best, mb = mb, mb * 2
    spec.mb_size = max(best, 1)
    return best


def price_candidate(spec, fleet: list, step_tokens: int) -> dict:
    """Modelled step of a finalized candidate spec on the fleet: the
    zero-bubble makespan of its stages' F / B / W costs (FLOP model at the
    slowest replica's rate times _EFF, recompute adding a forward), plus the
    optimizer pass (HBM, or PCIe for host moments) and, on wide stages, the
    ZeRO-1 exchange over the link. -> {step_s, tokens_per_s, bubble, ...}."""
    from elysium_wan_b200.scheduler import admission as ad
    from elysium_wan_b200.scheduler.planner import zb_config
    from elysium_wan_b200.scheduler.zero_bubble import zero_bubble

    S = spec.stages
    rates = []
    k = 0
    for w in spec.stage_widths:
        nodes = fleet[k:k + w]
        k += w
        rates.append(sum((n.tflops_bf16 or 1.0) for n in nodes) * 1e12 * _EFF)
    fs, bs, ws, opt, exch = [], [], [], [], []
    for r in range(S):
        t = ad.stage_terms(spec, r)
        f = t.flops_mb / 3.0 / rates[r]
        fs.append(f)
        bs.append(f * (2.0 if spec.recomputes(r) else 1.0))
        ws.append(f)
        w = spec.stage_widths[r]
        state = 16.0 * t.trainable / w
        opt.append(state / (_PCIE_BPS if spec.optimizer == "adamw-host" else _HBM_BPS))
        rs, ag = ad.exchange_bytes(t, w, spec.shard)
        exch.append((rs + ag) / _LINK_BPS)
    saved = spec.stage_costs
    spec.stage_costs = [[f, b, w] for f, b, w in zip(fs, bs, ws)]
    try:
        cfg = zb_config(spec)
        sched = zero_bubble(cfg, "2p")
        makespan = sched.makespan
        bubble = sched.bubble_rate
    finally:
        spec.stage_costs = saved
    step = makespan + max(opt) + max(exch)
    return {"step_s": step, "tokens_per_s": step_tokens / step, "bubble": bubble,
            "optimizer_s": max(opt), "exchange_s": max(exch)}


def plan_job(plan: dict, fleet: list, stages: int | None = None,
             bubble_target: float = 0.05) -> tuple:
    """Plan mode (reference: src/wantrain/scheduler/planner.py:767 `plan_job`,
    semantics only): a measured fleet -> a complete JobSpec and the rationale
    of every choice, or ValueError with the refusal.

    Candidates are every (depth, AdamW moments on the device or the host,
    recompute off or on) the plan leaves open; per candidate:
      - boundary precision: the plan's, else the rung admission picks for the
        fleet's link (scheduler/autoconfig.py `plan`, policy "balanced");
      - microbatch size: the plan's, else the largest power of two whose
        heaviest stage (parameter state plus the in-flight activations of the
        zero-bubble order) fits the smallest device less its reserve;
      - width: the fleet spread over the stages, ZeRO-1 if admission passes,
        else pieces, else width 1 (the rest are spares);
      - microbatches: the plan's, else the fewest whose schedule idles at
        most `bubble_target`, keeping the plan's tokens per step when it
        names them;
      - price: the modelled step (`price_candidate`).
    The fastest fitting candidate wins (ties: fewer stages, device moments,
    no recompute); the table of every candidate and refusal is the rationale."""
    from elysium_wan_b200.resources.node import mixed_fleet
    from elysium_wan_b200.scheduler import admission as ad
    from elysium_wan_b200.scheduler import autoconfig
    from elysium_wan_b200.scheduler.planner import stage_memory_model
    from elysium_wan_b200.scheduler.solve import solve_microbatches

    if not fleet:
        raise ValueError("plan mode needs a fleet")
    why = mixed_fleet(fleet)
    if why:
        raise ValueError(why)
    cfg = model_config(plan)
    gpu = all(n.device.startswith("cuda") for n in fleet)
    mems = [n.memory_bytes() for n in fleet if n.memory_bytes()]
    cap = min(mems) - ad.vram_reserve(min(mems)) if mems else None
    fixed = stages or plan.get("stages")
    n_max = min(len(fleet), cfg.n_layer)
    step_tokens = None
    if "microbatches" in plan and "mb_size" in plan:
        step_tokens = int(plan["microbatches"]) * int(plan["mb_size"]) * cfg.seq_len

    def worst_need(spec) -> float:
        spec.partition = None
        spec.partition = build_spec(dict(plan, optimizer=spec.optimizer), spec.stages,
                                    fleet[:spec.stages]).partition
        worst = 0.0
        for r in range(spec.stages):
            t = ad.stage_terms(spec, r)
            mem_f, _, _ = stage_memory_model(spec, r)
            w = spec.stage_widths[r]
            b = ad.device_bytes(t, w, spec.shard, 0, spec.optimizer == "adamw-host") + \
                max(1, spec.stages - r) * mem_f
            worst = max(worst, b)
        return worst

    def fits(spec) -> bool:
        return cap is None or worst_need(spec) <= cap

    rows, best = [], None
    for optimizer in ("adamw", "adamw-host"):
        for recompute in ((False, True) if "recompute" not in plan else (bool(plan["recompute"]),)):
            for S in ([int(fixed)] if fixed else range(1, n_max + 1)):
                p = dict(plan, optimizer=optimizer, recompute=recompute)
                spec = build_spec(p, S, fleet[:S])
                spec.optimizer, spec.recompute = optimizer, recompute
                row = {"stages": S, "optimizer": optimizer, "recompute": recompute}
                # boundary rung
                if "boundary_dtype" not in plan and "precision" not in plan and S > 1:
                    t0 = ad.stage_terms(spec, 0)
                    link_mbps = (_LINK_BPS if gpu else 1e9 / 8) * 8 / 1e6
                    rung = autoconfig.plan(cfg, t0.trainable, max(1, cfg.n_layer // S), link_mbps,
                                           0.2, cap or 1e18, mb_size=spec.mb_size,
                                           recompute=recompute,
                                           host_adam=optimizer == "adamw-host")
                    if rung["chosen"] is not None:
                        spec.model.boundary_dtype = rung["chosen"]["boundary"]
                row["boundary"] = spec.model.boundary_dtype
                # width and layout
                width = max(1, len(fleet) // S) if "stage_widths" not in plan else None
                spec.stage_widths = list(plan["stage_widths"]) if width is None else [1] * S
                spec.shard = "zero1"
                # microbatch size
                if "mb_size" not in plan:
                    mb = largest_mb_size(spec, fits)
                    if mb == 0:
                        row["refused"] = "one sequence per microbatch does not fit"
                        rows.append(row)
                        continue
                elif not fits(spec):
                    row["refused"] = (f"needs {worst_need(spec) / 2**30:.1f} GiB on the largest "
                                      f"stage, {(cap or 0) / 2**30:.1f} GiB per device")
                    rows.append(row)
                    continue
                row["mb_size"] = spec.mb_size
                layout = None
                if width and width > 1:
                    spec.stage_widths = [width] * S
                    devs = ad.devices_from_nodes(fleet[:width * S])
                    for shard in ("zero1", "pieces"):
                        spec.shard = shard
                        spec.peer_weights, spec.mb_owner = None, None
                        spec.microbatches = max(spec.microbatches, width)
                        spec.schedule_order = None
                        ok, reasons, _ = ad.admit(spec.finalize(), devs)
                        if ok and fits(spec):
                            layout = shard
                            break
                        row.setdefault("refused_layouts", {})[shard] = \
                            [r.text() for r in reasons] or ["memory"]
                    if layout is None:
                        spec.stage_widths, spec.shard = [1] * S, "zero1"
                row["widths"] = list(spec.stage_widths)
                row["layout"] = layout
                # microbatches
                w = max(spec.stage_widths)
                if "microbatches" in plan:
                    reason = "given by the plan"
                else:
                    sol = solve_microbatches(S, bubble_target, mb_size=spec.mb_size,
                                             seq_len=cfg.seq_len, floor=w)
                    spec.microbatches = -(-sol["microbatches"] // w) * w
                    reason = sol["reason"]
                row["microbatches"] = spec.microbatches
                row["microbatches_reason"] = reason
                spec.peer_weights, spec.mb_owner, spec.schedule_order = None, None, None
                spec.finalize()
                tokens = step_tokens or spec.microbatches * spec.mb_size * cfg.seq_len
                price = price_candidate(spec, fleet, tokens)
                row.update({k: round(v, 6) if isinstance(v, float) else v for k, v in price.items()})
                rows.append(row)
                key = (-price["tokens_per_s"], S, optimizer != "adamw", recompute)
                if best is None or key < best[0]:
                    best = (key, spec, row)
    if best is None:
        raise ValueError(f"no candidate fits {cfg.n_layer} layers on "
                         f"{(cap or 0) / 2**30:.1f} GiB devices: "
                         + "; ".join(f"{r['stages']} stages/{r['optimizer']}"
                                     f"/recompute={r['recompute']}: {r.get('refused')}"
                                     for r in rows if r.get("refused"))[:800])
    _, spec, row = best
    rationale = {
        "fleet": len(fleet),
        "depth": {"stages": spec.stages, "optimizer": spec.optimizer, "given": bool(fixed),
                  "recompute": spec.recompute,
                  "device_budget_gib": None if cap is None else round(cap / 2**30, 2)},
        "precision": {"boundary": spec.model.boundary_dtype,
                      "given": "boundary_dtype" in plan or "precision" in plan},
        "mb_size": {"value": spec.mb_size, "given": "mb_size" in plan},
        "width": {"replicas": spec.stage_widths, "layout": row.get("layout"),
                  "spares": len(fleet) - sum(spec.stage_widths)},
        "microbatches": {"value": spec.microbatches, "reason": row["microbatches_reason"]},
        "price": {k: row[k] for k in ("step_s", "tokens_per_s", "bubble", "optimizer_s",
                                      "exchange_s")},
        "candidates": rows,
        "partition": spec.partition,
        "device": "cuda" if gpu else "cpu",
    }
    return spec, rationale
