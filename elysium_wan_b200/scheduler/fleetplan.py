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
def plan_job(plan: dict, fleet: list, stages: int | None = None,
             bubble_target: float = 0.05) -> tuple:
    """Plan mode (reference: src/wantrain/scheduler/planner.py:767 `plan_job`):
    a measured fleet -> a complete JobSpec and the rationale of every choice,
    or ValueError with the refusal.

    - depth: the `stages` given (argument or plan), else the fewest stages whose
      largest stage holds its parameter state (bf16 working copy, fp32 master,
      gradient and AdamW moments) and its in-flight activations on the
      smallest device of the fleet; with no such depth, the moments go to the
      host ("adamw-host") and the search repeats;
    - width: the fleet spread over the stages (fleet // depth replicas each,
      the rest spares); a wide stage takes the ZeRO-1 layout if admission
      passes (scheduler/admission.py), else pieces, else width 1;
    - microbatches: the plan's, else the fewest whose zero-bubble schedule
      idles at most `bubble_target` (solve.solve_microbatches);
    - the cut: even blocks on a uniform fleet, else proportional to speed."""
    from elysium_wan_b200.resources.node import mixed_fleet
    from elysium_wan_b200.scheduler import admission as ad
    from elysium_wan_b200.scheduler.planner import stage_memory_model
    from elysium_wan_b200.scheduler.solve import solve_microbatches

    if not fleet:
        raise ValueError("plan mode needs a fleet")
    why = mixed_fleet(fleet)
    if why:
        raise ValueError(why)
    cfg = model_config(plan)
    rationale: dict = {"fleet": len(fleet)}
    gpu = all(n.device.startswith("cuda") for n in fleet)
    mems = [n.memory_bytes() for n in fleet if n.memory_bytes()]
    cap = min(mems) - ad.vram_reserve(min(mems)) if mems else None
    fixed = stages or plan.get("stages")
    n_max = min(len(fleet), cfg.n_layer)

    def trial(S: int, optimizer: str):
        p = dict(plan)
        p["optimizer"] = optimizer
        spec = build_spec(p, S, fleet[:S])
        spec.stage_widths = [1] * S
        spec.microbatches = spec.microbatches or 1
        spec.peer_weights = None
        spec.mb_owner = None
        worst, need = 0.0, []
        for r in range(S):
            t = ad.stage_terms(spec, r)
            mem_f, _, _ = stage_memory_model(spec, r)
            inflight = max(1, S - r)
            b = ad.device_bytes(t, 1, "zero1", 0, optimizer == "adamw-host") + inflight * mem_f
            need.append(b)
            worst = max(worst, b)
        return spec, worst, need

    chosen = None
    for optimizer in ("adamw", "adamw-host"):
        depths = [int(fixed)] if fixed else range(1, n_max + 1)
        for S in depths:
            spec, worst, need = trial(S, optimizer)
            if cap is None or worst <= cap:
                chosen = (spec, S, optimizer, need)
                break
        if chosen:
            break
    if chosen is None:
        raise ValueError(f"no depth up to {n_max} stages fits {cfg.n_layer} layers on "
                         f"{(cap or 0) / 2**30:.1f} GiB devices, even with host AdamW moments")
    spec, S, optimizer, need = chosen
    rationale["depth"] = {"stages": S, "optimizer": optimizer, "given": bool(fixed),
                          "stage_gib": [round(b / 2**30, 2) for b in need],
                          "device_budget_gib": None if cap is None else round(cap / 2**30, 2)}
    # widths and layout
    width = max(1, len(fleet) // S) if "stage_widths" not in plan else None
    layout = None
    if width and width > 1:
        spec.stage_widths = [width] * S
        devs = ad.devices_from_nodes(fleet[:width * S])
        for shard in ("zero1", "pieces"):
            spec.shard = shard
            spec.peer_weights = None
            spec.mb_owner = None
            spec.microbatches = max(spec.microbatches, width)
            ok, reasons, _ = ad.admit(spec.finalize(), devs)
            if ok:
                layout = shard
                break
            rationale.setdefault("refused_layouts", {})[shard] = [r.text() for r in reasons]
        if layout is None:
            spec.stage_widths = [1] * S
            spec.shard = "zero1"
            width = 1
    rationale["width"] = {"replicas": width or spec.stage_widths, "layout": layout,
                          "spares": len(fleet) - sum(spec.stage_widths)}
    # microbatches
    if "microbatches" not in plan:
        sol = solve_microbatches(S, bubble_target, mb_size=spec.mb_size,
                                 seq_len=cfg.seq_len, floor=max(spec.stage_widths))
        w = max(spec.stage_widths)
        spec.microbatches = -(-sol["microbatches"] // w) * w  # every replica the same count
        rationale["microbatches"] = {"value": spec.microbatches, "reason": sol["reason"]}
    else:
        rationale["microbatches"] = {"value": spec.microbatches, "reason": "given by the plan"}
    spec.optimizer = optimizer
    spec.peer_weights = None
    spec.mb_owner = None
    spec.schedule_order = None
    spec.finalize()
    rationale["partition"] = spec.partition
    rationale["device"] = "cuda" if gpu else "cpu"
    return spec, rationale
