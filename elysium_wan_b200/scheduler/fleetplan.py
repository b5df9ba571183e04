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
