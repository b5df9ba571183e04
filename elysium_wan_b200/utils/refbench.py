"""Reference arm of bench.py: the UNMODIFIED reference (virgiliolrf/elysium-wan,
laid out in baseline/_ref) run through its own public API on the same config.

Path: rank 0 builds the reference's own JobSpec for the 15.8B GPT (48 layers,
d 5120, 40 heads, seq 2048, vocab 50257, bf16 compute, sdpa/flash attention,
fp8 e4m3 boundaries -- the reference's per-token-scaled recipe, the closest it
has to the 1x128 block recipe -- zero-bubble schedule, 64 microbatches of 1
sequence, activation recompute as its production flags set) cut into N stages
of 48/N layers, one stage per GPU (`devices`), and runs it with the
reference's single-machine launcher `wantrain.launch.local.run_local` (one
stage process per slot, its framed TCP data plane over loopback). The other
torchrun ranks only wait. Step time per stage is the reference's own WT_TELEM
`step_ms` (host monotonic clock; the reference exposes no device timer); the
job's step time is the max over stages, averaged over the K timed steps after
W warm-up steps.
"""

from __future__ import annotations

import json
import os
import re
import socket
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF = os.path.join(ROOT, "baseline", "_ref")


def unavailable(why: str) -> dict:
    return {"impl": "reference", "unavailable": why}


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _wait_for_rank0(world: int):
    """Non-zero torchrun ranks idle until rank 0's run ends (gloo barrier)."""
    import datetime

    import torch.distributed as dist

    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=7200))
    dist.barrier()
    dist.destroy_process_group()


def step_times(log_path: str) -> dict:
    """{step: step_ms} from a reference stage log's WT_TELEM lines."""
    out = {}
    if not os.path.exists(log_path):
        return out
    with open(log_path, errors="replace") as f:
        for line in f:
            if line.startswith("WT_TELEM "):
                try:
                    d = json.loads(line[len("WT_TELEM "):])
                except ValueError:
                    continue
                if "step" in d and "step_ms" in d:
                    out[int(d["step"])] = float(d["step_ms"])
    return out


def run_reference_arm(args) -> dict | None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    n = args.gpus
    if not os.path.isdir(os.path.join(REF, "wantrain")):
        return unavailable("the reference is not laid out in baseline/_ref")
    if world > 1 and rank != 0:
        _wait_for_rank0(world)
        return None
    import torch

    n_layer = args.n_layer or 48
    d, V, S = 5120, 50257, 2048
    params = V * d * 2 + S * d + n_layer * (12 * d * d + 13 * d) + 2 * d
    if n == 1:
        total = torch.cuda.get_device_properties(0).total_memory if torch.cuda.is_available() else 0
        need = 3 * 4 * params  # fp32 params + accumulated grads + one microbatch's grads
        if need > total:
            out = unavailable(
                f"the reference's single-device path holds fp32 parameters, the accumulated fp32 "
                f"gradients and one microbatch's fp32 gradients ({need / 1e9:.0f} GB for "
                f"{params / 1e9:.1f}B parameters) on one device of {total / 1e9:.0f} GB")
            if world > 1:
                _wait_for_rank0(world)
            return out
    if n_layer % n:
        return unavailable(f"{n_layer} layers do not split over {n} stages")
    sys.path.insert(0, REF)
    from wantrain.launch.local import run_local
    from wantrain.model.gpt import GPTConfig
    from wantrain.runtime.spec import JobSpec

    model = GPTConfig(vocab_size=V, n_layer=n_layer, n_head=40, d_model=d, seq_len=S,
                      compute_dtype="bf16", boundary_dtype="fp8_e4m3", attn_impl="sdpa",
                      sdpa_backend="flash")
    per = n_layer // n
    partition = [[0 if r == 0 else 1 + r * per, n_layer + 2 if r == n - 1 else 1 + (r + 1) * per]
                 for r in range(n)]
    out_dir = os.environ.get("EWB_REF_LOGDIR") or tempfile.mkdtemp(prefix="refbench-")
    os.makedirs(out_dir, exist_ok=True)
    stage_params = max((b - a) for a, b in partition) * 12 * d * d
    spec = JobSpec(model=model, stages=n, microbatches=args.microbatches, mb_size=args.mb_size,
                   steps=args.warmup + args.steps, device="cuda",
                   devices=[[f"cuda:{r}"] for r in range(n)], recompute=True, partition=partition,
                   optimizer="adamw-host" if stage_params * 16 > 120e9 else "adamw",
                   lr=1e-4, out_dir=out_dir, tag="refbench", port_base=_free_port(),
                   wire_codec="raw")
    t0 = time.time()
    res = run_local(spec, timeout=float(os.environ.get("EWB_REF_TIMEOUT_S", "3000")))
    wall = time.time() - t0
    if world > 1:
        import torch.distributed as dist
        import datetime

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
        dist.barrier()
        dist.destroy_process_group()
    if not res.get("ok"):
        first = []
        for r in range(n):
            lp = os.path.join(out_dir, f"refbench_r{r}p0.log")
            if os.path.exists(lp):
                with open(lp, errors="replace") as f:
                    errs = [ln for ln in f.read().splitlines()
                            if re.search(r"Error|error:|Traceback|WT_DONE", ln)]
                first.append(f"stage {r}: " + " | ".join(errs[-3:])[-240:])
        return unavailable(f"the reference run failed (rc {res.get('rc')}): " + " ;; ".join(first))
    timed = range(args.warmup, args.warmup + args.steps)
    per_stage = []
    for r in range(n):
        st = step_times(os.path.join(out_dir, f"refbench_r{r}p0.log"))
        if not all(s in st for s in timed):
            return unavailable(f"stage {r} reported no WT_TELEM step_ms for the timed steps")
        per_stage.append(sum(st[s] for s in timed))
    ms = max(per_stage)
    tokens = spec.microbatches * spec.mb_size * S
    value = tokens * args.steps / (ms / 1e3)
    out = {"impl": "reference", "metric": "tokens/s (8xB200, max over ranks) 15.8B GPT PP+ZeRO-1",
           "value": round(value, 1), "unit": "tokens/s", "n_gpus": n, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
           "scaling": "strong", "vs_baseline": round(value / 3344.0, 3), "dtype": "bf16",
           "data": "synthetic (seeded uniform token ids, random-init weights)",
           "config": {"model": f"reference GPTConfig {n_layer}L d{d} 40h seq{S} vocab{V} "
                               f"(fp8_e4m3 per-token boundaries, sdpa/flash, recompute)",
                      "global_batch": spec.microbatches * spec.mb_size, "seq_len": S,
                      "parallelism": f"pp{n}", "optimizer": spec.optimizer,
                      "timer": "reference WT_TELEM step_ms (host monotonic), max over stages"},
           "wall_s": round(wall, 1)}
    if args.n_layer:
        out["diagnostic"] = "reduced config: not the benchmark"
    return out
