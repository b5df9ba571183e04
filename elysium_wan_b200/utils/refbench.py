"""Reference arm of bench.py: the UNMODIFIED reference (virgiliolrf/elysium-wan,
laid out in baseline/_ref) run through its own public API on the same config.

Path: rank 0 builds the reference's own JobSpec for the benchmark model (the
15.8B GPT by default: 48 layers, d 5120, 40 heads, seq 2048, vocab 50257,
bf16 compute, sdpa/flash attention, fp8 e4m3 boundaries -- the reference's
per-token-scaled recipe, the closest it has to the 1x128 block recipe), 64
microbatches of 1 sequence, the zero-bubble schedule, and the reference's
production flags (recompute on, 8 flows per hop). The cut is the reference's
own compute-balanced default (`JobSpec.default_partition`), one stage per GPU
(`devices`). It runs under the reference's single-machine launcher
`wantrain.launch.local.run_local` (one stage process per slot, its framed TCP
data plane over loopback), in a child process of its own session.

Wire codec: the reference's production flag is "planes" (its
`scheduler/production.py`), a lossless byte-plane codec of the boundary
dtype. For a scaled fp8 boundary the reference routes the lossless wire
through "fp8_planes", whose `encode_scaled_fp8` carries the fp8 bytes plus one
exponent per row (`runtime/stage.py` `_encode_body`); "planes" would cast the
scaled tensor to fp8 unscaled, and "raw" accepts only fp32 and int64
(`transport/framing.py` `tensor_payload`). So fp8 boundaries take
"fp8_planes" and every other boundary "planes".

Timing: each stage prints the reference's own WT_TELEM `step_ms` per step (host
monotonic clock; the reference has no device timer). The job's step time is
the max over stages of the sum over the K timed steps after W warm-up steps.
As soon as every stage has reported every timed step, the child's session is
ended: the reference's unconditional final checkpoint (the whole fp32 state,
about 24 GB per stage of the 15.8B model at 8 stages) is not part of the
measured work and would not fit the scratch disk at one stage.
"""

from __future__ import annotations

import json
import os
import re
import shutil
import signal
import socket
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF = os.path.join(ROOT, "baseline", "_ref")

# Benchmark models in the reference's GPTConfig terms.
REF_MODELS = {
    "gpt15b": dict(n_layer=48, n_head=40, d_model=5120, boundary_dtype="fp8_e4m3"),
    "gpt0p6b": dict(n_layer=20, n_head=12, d_model=1536, boundary_dtype="bf16"),
    "gpt2p8b": dict(n_layer=32, n_head=32, d_model=2560, boundary_dtype="bf16"),
    "gpt25b": dict(n_layer=60, n_head=46, d_model=5888, boundary_dtype="fp8_e4m3"),
}


def unavailable(why: str) -> dict:
    return {"impl": "reference", "unavailable": why}


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rendezvous(world: int, timeout_s: float):
    """All torchrun ranks meet once (gloo) after rank 0's reference run."""
    import datetime

    import torch.distributed as dist

    if world <= 1:
        return
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=timeout_s))
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


def _errors(out_dir: str, tag: str, slots) -> str:
    first = []
    for r, p in slots:
        lp = os.path.join(out_dir, f"{tag}_r{r}p{p}.log")
        if os.path.exists(lp):
            with open(lp, errors="replace") as f:
                errs = [ln for ln in f.read().splitlines()
                        if re.search(r"Error|error:|Traceback|WT_DONE", ln)]
            if errs:
                first.append(f"stage {r}.{p}: " + " | ".join(errs[-3:])[-240:])
    return " ;; ".join(first)


def reference_spec_kwargs(model: str, n: int, widths: list | None, steps: int, microbatches: int,
                          mb_size: int, n_layer: int | None, out_dir: str) -> dict:
    """Keyword arguments of the reference's JobSpec for one benchmark run
    (plain data, so the child process can rebuild it)."""
    m = dict(REF_MODELS[model])
    if n_layer:
        m["n_layer"] = n_layer
    widths = list(widths or [1] * n)
    stages = len(widths)
    d = m["d_model"]
    params = 50257 * d * 2 + 2048 * d + m["n_layer"] * (12 * d * d + 13 * d)
    per_stage = params / stages
    # The reference keeps fp32 params, grads and the two moments (16 B/param);
    # its own adamw-host holds the moments in host memory when that does not fit.
    optimizer = "adamw-host" if per_stage * 16 > 120e9 else "adamw"
    bdt = m.pop("boundary_dtype")
    return dict(
        model=dict(vocab_size=50257, seq_len=2048, compute_dtype="bf16", boundary_dtype=bdt,
                   attn_impl="sdpa", sdpa_backend="flash", **m),
        spec=dict(stages=stages, stage_widths=widths, microbatches=microbatches, mb_size=mb_size,
                  steps=steps, device="cuda", recompute=True, p2p_streams=8,
                  wire_codec="fp8_planes" if bdt.startswith("fp8") else "planes",
                  optimizer=optimizer, lr=1e-4, ckpt_every=0, out_dir=out_dir, tag="refbench",
                  port_base=_free_port()),
        n_gpus=n)


def _child(path: str) -> int:
    """Runs inside the child session: the reference's own launcher."""
    with open(path) as f:
        kw = json.load(f)
    sys.path.insert(0, REF)
    from wantrain.launch.local import run_local
    from wantrain.model.gpt import GPTConfig
    from wantrain.runtime.spec import JobSpec

    s = dict(kw["spec"])
    widths = s["stage_widths"]
    gpu = 0
    devices = []
    for w in widths:
        devices.append([f"cuda:{gpu + p}" for p in range(w)])
        gpu += w
    spec = JobSpec(model=GPTConfig(**kw["model"]), devices=devices, **s)
    res = run_local(spec, timeout=float(kw.get("timeout_s", 3600)))
    print("REFBENCH_RESULT " + json.dumps(res), flush=True)
    return 0 if res.get("ok") else 1


def _kill_session(p: subprocess.Popen):
    try:
        os.killpg(p.pid, signal.SIGKILL)
    except (ProcessLookupError, PermissionError):
        pass
    try:
        p.wait(timeout=60)
    except subprocess.TimeoutExpired:
        pass


def run_reference_arm(args) -> dict | None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    n = args.gpus
    # The run is stopped at this deadline (seconds from its launch), under the
    # driver's per-run limit; the timed steps finished by then are reported.
    wait_s = float(os.environ.get("EWB_REF_TIMEOUT_S", "780"))
    if not os.path.isdir(os.path.join(REF, "wantrain")):
        out = unavailable("the reference is not laid out in baseline/_ref")
        _rendezvous(world, wait_s + 600)
        return out if rank == 0 else None
    if rank != 0:
        _rendezvous(world, wait_s + 600)
        return None
    model = getattr(args, "ref_model", "gpt15b")
    if model not in REF_MODELS:
        _rendezvous(world, wait_s + 600)
        return unavailable(f"no reference recipe for model {model}")
    widths = getattr(args, "ref_widths", None)
    if widths is not None and sum(widths) != n:
        _rendezvous(world, wait_s + 600)
        return unavailable(f"stage widths {widths} do not use {n} GPUs")
    # The reference's out_dir (its stage logs, and the start of its final
    # checkpoint before the run is stopped) is a scratch directory; with
    # EWB_REF_LOGDIR set, only the logs are copied there afterwards.
    scratch = tempfile.mkdtemp(prefix="refbench-")
    kw = reference_spec_kwargs(model, n, widths, args.warmup + args.steps, args.microbatches,
                               args.mb_size, args.n_layer, scratch)
    kw["timeout_s"] = wait_s
    slots = [(r, p) for r, w in enumerate(kw["spec"]["stage_widths"]) for p in range(w)]
    kpath = os.path.join(scratch, "refbench_args.json")
    with open(kpath, "w") as f:
        json.dump(kw, f)
    env = dict(os.environ)
    env.pop("CUDA_MODULE_LOADING", None)
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT",
              "GROUP_RANK", "ROLE_RANK", "TORCHELASTIC_RUN_ID"):
        env.pop(k, None)
    child_log = open(os.path.join(scratch, "refbench_child.log"), "wb")
    t0 = time.time()
    # The child runs this file as a script, so nothing of this package (no
    # kernel library) is imported on the reference's path.
    p = subprocess.Popen([sys.executable, os.path.abspath(__file__), "--child", kpath],
                         cwd=ROOT, env=env, stdout=child_log, stderr=subprocess.STDOUT,
                         start_new_session=True)
    timed = list(range(args.warmup, args.warmup + args.steps))
    # Timing per slot; the step time of a stage is the slowest of its peers.
    result, partial = None, False
    try:
        while True:
            done = p.poll() is not None
            per_slot = {s: step_times(os.path.join(scratch, f"refbench_r{s[0]}p{s[1]}.log"))
                        for s in slots}
            if all(all(t in st for t in timed) for st in per_slot.values()):
                result = per_slot
                break
            if done:
                break
            if time.time() - t0 > wait_s:
                # Out of time: keep the timed steps that every stage finished.
                got = [t for t in timed if all(t in st for st in per_slot.values())]
                if got:
                    timed, result, partial = got, per_slot, True
                break
            time.sleep(2.0)
    finally:
        wall = time.time() - t0
        _kill_session(p)
        child_log.close()
    err = _errors(scratch, "refbench", slots)
    if result is None:
        why = "timed out" if p.returncode is None or wall > wait_s else f"exited (rc {p.returncode})"
        out = unavailable(f"the reference run {why} before every stage reported a timed step "
                          f"({wall:.0f} s): " + (err or "no error line in the stage logs"))
    else:
        ms = max(sum(st[t] for t in timed) for st in result.values())
        S = 2048
        tokens = kw["spec"]["microbatches"] * kw["spec"]["mb_size"] * S
        value = tokens * len(timed) / (ms / 1e3)
        m = kw["model"]
        layout = "x".join(str(w) for w in kw["spec"]["stage_widths"])
        out = {"impl": "reference", "metric": args.metric, "value": round(value, 1),
               "unit": "tokens/s", "n_gpus": n, "steps": len(timed), "warmup": args.warmup,
               "ms_per_step": round(ms / len(timed), 3), "higher_is_better": True,
               "scaling": "strong", "vs_baseline": round(value / 3344.0, 3), "dtype": "bf16",
               "data": "synthetic (seeded uniform token ids, random-init weights)",
               "config": {"model": f"reference GPTConfig {m['n_layer']}L d{m['d_model']} "
                                   f"{m['n_head']}h seq{S} vocab50257 ({m['boundary_dtype']} "
                                   f"boundaries, sdpa/flash, recompute)",
                          "global_batch": kw["spec"]["microbatches"] * kw["spec"]["mb_size"],
                          "seq_len": S, "parallelism": f"pp{len(kw['spec']['stage_widths'])}"
                          + (f" widths {layout}" if max(kw["spec"]["stage_widths"]) > 1 else ""),
                          "optimizer": kw["spec"]["optimizer"],
                          "wire_codec": kw["spec"]["wire_codec"],
                          "timer": "reference WT_TELEM step_ms (host monotonic), max over stages"},
               "e2e": {"value": round(value, 1), "unit": "tokens/s",
                       "note": "the reference's own per-step host clock through its launcher"},
               "wall_s": round(wall, 1),
               "note": "the run is stopped once every stage has reported the timed steps "
                       "(its final checkpoint is not part of the measured work)"}
        if partial:
            out["steps_requested"] = args.steps
            out["partial"] = (f"the reference needed more than {wait_s:.0f} s for {args.warmup} "
                              f"warm-up and {args.steps} timed steps; its rate is over the "
                              f"{len(timed)} timed steps every stage finished")
        if args.n_layer:
            out["diagnostic"] = "reduced config: not the benchmark"
    keep = os.environ.get("EWB_REF_LOGDIR")
    if keep:
        os.makedirs(keep, exist_ok=True)
        for name in os.listdir(scratch):
            if name.endswith((".log", ".json")) and os.path.getsize(os.path.join(scratch, name)) < (8 << 20):
                shutil.copy(os.path.join(scratch, name), os.path.join(keep, name))
    shutil.rmtree(scratch, ignore_errors=True)
    _rendezvous(world, 600)
    return out


if __name__ == "__main__":
    if len(sys.argv) == 3 and sys.argv[1] == "--child":
        sys.exit(_child(sys.argv[2]))
    raise SystemExit("usage: refbench.py --child <args.json>")
