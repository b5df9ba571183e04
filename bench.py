#!/usr/bin/env python
"""Headline benchmark: whole-job tokens/s of the 15.8B GPT pipeline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P \
        bench.py --gpus N --steps K --warmup W

Config (BASELINE): dense GPT, 48 layers, d_model 5120, 40 heads, MLP 20480,
seq 2048, vocab 50257, bf16 compute, fp8 e4m3 1x128 boundaries, zero-bubble
schedule, 64 microbatches of 1 sequence per step (131,072 tokens), synthetic
seeded-uniform tokens and random-init weights. The SAME model and step run at
every N: N pipeline stages of 48/N layers (strong scaling). Memory plan per
stage: fp32 master + fp32 gradient + bf16 working copy on the device; AdamW
moments on the device when they fit, else in pinned host memory ("adamw-host",
the same kernel and bits); per-layer recompute only where a microbatch's
activations would not fit.

Timing: W untimed warm-up steps; then a barrier + cuda synchronize, CUDA
events on each rank's compute stream around exactly K steps, synchronize +
barrier, max over ranks. Every step's working set (GBs of weights) is larger
than L2. `e2e` times the same K steps on the host clock through the public
engine API, including each step's host->device copy of the token ids and
targets from pinned memory and the device->host read of the step's losses.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

# Every kernel is loaded when the CUDA context is created (before torch
# initialises CUDA): a module loaded lazily while an NCCL receive is pending can
# wait on that receive, a cross-rank deadlock.
if "reference" not in sys.argv:  # the reference arm runs the reference's own environment
    os.environ.setdefault("CUDA_MODULE_LOADING", "EAGER")

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

BASELINE_TOK_S = 3344.0  # the reference's published 15.8B GPT rate (2x H100 NVL over WAN, run 3)
METRIC = "tokens/s (8xB200, max over ranks) 15.8B GPT PP+ZeRO-1"
GiB = 1 << 30


def _env_rank():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    def __init__(self, gpus: list):
        self.gpus = gpus
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.flush()
        self.f.seek(0)
        mhz, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                idx = int(parts[0])
            except ValueError:
                continue
            if idx not in self.gpus:
                continue
            try:
                mhz.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                pass
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.f.name)
        return {"sm_mhz": statistics.median(mhz) if mhz else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(mhz)}


# model preset, microbatches x sequences per step, pipeline
# depth at 8 GPUs (the rest of the GPUs are ZeRO-1 replicas of each stage).
CONFIGS = {
    "15.8b": dict(model="gpt15b", microbatches=64, mb_size=1, stages=None, recompute=None,
                  metric=METRIC, shape="48L d5120 40h MLP20480 seq2048 vocab50257, fp8 e4m3 1x128 boundaries"),
    "0.6b": dict(model="gpt0_6b", microbatches=16, mb_size=4, stages=2, recompute=None,
                 metric="tokens/s (max over ranks) 0.6B GPT PP x ZeRO-1",
                 shape="20L d1536 12h MLP6144 seq2048 vocab50257, bf16 boundaries"),
    "2.8b": dict(model="gpt2_8b", microbatches=32, mb_size=2, stages=4, recompute=None,
                 metric="tokens/s (max over ranks) 2.8B GPT PP x ZeRO-1",
                 shape="32L d2560 32h MLP10240 seq2048 vocab50257, bf16 boundaries"),
    "25.1b": dict(model="gpt25b", microbatches=32, mb_size=1, stages=4, recompute=True,
                  metric="tokens/s (max over ranks) 25.1B GPT PP x ZeRO-1",
                  shape="60L d5888 46h MLP23552 seq2048 vocab50257, fp8 e4m3 1x128 boundaries, recompute"),
}


def layout(args, n: int) -> list:
    """Stage widths for N GPUs: --widths when given, else the config's depth
    (capped by N) with the remaining GPUs as ZeRO-1 replicas of every stage."""
    if args.widths:
        w = [int(x) for x in args.widths.split(",")]
        if sum(w) != n:
            raise SystemExit(f"--widths {args.widths} uses {sum(w)} GPUs, not {n}")
        return w
    depth = CONFIGS[args.config]["stages"]
    if depth is None:
        return [1] * n
    stages = min(depth, n)
    if n % stages:
        raise SystemExit(f"{n} GPUs do not split into {stages} stages of equal width")
    return [n // stages] * stages


def _numel(cfg, a: int, b: int) -> int:
    from elysium_wan_b200.models.gpt import entry_specs

    tot = 0
    for e in range(a, b):
        for s in entry_specs(cfg, e):
            k = 1
            for x in s.shape:
                k *= x
            tot += k
    return tot


def plan_spec(args, n: int, free_bytes: float | None):
    """The benchmark spec on N GPUs, with the per-slot memory plan."""
    from elysium_wan_b200.models.config import make_config
    from elysium_wan_b200.runtime.spec import JobSpec
    from elysium_wan_b200.scheduler import partition as part

    over = {"n_layer": args.n_layer} if getattr(args, "n_layer", None) else {}
    cfg = make_config(args.model, **over)
    widths = layout(args, n)
    stages = len(widths)
    spec = JobSpec(model=cfg, stages=stages, stage_widths=widths, microbatches=args.microbatches,
                   mb_size=args.mb_size, steps=args.warmup + args.steps, device="cuda",
                   backend="nccl", grad_sync=args.grad_sync, init_seed=1234, data_seed=5678,
                   lr=1e-4, out_dir=tempfile.gettempdir(), tag="bench")
    # Cost-aware contiguous cut (exact min-max DP over the per-entry FLOP
    # model: block h(72h + 12s), head 6hV, embedding 3h).
    spec.partition = part.proportional_partition(cfg, [float(w) for w in widths])
    # Largest slot decides the plan (all ranks must agree on the spec).
    biggest = max(_numel(cfg, a, b) for a, b in spec.partition)
    wmin = min(widths)
    cap = free_bytes if free_bytes else 178 * GiB
    # fp32 master + fp32 gradient + bf16 working copy on every replica; a
    # replica of a wide stage also holds the fused path's fp32 exchange slots
    # (one stage-sized buffer) and its shard of the moments.
    resident = biggest * (4 + 4 + 2) + (4 * biggest if wmin > 1 else 0)
    moments = 8 * biggest / wmin
    if resident + 8 * GiB > cap:
        raise SystemExit(f"{args.config} on {n} GPU(s): the largest stage's weights and gradients "
                         f"({resident / GiB:.0f} GiB) do not fit a {cap / GiB:.0f} GiB device; "
                         f"use more GPUs")
    host_adam = resident + moments > 0.80 * cap
    spec.optimizer = "adamw-host" if host_adam else "adamw"
    # With the moments on the device the activations fill what is left; keep a
    # tenth of the device free on top of the 8 GiB so the caching allocator
    # does not run into its retry path near the cap (seen at 2 stages:
    # 168.5 of 178 GiB, 18 retries per step).
    slack = 8 * GiB + (0 if host_adam else 0.10 * cap)
    budget = cap - resident - (0 if host_adam else moments) - slack
    # Width-1 stages of at most 12 layers fold the weight gradients of
    # microbatch pairs with one GEMM each (their W ops are deferred and memory
    # is ample); one device runs W inline in B, and 24-layer stages are short of
    # memory, where pairing would hold one more microbatch's W inputs.
    blocks = max(sum(1 for e in range(a, b) if 1 <= e <= cfg.n_layer) for a, b in spec.partition)
    spec.w_pair = stages > 1 and wmin == 1 and blocks <= 12 and not getattr(args, "no_w_pair", False)
    from elysium_wan_b200.scheduler.planner import stage_memory_model

    spec.peer_weights = [[1.0] * w for w in widths]
    forced = CONFIGS[args.config]["recompute"]
    spec.recompute = bool(forced)
    if n == 1:
        # Single device: F, B, W per microbatch (W inline in B); recompute if one
        # microbatch's activations do not fit.
        if not forced:
            f, _, _ = stage_memory_model(spec, 0)
            spec.recompute = f > budget
        spec.mb_owner = [[0] * spec.microbatches]
        spec.schedule_order = [[sum(([["F", mb], ["B", mb], ["W", mb]]
                                     for mb in range(spec.microbatches)), [])]]
    else:
        from elysium_wan_b200.scheduler.planner import default_schedule

        spec.zb_mem_mode = "auto"
        spec.mb_owner = None
        spec.finalize()  # ownership (IWRR over each stage's replicas)
        try:
            spec.schedule_order = default_schedule(spec, [budget] * stages)
        except ValueError:  # one microbatch does not fit without recompute
            spec.recompute = True
            spec.schedule_order = default_schedule(spec, [budget] * stages)
        if spec.recompute:
            # stages whose in-flight activations fit keep F's tensors
            from elysium_wan_b200.scheduler.zero_bubble import selective_recompute

            spec.recompute_stages = selective_recompute(spec, budget_bytes=[budget] * stages)
    spec.finalize()
    return spec


def run_ours(args) -> dict | None:
    import torch
    import torch.distributed as dist

    from elysium_wan_b200 import ops
    from elysium_wan_b200.parallel.p2p import PipeComm
    from elysium_wan_b200.runtime.engine import StageEngine
    from elysium_wan_b200.runtime.stage_main import init_group
    from elysium_wan_b200.utils.determinism import setup_determinism

    rank, world, local = _env_rank()
    n = args.gpus
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}: launch N>1 with torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ops.ext()
    free, _ = torch.cuda.mem_get_info(dev)
    if world > 1:
        os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "1")
    spec = plan_spec(args, n, float(free))
    # W GEMMs on a side stream need memory headroom (deferred frees); a stage
    # that keeps its AdamW moments on the host has none.
    os.environ.setdefault("EWB_W_STREAM", "0" if spec.optimizer == "adamw-host" else "1")
    setup_determinism(spec.init_seed)
    init_group(spec, rank, timeout_s=float(os.environ.get("EWB_PG_TIMEOUT_S", "600")))
    stage, peer = spec.slot_of(rank)
    eng = StageEngine(spec, stage, peer, None, dev)
    eng.log = lambda line: print(f"[bench] rank {rank}: {line}", file=sys.stderr, flush=True)
    eng.warm_kernels()
    comm = PipeComm(spec, stage, peer, dev) if world > 1 else None
    eng.attach_comm(comm)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for s in range(args.warmup):
        t = time.perf_counter()
        eng.run_step(s)
        torch.cuda.synchronize()
        if rank == 0:
            ms = torch.cuda.memory_stats()
            print(f"[bench] warm-up step {s}: {time.perf_counter() - t:.2f} s "
                  f"(max alloc {torch.cuda.max_memory_allocated() / 2**30:.1f} GiB, "
                  f"alloc retries {ms.get('num_alloc_retries', 0)}, phases {eng.phase_ms()})",
                  file=sys.stderr, flush=True)
    torch.cuda.synchronize()
    st = ops.ext().status_read_clear()
    if st != 0:
        raise RuntimeError(f"device status word {st} after warm-up")
    barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(list(range(n))) if local == 0 else None
    l0 = ops.launch_count()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    for s in range(args.warmup, args.warmup + args.steps):
        eng.run_step(s)
    e1.record()
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    barrier()
    launches = ops.launch_count() - l0
    clocks = sampler.stop() if sampler else None
    dev_ms = e0.elapsed_time(e1)
    wall_ms = (t1 - t0) * 1e3
    busy = None
    ot = eng.op_times_ms()
    if ot:
        from elysium_wan_b200.runtime.telemetry import summarize_step

        summ = summarize_step(0, rank, 0, 0.0, ot, 0, 0)
        busy = summ["busy_frac"]
        # Per-rank diagnostics of the last timed step (stderr): busy fraction
        # of the op span, op medians, ops / optimizer phase split.
        print("[bench] rank %d: %s" % (rank, json.dumps(
            {"busy_frac": busy, "busy_ms": summ["busy_ms"], "ops": summ.get("ops"),
             "phases": eng.phase_ms()})), file=sys.stderr, flush=True)
    ph = eng.phase_ms()
    vec = torch.tensor([dev_ms, wall_ms, float(launches), busy or 0.0, busy or 2.0,
                        ph.get("ops_ms", 0.0), ph.get("opt_ms", 0.0)],
                       dtype=torch.float64, device=dev)
    if world > 1:
        mx = vec.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = vec.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        mn = vec.clone()
        dist.all_reduce(mn, op=dist.ReduceOp.MIN)
        dev_ms, wall_ms = mx[0].item(), mx[1].item()
        launches = int(sm[2].item())
        busy_min = mn[4].item()
        ops_ms, opt_ms = mx[5].item(), mx[6].item()
    else:
        busy_min = busy
        ops_ms, opt_ms = ph.get("ops_ms", 0.0), ph.get("opt_ms", 0.0)
    st = ops.ext().status_read_clear()
    losses = [v for _, _, v in eng.losses[-spec.microbatches:]] if eng.last else []
    if comm is not None:
        comm.close()
    if world > 1:
        dist.destroy_process_group()
    if st != 0:
        raise RuntimeError(f"device status word {st} after the timed steps")
    if rank != 0:
        return None
    tokens = spec.microbatches * spec.mb_size * spec.model.seq_len
    value = tokens * args.steps / (dev_ms / 1e3)
    e2e = tokens * args.steps / (wall_ms / 1e3)
    h2d = spec.microbatches * spec.mb_size * spec.model.seq_len * 8 * 2
    conf = CONFIGS[args.config]
    widths = spec.stage_widths
    par = f"pp{spec.stages}" + (f"xdp{widths[0]}" if len(set(widths)) == 1 and widths[0] > 1
                                else ("" if max(widths) == 1 else " widths " + ",".join(map(str, widths))))
    return {
        "metric": conf["metric"], "value": round(value, 1), "unit": "tokens/s", "n_gpus": n,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 3),
        "higher_is_better": True, "scaling": "strong",
        "vs_baseline": round(value / BASELINE_TOK_S, 3), "dtype": "bf16",
        "data": "synthetic (seeded uniform token ids, random-init weights)",
        "config": {"model": f"{args.model} ({conf['shape']})",
                   "global_batch": spec.microbatches * spec.mb_size, "seq_len": spec.model.seq_len,
                   "parallelism": par, "partition": spec.partition,
                   "grad_sync": spec.grad_sync if max(widths) > 1 else None,
                   "microbatches": spec.microbatches,
                   "schedule": "zero-bubble", "optimizer": spec.optimizer,
                   "recompute": spec.recompute, "w_pair": spec.w_pair,
                   "l2": "working set larger than L2 (no flush)"},
        "clocks": clocks,
        "e2e": {"value": round(e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": spec.microbatches * 4},
        "gpu_launches": launches,
        "busy_frac_min_over_stages": None if busy_min is None else round(busy_min, 4),
        # The last timed step split at its last op (max over ranks): the F/B/W
        # span and the optimizer / parameter-exchange phase after it, and the
        # tokens/s of the F/B/W span alone (comparable across N whatever the
        # optimizer placement, e.g. host moments at N = 1).
        "phases": {"ops_ms": round(ops_ms, 2), "opt_ms": round(opt_ms, 2),
                   "ops_only_tokens_per_s": round(tokens / (ops_ms / 1e3), 1) if ops_ms else None},
        "last_losses": losses[:4],
    }


def run_reference(args) -> dict:
    from elysium_wan_b200.utils.refbench import run_reference_arm

    args.ref_widths = layout(args, args.gpus)
    return run_reference_arm(args)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="15.8b", choices=sorted(CONFIGS),
                    help="BASELINE config (the headline is 15.8b)")
    ap.add_argument("--widths", default=None,
                    help="comma-separated replicas per stage (default: the config's layout)")
    ap.add_argument("--grad-sync", default="fused", choices=["fused", "nccl"],
                    help="ZeRO-1 gradient/parameter exchange of wide stages: fused into the "
                         "kernels over NVLink peer memory, or NCCL collectives")
    ap.add_argument("--microbatches", type=int, default=None)
    ap.add_argument("--mb-size", type=int, default=None)
    # Diagnostics only (profiling on a shallower model of the same width): a
    # line printed with it is marked "diagnostic" and is not the benchmark.
    ap.add_argument("--n-layer", type=int, default=None)
    ap.add_argument("--no-w-pair", action="store_true",
                    help="fold every microbatch's weight gradient on its own")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    conf = CONFIGS[args.config]
    args.model = conf["model"]
    args.metric = conf["metric"]
    reduced = args.microbatches not in (None, conf["microbatches"]) or \
        args.mb_size not in (None, conf["mb_size"])
    args.microbatches = args.microbatches or conf["microbatches"]
    args.mb_size = args.mb_size or conf["mb_size"]
    ref_model = {"15.8b": "gpt15b", "0.6b": "gpt0p6b", "2.8b": "gpt2p8b", "25.1b": "gpt25b"}
    args.ref_model = ref_model[args.config]
    args.widths_list = [int(x) for x in args.widths.split(",")] if args.widths else None
    if args.impl == "reference":
        out = run_reference(args)
    else:
        out = run_ours(args)
    if out is not None:
        if args.n_layer or reduced:
            out["diagnostic"] = "reduced config: not the benchmark"
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
