#!/usr/bin/env python
"""The CPU plumbing configuration, end to end, with a worker lost mid-run.

Defaults reproduce BASELINE config 1: a dense GPT decoder (8 layers, d_model
256, 4 heads, MLP 4x, GELU, pre-LN, learned positions, vocab 50257, seq 128,
fp32) cut into 4 pipeline stages of 2 layers, run by 5 worker agents (one
spare) in two emulated regions joined by a 60 Mb/s, 60 ms RTT link; 4
microbatches of 2 sequences per step for 60 steps (240 losses); synthetic
tokens from seed 0. One worker is killed at step 6; the coordinator convicts
it, moves its slot to the spare, restores the slot's newest checkpoint wave
there, relaunches every stage, and the final 240 losses are compared bit for
bit with the single-device oracle.

    python examples/wan_cluster_demo.py [--workers 5 --stages 4 --kill-at 6 --steps 60]
"""

import argparse
import json
import os
import sys
import tempfile
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from elysium_wan_b200.control.coordinator import Job  # noqa: E402
from elysium_wan_b200.launch.cluster import LocalCluster  # noqa: E402
from elysium_wan_b200.models.config import make_config  # noqa: E402
from elysium_wan_b200.runtime.spec import JobSpec  # noqa: E402
from elysium_wan_b200.validation.compare import compare  # noqa: E402
from elysium_wan_b200.validation.reference import run_baseline  # noqa: E402


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--workers", type=int, default=5)
    ap.add_argument("--stages", type=int, default=4)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--microbatches", type=int, default=4)
    ap.add_argument("--mb-size", type=int, default=2)
    ap.add_argument("--kill-at", type=int, default=6)
    ap.add_argument("--kill-stage", type=int, default=2)
    ap.add_argument("--n-layer", type=int, default=8)
    ap.add_argument("--vocab", type=int, default=50257)
    ap.add_argument("--wan", default="60mbps:60ms")
    ap.add_argument("--ckpt-every", type=int, default=2)
    ap.add_argument("--workdir", default=None)
    a = ap.parse_args(argv)
    from elysium_wan_b200.cli import parse_wan_profile

    workdir = a.workdir or tempfile.mkdtemp(prefix="wan-demo-")
    half = (a.workers + 1) // 2
    regions = ["us-east"] * (a.workers - half) + ["eu-central"] * half
    cfg = make_config("cpu_plumbing", n_layer=a.n_layer, vocab_size=a.vocab)
    spec = JobSpec(model=cfg, stages=a.stages, microbatches=a.microbatches, mb_size=a.mb_size,
                   steps=a.steps, init_seed=0, data_seed=0, lr=1e-3, ckpt_every=a.ckpt_every,
                   backend="gloo", tag="demo")
    t0 = time.time()
    cl = LocalCluster(workdir, regions, wan_links={"eu-central|us-east": parse_wan_profile(a.wan)})
    killed = {}

    def on_progress(slot, step, nid):
        if not killed and step >= a.kill_at:
            name = cl.worker_of_slot((a.kill_stage, 0))
            killed["worker"] = name
            killed["step"] = step
            print(f"[demo] killing worker {name} (stage {a.kill_stage}) at step {step}", flush=True)
            cl.kill_worker(name)

    cl.coord.on_progress = on_progress
    try:
        res = cl.run(Job(spec=spec))
    finally:
        cl.close()
    wall = time.time() - t0
    print(f"[demo] run ok={res.ok} attempts={res.attempts} heals={res.heals} in {wall:.1f}s", flush=True)
    if not res.ok:
        print(f"[demo] failed: {res.why}")
        return 1
    ref_spec = JobSpec.from_dict(spec.to_dict())
    ref_spec.out_dir = os.path.join(workdir, "oracle")
    ref_spec.finalize()
    ref = run_baseline(ref_spec, "reference")
    r = compare(ref, res.losses_path)
    out = {"compared": r["compared"], "mismatches": r["mismatches"], "ok": r["ok"], "heals": res.heals,
           "killed": killed, "wall_s": round(wall, 1), "run_dir": res.run_dir}
    print("WT_DEMO " + json.dumps(out), flush=True)
    return 0 if r["ok"] else 1


if __name__ == "__main__":
    sys.exit(main())
