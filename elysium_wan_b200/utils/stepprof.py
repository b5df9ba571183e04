"""One training step of a shallow model of the benchmark's width, for a launch
list of every kernel it runs (the small case an Nsight Compute capture wants).

    python -m elysium_wan_b200.utils.stepprof [--model gpt15b] [--n-layer 2]
        [--microbatches 2] [--warmup 3]

It builds one stage holding the whole model (embedding, n_layer blocks, head)
on cuda:0, runs the warm-up steps, then one step inside an NVTX range named
"prof", so a capture can keep exactly that step's kernels:

    ncu --nvtx --nvtx-include "prof/" --metrics gpu__time_duration.sum \
        --clock-control none --csv --log-file launches.csv \
        python -m elysium_wan_b200.utils.stepprof

Without a profiler it prints the step's F / B / W op times (CUDA events).
"""

from __future__ import annotations

import argparse
import json
import tempfile

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="gpt15b")
    ap.add_argument("--n-layer", type=int, default=2)
    ap.add_argument("--microbatches", type=int, default=2)
    ap.add_argument("--mb-size", type=int, default=1)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    from elysium_wan_b200 import ops
    from elysium_wan_b200.models.config import make_config
    from elysium_wan_b200.runtime.engine import StageEngine
    from elysium_wan_b200.runtime.spec import JobSpec
    from elysium_wan_b200.utils.determinism import setup_determinism

    cfg = make_config(a.model, n_layer=a.n_layer)
    M = a.microbatches
    spec = JobSpec(model=cfg, stages=1, microbatches=M, mb_size=a.mb_size, steps=a.warmup + 1,
                   device="cuda", backend="nccl", lr=1e-4, out_dir=tempfile.gettempdir(),
                   tag="stepprof")
    spec.schedule_order = [[sum(([["F", mb], ["B", mb], ["W", mb]] for mb in range(M)), [])]]
    spec.finalize()
    setup_determinism(spec.init_seed)
    dev = torch.device("cuda", 0)
    ops.ext()
    eng = StageEngine(spec, 0, 0, None, dev)
    eng.warm_kernels()
    for s in range(a.warmup):
        eng.run_step(s)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("prof")
    eng.run_step(a.warmup)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ops_ms = {}
    for op, mb, start, dur in eng.op_times_ms():
        ops_ms.setdefault(op, []).append(round(dur, 3))
    print(json.dumps({"model": a.model, "n_layer": a.n_layer, "microbatches": M,
                      "op_ms": ops_ms, "phases": eng.phase_ms(),
                      "status": ops.ext().status_read_clear()}), flush=True)


if __name__ == "__main__":
    main()
