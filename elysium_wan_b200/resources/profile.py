"""F / B / W profiler: times one stage's ops on its own device exactly as the
engine runs them (median after warm-up, CUDA events on the GPU).
Reference: src/wantrain/resources/profile.py:58-195."""

from __future__ import annotations

import statistics
import time

import torch


def profile_stage(spec, stage: int, device: str = "cpu", reps: int = 3) -> dict:
    from elysium_wan_b200.models.data import make_batch
    from elysium_wan_b200.models.gpt import Act
    from elysium_wan_b200.runtime.engine import StageEngine

    dev = torch.device(device if device != "cuda" else "cuda:0")
    eng = StageEngine(spec, stage, 0, None, dev)
    T = spec.mb_size * spec.model.seq_len
    cuda = dev.type == "cuda"

    def clock():
        if cuda:
            torch.cuda.synchronize(dev)
        return time.perf_counter()

    ts = {"F": [], "B": [], "W": []}
    for r in range(reps + 1):
        x, t = make_batch(spec.data_seed, 0, r, spec.mb_size, spec.model.seq_len, spec.model.vocab_size)
        if eng.first:
            inp = x.to(dev)
        else:
            dt = torch.bfloat16 if cuda else torch.float32
            inp = Act(torch.randn(T, spec.model.d_model, device=dev).to(dt))
        t0 = clock()
        out, st = eng.model.forward(inp, t.to(dev) if eng.last else None)
        t1 = clock()
        dy = None if eng.last else torch.randn(T, spec.model.d_model, device=dev).to(
            torch.bfloat16 if cuda else torch.float32)
        tasks: list = []
        eng.model.backward(st, dy, tasks)
        t2 = clock()
        for tk in tasks:
            tk.run()
        t3 = clock()
        if r > 0:
            ts["F"].append(t1 - t0)
            ts["B"].append(t2 - t1)
            ts["W"].append(t3 - t2)
    return {k: statistics.median(v) for k, v in ts.items()}


def main(argv=None) -> int:
    """python -m elysium_wan_b200.resources.profile --spec s.json --stage R
    [--device cuda] [--reps 3]: prints one WT_PROFILE {stage, F, B, W} line
    (seconds per microbatch)."""
    import argparse
    import json

    from elysium_wan_b200.runtime.spec import JobSpec

    ap = argparse.ArgumentParser(prog="profile")
    ap.add_argument("--spec", required=True)
    ap.add_argument("--stage", type=int, required=True)
    ap.add_argument("--device", default="cpu")
    ap.add_argument("--reps", type=int, default=3)
    a = ap.parse_args(argv)
    spec = JobSpec.load(a.spec).finalize()
    r = profile_stage(spec, a.stage, a.device, a.reps)
    print("WT_PROFILE " + json.dumps({"stage": a.stage, **{k: round(v, 6) for k, v in r.items()}}),
          flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
