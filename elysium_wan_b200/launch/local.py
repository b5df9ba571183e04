"""Every slot of a job as its own OS process on this machine, plus the oracle
and the bitwise diff.

Reference: run_local / run_and_compare (src/wantrain/launch/local.py:399-503).
Slots are spawned as `python -m elysium_wan_b200.runtime.stage_main`; on the
first failure every other slot is killed (by its own PID). GPU slots get
LOCAL_RANK = their rank, so rank r runs on cuda:r.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
import time

from elysium_wan_b200.utils.determinism import pinned_env


def merge_losses(spec) -> str:
    from elysium_wan_b200.runtime.stage_main import loss_path

    recs = []
    last = spec.stages - 1
    for p in range(spec.stage_widths[last]):
        path = loss_path(spec, last, p)
        if os.path.exists(path):
            with open(path) as f:
                recs += json.load(f)["losses"]
    recs.sort(key=lambda r: (r["step"], r["mb"]))
    out = os.path.join(spec.out_dir, f"{spec.tag}_losses.json")
    with open(out, "w") as f:
        json.dump({"losses": recs}, f, indent=1)
    return out


def run_local(spec, timeout: float = 1800.0, log_dir: str | None = None, extra_env=None) -> str:
    spec.finalize()
    os.makedirs(spec.out_dir, exist_ok=True)
    spec_path = os.path.join(spec.out_dir, f"{spec.tag}_spec.json")
    with open(spec_path, "w") as f:
        f.write(spec.to_json())
    env = pinned_env()
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    env["PYTHONPATH"] = root + os.pathsep + env.get("PYTHONPATH", "")
    # Load every kernel at context creation: a module loaded lazily while an
    # NCCL receive is pending can wait on that receive (cross-rank deadlock).
    env.setdefault("CUDA_MODULE_LOADING", "EAGER")
    # shared WAN budgets (NIC, uplink) of this run live in one directory
    env["EWB_PACER_DIR"] = os.path.join(os.path.abspath(spec.out_dir), ".pacers")
    if extra_env:
        env.update(extra_env)
    procs = []
    log_dir = log_dir or spec.out_dir
    for r, w in enumerate(spec.stage_widths):
        for p in range(w):
            rank = spec.rank_of(r, p)
            e = dict(env)
            e["LOCAL_RANK"] = str(rank)
            log = open(os.path.join(log_dir, f"{spec.tag}_r{r}p{p}.log"), "w")
            cmd = [sys.executable, "-m", "elysium_wan_b200.runtime.stage_main", "--spec", spec_path,
                   "--rank", str(r), "--peer", str(p), "--timeout", str(min(timeout, 600.0))]
            procs.append((subprocess.Popen(cmd, stdout=log, stderr=subprocess.STDOUT, env=e), log))
    t0 = time.time()
    failed = None
    while True:
        codes = [pr.poll() for pr, _ in procs]
        if any(c not in (None, 0) for c in codes):
            failed = [i for i, c in enumerate(codes) if c not in (None, 0)]
            break
        if all(c == 0 for c in codes):
            break
        if time.time() - t0 > timeout:
            failed = "timeout"
            break
        time.sleep(0.05)
    if failed is not None:
        for pr, _ in procs:
            if pr.poll() is None:
                pr.kill()
        for pr, log in procs:
            pr.wait()
            log.close()
        raise RuntimeError(f"local run failed ({failed}); logs in {log_dir}")
    for _, log in procs:
        log.close()
    return merge_losses(spec)


def ensure_reference(spec, tag: str = "reference") -> str:
    from elysium_wan_b200.validation.reference import run_baseline

    path = os.path.join(spec.out_dir, f"{tag}_losses.json")
    if not os.path.exists(path):
        run_baseline(spec, tag)
    return path


def run_and_compare(spec, timeout: float = 1800.0) -> dict:
    from elysium_wan_b200.validation.compare import compare

    got = run_local(spec, timeout)
    ref = ensure_reference(spec)
    return compare(ref, got)
