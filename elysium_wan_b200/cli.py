"""`wantrain` command line (same subcommands and flags as the reference,
src/wantrain/cli.py:203-346).

  wantrain coordinator --port 28000 --job job.json      control plane, runs one job
  wantrain worker --coordinator HOST:28000 --coordinator-id ID --advertise-host IP
  wantrain stage --spec spec.json --rank R [--peer P]    one slot, no control plane
  wantrain local --spec spec.json [--compare]            every slot on this machine
  wantrain plan --fleet fleet.json --out spec.json       planner only
  wantrain reference --spec spec.json                    single-device oracle
  wantrain compare A_losses.json B_losses.json           bitwise diff
  wantrain probe | fit | validate-model | prepare-data

A job file is {"spec": <JobSpec JSON>} or {"plan": <job description>, "stages": N}.
"""

from __future__ import annotations

import argparse
import json
import os
import sys


def _load_job(path: str):
    from elysium_wan_b200.control.coordinator import Job
    from elysium_wan_b200.runtime.spec import JobSpec

    with open(path) as f:
        d = json.load(f)
    if "spec" in d:
        return Job(spec=JobSpec.from_dict(d["spec"]))
    if "plan" in d:
        return Job(plan=d["plan"], stages=d.get("stages"))
    return Job(spec=JobSpec.from_dict(d))


def cmd_coordinator(a) -> int:
    import time

    from elysium_wan_b200.control.coordinator import Coordinator, CoordinatorConfig

    token = a.token or os.environ.get("WANTRAIN_COORD_TOKEN", "")
    cfg = CoordinatorConfig(state_dir=a.state_dir, token=token, wait_workers_s=a.wait_workers_s,
                            no_probe=a.no_probe, no_fit_check=a.no_fit_check, group_by=a.group_by,
                            allow_shared_hosts=a.allow_shared_hosts, any_region=a.any_region,
                            zb_mem_mode=a.zb_mem_mode, replacement_match=a.replacement_match,
                            max_heals=a.max_heals, keep_workers=a.keep_workers,
                            profile=not a.no_profile,
                            recut=not a.no_recut, replan=not a.no_replan,
                            recut_min_gain=a.recut_min_gain,
                            recut_cost_s=a.recut_cost_s, max_replans=a.max_replans,
                            watch_slow=not a.no_watch_slow, slow_ratio=a.slow_ratio,
                            slow_runs=a.slow_runs)
    if a.wan_link:
        for item in a.wan_link:
            key, _, prof = item.partition("=")
            cfg.wan_links[key] = parse_wan_profile(prof)
    c = Coordinator(a.host, a.port, cfg).start()
    print(f"COORDINATOR_LISTEN {a.host}:{c.port}", flush=True)
    try:
        if not a.job:
            while True:
                time.sleep(3600)
        res = c.run_job(_load_job(a.job))
        print(f"WT_RESULT {json.dumps(res.__dict__)}", flush=True)
        return 0 if res.ok else 1
    finally:
        c.stop()


def parse_wan_profile(s: str | None) -> dict:
    """"60mbps:60ms[:jitter_ms]" (round-trip latency) or a JSON object -> link dict."""
    if not s:
        return {}
    s = s.strip()
    if s.startswith("{"):
        return json.loads(s)
    parts = s.lower().split(":")
    out = {"bw_mbps": 0.0, "latency_ms": 0.0, "jitter_ms": 0.0}
    for p in parts:
        if p.endswith("mbps"):
            out["bw_mbps"] = float(p[:-4])
        elif p.endswith("ms") and out["latency_ms"] == 0.0:
            out["latency_ms"] = float(p[:-2]) / 2.0  # RTT -> one way
        elif p.endswith("ms"):
            out["jitter_ms"] = float(p[:-2])
    return out


def cmd_worker(a) -> int:
    from elysium_wan_b200.control.agent import WorkerAgent

    declare = json.loads(a.declare) if a.declare else {}
    w = WorkerAgent(a.coordinator, coordinator_id=a.coordinator_id, name=a.name,
                    workdir=a.workdir, device=a.device, region=a.region, wan_profile=a.wan_profile,
                    declare=declare, no_bench=a.no_bench, advertise_host=a.advertise_host,
                    probe_port=(a.probe_listen_port if a.probe_listen_port is not None
                                else a.probe_port))
    if a.probe_port is not None and a.probe_listen_port is not None:
        w.probe_port = a.probe_port  # advertised (a forwarded port), the server binds the other
    return w.run() or 0


def cmd_stage(a) -> int:
    from elysium_wan_b200.runtime import stage_main

    return stage_main.main(["--spec", a.spec, "--rank", str(a.rank), "--peer", str(a.peer)])


def cmd_local(a) -> int:
    from elysium_wan_b200.launch.local import run_and_compare, run_local
    from elysium_wan_b200.runtime.spec import JobSpec

    spec = JobSpec.load(a.spec)
    if a.out_dir:
        spec.out_dir = a.out_dir
    if a.compare:
        r = run_and_compare(spec, timeout=a.timeout)
        print(json.dumps(r, indent=2))
        return 0 if r["ok"] else 1
    print(run_local(spec, timeout=a.timeout))
    return 0


def cmd_plan(a) -> int:
    from elysium_wan_b200.resources.node import NodeInfo
    from elysium_wan_b200.scheduler.fleetplan import build_spec

    with open(a.fleet) as f:
        d = json.load(f)
    fleet = [NodeInfo.from_caps(n.get("name", f"n{i}"), n) for i, n in enumerate(d.get("nodes", []))]
    stages = d.get("stages") or d["plan"].get("stages")
    if stages is None and fleet:
        # plan mode: depth, widths, layout and microbatches chosen from the fleet
        from elysium_wan_b200.scheduler.fleetplan import plan_job

        try:
            spec, rationale = plan_job(d["plan"], fleet)
        except ValueError as e:
            print(f"WT_PLAN_REFUSED {json.dumps({'why': str(e)})}")
            return 1
    else:
        spec, rationale = build_spec(d["plan"], stages, fleet).finalize(), None
    with open(a.out, "w") as f:
        f.write(spec.to_json())
    print(f"WT_PLAN {json.dumps({'stages': spec.stages, 'partition': spec.partition, 'stage_widths': spec.stage_widths, 'shard': spec.shard, 'microbatches': spec.microbatches, 'rationale': rationale})}")
    return 0


def cmd_reference(a) -> int:
    from elysium_wan_b200.validation import reference

    return reference.main(["--spec", a.spec] + (["--tag", a.tag] if a.tag else []))


def cmd_compare(a) -> int:
    from elysium_wan_b200.validation.compare import main

    return main([a.a, a.b])


def cmd_probe(a) -> int:
    from elysium_wan_b200.resources.probe import measure

    print(json.dumps(measure(a.device, bench=a.bench), indent=2))
    return 0


def cmd_fit(a) -> int:
    from elysium_wan_b200.resources.fit import measure
    from elysium_wan_b200.runtime.spec import JobSpec

    spec = JobSpec.load(a.spec).finalize()
    r = measure(spec, a.rank, a.device)
    print(f"WT_FIT {json.dumps(r)}")
    return 0 if r["fits"] else 1


def cmd_validate_model(a) -> int:
    from elysium_wan_b200.validation.model_contract import validate

    with open(a.source) as f:
        r = validate(f.read(), json.loads(a.target))
    print(json.dumps(r, indent=2))
    return 0 if r["ok"] else 1


def cmd_prepare_data(a) -> int:
    from elysium_wan_b200.models import dataset as ds

    m = ds.prepare(a.corpus, a.out, tokenizer=a.tokenizer, source_type=a.source_type,
                   text_key=a.text_key, n_shards=a.shards, limit_tokens=a.limit_tokens)
    print("WT_CORPUS " + json.dumps(m))
    return 0


def cmd_import_hf(a) -> int:
    """A Hugging Face checkpoint (Llama family or GPT-2) -> a job spec whose
    model is the matching built-in decoder, initialised from the checkpoint."""
    from elysium_wan_b200.models import hf
    from elysium_wan_b200.runtime.spec import JobSpec

    cfg, _ = hf.import_checkpoint(a.path, seq_len=a.seq_len,
                                  compute_dtype=a.compute_dtype, boundary_dtype=a.boundary_dtype)
    spec = JobSpec(model=cfg, stages=a.stages, init_from=os.path.abspath(a.path),
                   init_sha256=hf.checkpoint_digest(a.path), device=a.device,
                   backend="nccl" if a.device.startswith("cuda") else "gloo")
    spec.finalize()
    with open(a.out, "w") as f:
        f.write(spec.to_json())
    print("WT_IMPORT " + json.dumps({"out": a.out, "params": cfg.n_params(),
                                     "init_sha256": spec.init_sha256}))
    return 0


def cmd_recut(a) -> int:
    """Move a width-1 chain's waves to another partition (resume with the new spec)."""
    from elysium_wan_b200.fault_tolerance.recut import recut
    from elysium_wan_b200.runtime.spec import JobSpec

    old = JobSpec.load(a.spec).finalize()
    new = JobSpec.load(a.new_spec).finalize()
    step = recut(old, new, a.step)
    print("WT_RECUT " + json.dumps({"step": step, "from": old.partition, "to": new.partition}))
    return 0


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="wantrain")
    sub = ap.add_subparsers(dest="cmd", required=True)

    c = sub.add_parser("coordinator", help="control plane: run one job over worker agents")
    c.add_argument("--host", default="127.0.0.1")
    c.add_argument("--port", type=int, default=28000)
    c.add_argument("--state-dir", default="coordinator_state")
    c.add_argument("--token", default=None)
    c.add_argument("--job", default=None)
    c.add_argument("--wait-workers-s", type=float, default=120.0)
    c.add_argument("--no-probe", action="store_true")
    c.add_argument("--no-fit-check", action="store_true")
    c.add_argument("--group-by", default="region")
    c.add_argument("--allow-shared-hosts", action="store_true")
    c.add_argument("--any-region", action="store_true")
    c.add_argument("--zb-mem-mode", default="auto", choices=["auto", "2p", "1p", "given"])
    c.add_argument("--replacement-match", default="any", choices=["any", "device", "model"])
    c.add_argument("--max-heals", type=int, default=3)
    c.add_argument("--keep-workers", action="store_true")
    c.add_argument("--wan-link", action="append", help="regionA|regionB=60mbps:60ms")
    c.add_argument("--no-profile", action="store_true",
                   help="keep the analytic schedule (no F/B/W profile of the slots before launch)")
    c.add_argument("--no-recut", action="store_true", help="never re-cut from telemetry")
    c.add_argument("--no-replan", action="store_true",
                   help="never re-solve the zero-bubble order from telemetry")
    c.add_argument("--recut-min-gain", type=float, default=0.05)
    c.add_argument("--recut-cost-s", type=float, default=60.0)
    c.add_argument("--max-replans", type=int, default=2)
    c.add_argument("--no-watch-slow", action="store_true", help="do not act on slow slots")
    c.add_argument("--slow-ratio", type=float, default=1.3)
    c.add_argument("--slow-runs", type=int, default=3)
    c.set_defaults(fn=cmd_coordinator)

    w = sub.add_parser("worker", help="worker agent: supervises one stage process")
    w.add_argument("--coordinator", required=True)
    w.add_argument("--coordinator-id", default="")
    w.add_argument("--advertise-host", default="127.0.0.1")
    w.add_argument("--data-port", type=int, default=29000)
    w.add_argument("--listen-port", type=int, default=None)
    w.add_argument("--probe-port", type=int, default=None,
                   help="serve link probes on this port (the coordinator's probe matrix and "
                        "chain routing need one on every worker)")
    w.add_argument("--probe-listen-port", type=int, default=None)
    w.add_argument("--name", default=None)
    w.add_argument("--workdir", default="worker")
    w.add_argument("--device", default="cpu")
    w.add_argument("--region", default="default")
    w.add_argument("--wan-profile", default=None,
                   help="region-pair link model for this worker's probes: a JSON file (or the "
                        "JSON itself) {\"intra\": {...}, \"inter\": {...}, \"pairs\": "
                        "{\"A|B\": {\"mbps\": .., \"rtt_ms\": ..}}}")
    w.add_argument("--declare", default=None)
    w.add_argument("--no-bench", action="store_true")
    w.set_defaults(fn=cmd_worker)

    s = sub.add_parser("stage", help="run one slot (no control plane)")
    s.add_argument("--spec", required=True)
    s.add_argument("--rank", type=int, required=True)
    s.add_argument("--peer", type=int, default=0)
    s.set_defaults(fn=cmd_stage)

    lo = sub.add_parser("local", help="every slot on this machine (+ oracle diff)")
    lo.add_argument("--spec", required=True)
    lo.add_argument("--out-dir", default=None)
    lo.add_argument("--compare", action="store_true")
    lo.add_argument("--timeout", type=float, default=1800.0)
    lo.set_defaults(fn=cmd_local)

    p = sub.add_parser("plan", help="planner only: fleet JSON -> spec JSON")
    p.add_argument("--fleet", required=True)
    p.add_argument("--out", required=True)
    p.set_defaults(fn=cmd_plan)

    r = sub.add_parser("reference", help="single-device oracle run")
    r.add_argument("--spec", required=True)
    r.add_argument("--tag", default=None)
    r.set_defaults(fn=cmd_reference)

    cm = sub.add_parser("compare", help="bitwise diff of two loss files")
    cm.add_argument("a")
    cm.add_argument("b")
    cm.set_defaults(fn=cmd_compare)

    pr = sub.add_parser("probe", help="measure this machine")
    pr.add_argument("--device", default="cpu")
    pr.add_argument("--bench", action="store_true")
    pr.set_defaults(fn=cmd_probe)

    fi = sub.add_parser("fit", help="fit-check one stage of a spec")
    fi.add_argument("--spec", required=True)
    fi.add_argument("--rank", type=int, default=0)
    fi.add_argument("--device", default="cpu")
    fi.set_defaults(fn=cmd_fit)

    vm = sub.add_parser("validate-model", help="check a build(cfg) model file")
    vm.add_argument("--source", required=True)
    vm.add_argument("--target", default="{}")
    vm.set_defaults(fn=cmd_validate_model)

    pd = sub.add_parser("prepare-data", help="tokenise a corpus into a token stream")
    pd.add_argument("--corpus", required=True)
    pd.add_argument("--out", required=True)
    pd.add_argument("--tokenizer", default="gpt2")
    pd.add_argument("--source-type", default="auto")
    pd.add_argument("--text-key", default="text")
    pd.add_argument("--shards", type=int, default=1)
    pd.add_argument("--limit-tokens", type=int, default=None)
    pd.set_defaults(fn=cmd_prepare_data)

    ih = sub.add_parser("import-hf", help="HF checkpoint (Llama / GPT-2) -> job spec")
    ih.add_argument("--path", required=True)
    ih.add_argument("--out", required=True)
    ih.add_argument("--seq-len", type=int, default=None)
    ih.add_argument("--stages", type=int, default=1)
    ih.add_argument("--device", default="cpu")
    ih.add_argument("--compute-dtype", default="fp32")
    ih.add_argument("--boundary-dtype", default="fp32")
    ih.set_defaults(fn=cmd_import_hf)

    rc = sub.add_parser("recut", help="move checkpoint waves to another stage partition")
    rc.add_argument("--spec", required=True, help="the spec the waves were written under")
    rc.add_argument("--new-spec", required=True, help="the spec to resume under")
    rc.add_argument("--step", type=int, default=None)
    rc.set_defaults(fn=cmd_recut)
    return ap


def main(argv=None) -> int:
    a = build_parser().parse_args(argv)
    return int(a.fn(a) or 0)


if __name__ == "__main__":
    sys.exit(main())
