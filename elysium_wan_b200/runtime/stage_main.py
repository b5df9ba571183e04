"""One slot (stage, peer) as its own OS process.

Reference: src/wantrain/worker/stage_main.py (run_stage; WT_* stdout markers;
`WT_DONE <rc>` always last). The process joins the job's torch.distributed
group (NCCL on GPUs, gloo on CPU; rank = stage-major slot index), builds its
StageEngine, resumes from its newest checkpoint wave when asked, runs the
steps and writes its losses.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys
import threading
import time
import traceback

import torch
import torch.distributed as dist


_PRINT_LOCK = threading.Lock()


def _print(tag: str, obj) -> None:
    # one marker per line even when the wave writer's thread prints too
    line = f"{tag} {json.dumps(obj) if not isinstance(obj, str) else obj}\n"
    with _PRINT_LOCK:
        sys.stdout.write(line)
        sys.stdout.flush()


class WaveWriter:
    """Commits checkpoint waves off the step (reference behaviour: its
    background wave commit, RUNTIME-I17): the step's state is copied at the
    step boundary, then a thread writes, fsyncs, hashes and renames the wave
    and only then announces it (WT_WAVE). One commit is in flight at a time.
    `wait()` returns when the commit in flight is done and raises its error,
    so a failed commit fails the run; a run that fails still waits for the
    commit of a step it finished, and reports its own error."""

    def __init__(self, spec, stage: int, peer: int):
        self.spec, self.stage, self.peer = spec, stage, peer
        self.thread: threading.Thread | None = None
        self.error: BaseException | None = None

    def submit(self, step: int, state: dict):
        from elysium_wan_b200.fault_tolerance import checkpoint as ckpt

        self.wait()

        def commit():
            try:
                path = ckpt.commit_wave(self.spec, self.stage, self.peer, step, state)
                _print("WT_WAVE", {"step": step, "dir": path})
            except BaseException as e:  # noqa: BLE001 - surfaced by wait()
                self.error = e

        self.thread = threading.Thread(target=commit, name=f"wave-{step}", daemon=True)
        self.thread.start()

    def wait(self):
        if self.thread is not None:
            self.thread.join()
            self.thread = None
        if self.error is not None:
            e, self.error = self.error, None
            raise RuntimeError(f"checkpoint wave commit failed: {e!r}") from e


def init_group(spec, rank: int, timeout_s: float):
    backend = "nccl" if spec.backend == "nccl" else "gloo"
    if spec.world_size == 1:
        return
    # Point-to-point ops are serialised per group by design (one group per hop
    # and direction); the warning about it is noise here.
    os.environ.setdefault("TORCH_NCCL_SHOW_EAGER_INIT_P2P_SERIALIZATION_WARNING", "false")
    if "MASTER_ADDR" in os.environ and "WORLD_SIZE" in os.environ:
        init = "env://"
    else:
        init = f"tcp://{spec.host}:{spec.port_base}"
    kw = {}
    if backend == "nccl":
        kw["device_id"] = torch.device("cuda", torch.cuda.current_device())
    dist.init_process_group(backend, init_method=init, rank=rank, world_size=spec.world_size,
                            timeout=datetime.timedelta(seconds=timeout_s), **kw)


def env_fingerprint(dev: str) -> dict:
    """What the run's numbers depend on besides the spec: versions, device,
    host (written once per run as <tag>_env.json)."""
    import platform

    fp = {"python": platform.python_version(), "torch": torch.__version__,
          "cuda": torch.version.cuda, "host": platform.node(), "device": dev}
    if dev.startswith("cuda") and torch.cuda.is_available():
        p = torch.cuda.get_device_properties(torch.device(dev))
        fp.update(gpu=p.name, sm=f"{p.major}.{p.minor}", gpu_mem_gib=round(p.total_memory / 2**30, 1),
                  nccl=".".join(map(str, torch.cuda.nccl.version())))
    fp["env"] = {k: v for k, v in os.environ.items()
                 if k.startswith(("EWB_", "NCCL_", "TORCH_NCCL", "CUDA_MODULE", "ELYSIUM_"))}
    return fp


def loss_path(spec, stage, peer) -> str:
    return os.path.join(spec.out_dir, f"{spec.tag}_losses_r{stage}p{peer}.json")


def _leaves_after(step: int, spec) -> bool:
    """EWB_TEST_LEAVE_AFTER_STEP=N (a failure-injection seam for tests, set on
    one worker): the first attempt's stage process exits right after step N."""
    v = os.environ.get("EWB_TEST_LEAVE_AFTER_STEP")
    return v is not None and not spec.resume and step == int(v)


def run_stage(spec, stage: int, peer: int, timeout_s: float = 600.0) -> int:
    from elysium_wan_b200.fault_tolerance import checkpoint as ckpt
    from elysium_wan_b200.parallel.p2p import PipeComm
    from elysium_wan_b200.runtime.engine import StageEngine
    from elysium_wan_b200.runtime.telemetry import summarize_step
    from elysium_wan_b200.utils.determinism import float_hex, setup_determinism
    from elysium_wan_b200.validation.reference import loss_records

    setup_determinism(spec.init_seed)
    rank = spec.rank_of(stage, peer)
    dev = spec.device_for(stage, peer)
    if dev.startswith("cuda"):
        local = int(os.environ.get("LOCAL_RANK", rank % max(1, torch.cuda.device_count())))
        dev = f"cuda:{local}" if dev == "cuda" else dev
        torch.cuda.set_device(torch.device(dev))
    _print("WT_PHASE", {"phase": "init", "stage": stage, "peer": peer, "rank": rank})
    if spec.dataset_path:
        # A data-reading slot verifies (and fetches) its shards before it connects.
        from elysium_wan_b200.models.provision import provision_slot

        rep = provision_slot(spec, stage, peer)
        if rep is not None:
            _print("WT_PHASE", {"phase": "provision", **rep})
    init_group(spec, rank, timeout_s)
    if spec.world_size == 1:
        comm = None
    elif spec.backend == "tcp":
        # Framed, sealed TCP between stages (runs across machines); the gloo
        # group still carries the collectives inside a wide stage.
        from elysium_wan_b200.transport.tcp import TcpPipeComm

        comm = TcpPipeComm(spec, stage, peer, torch.device(dev), timeout_s=timeout_s)
    else:
        comm = PipeComm(spec, stage, peer, torch.device(dev))
    eng = StageEngine(spec, stage, peer, comm, dev)
    _print("WT_STAGE", {"stage": stage, "peer": peer, "span": spec.partition[stage],
                        "params": eng.store.numel, "device": dev})
    _print("WT_OPT", {"optimizer": spec.optimizer, "trainable": eng.store.nt,
                      "frozen": eng.store.numel - eng.store.nt,
                      "zero1": type(eng.zero1).__name__ if eng.zero1 is not None else None})
    if spec.model.lora_rank:
        _print("WT_LORA", {"rank": spec.model.lora_rank, "targets": spec.model.lora_targets,
                           "adapted": len(eng.model.adapters), "trainable_params": eng.store.nt,
                           "frozen_params": eng.store.numel - eng.store.nt})
    if getattr(comm, "peers_seen", None):
        _print("WT_AEAD", {"cipher": "chacha20-poly1305", "peers": comm.peers_seen})
    if getattr(comm, "mesh", None) is not None:
        _print("WT_MESH", {"stage": stage, "peer": peer, "replicas": sorted(comm.mesh.links)})
    if getattr(comm, "tied_link", None) is not None:
        _print("WT_TIED_LINK", {"stage": stage, "peer": peer})
    if stage == 0 and peer == 0:
        os.makedirs(spec.out_dir, exist_ok=True)
        with open(os.path.join(spec.out_dir, f"{spec.tag}_env.json"), "w") as f:
            json.dump(env_fingerprint(dev), f, indent=1)
    start = 0
    if spec.resume:
        sd, step = ckpt.load_latest(spec, stage, peer, spec.resume_step)
        eng.load_state_dict(sd)
        start = step
        _print("WT_RESUME", {"step": step})
    # waves past the start belong to an abandoned timeline (all of them, on a
    # fresh launch), and a writer killed mid-commit leaves temporaries
    dropped = ckpt.drop_after(spec.out_dir, spec.tag, stage, peer, start if spec.resume else -1)
    if dropped:
        _print("WT_WAVES_DROPPED", {"steps": dropped})
    os.makedirs(spec.out_dir, exist_ok=True)
    stream = open(os.path.join(spec.out_dir, f"{spec.tag}_loss_stream.jsonl"), "a") if eng.last else None
    tel = open(os.path.join(spec.out_dir, f"{spec.tag}_rank{stage}p{peer}_telemetry.jsonl"), "a")
    net0 = (0, 0)
    t_run = time.perf_counter()
    waves = WaveWriter(spec, stage, peer)
    links0: dict = {}
    try:
        for step in range(start, spec.steps):
            t0 = time.perf_counter()
            res = eng.run_step(step)
            if eng.timing:
                torch.cuda.synchronize()
            dt = time.perf_counter() - t0
            for mb, v in res:
                rec = {"step": step, "mb": mb, "loss_hex": float_hex(v), "loss": v}
                if stream is not None:
                    stream.write(json.dumps(rec) + "\n")
                    stream.flush()
                _print("WT_METRIC", {"step": step, "mb": mb, "loss": v})
            links = None
            if hasattr(comm, "link_stats"):
                now = comm.link_stats()
                links = {k: {f: round(v[f] - links0.get(k, {}).get(f, 0), 3) for f in v}
                         for k, v in now.items()}
                links0 = now
            summary = summarize_step(step, stage, peer, dt * 1e3, eng.op_times_ms(),
                                     comm.bytes_sent if comm else 0, comm.frames if comm else 0,
                                     eng.phase_ms().get("opt_ms"), links)
            if "ops" not in summary:
                _print("WT_WARN", f"telemetry summary of step {step} exceeded 4096 bytes: its "
                                  "per-op medians were dropped")
            _print("WT_TELEM", summary)
            if eng.w_filled:
                _print("WT_WFILL", {"step": step, "tasks": eng.w_filled})
            tel.write(json.dumps({"step": step, "events": [[o, m, round(a, 4), round(d, 4)]
                                                            for o, m, a, d in eng.op_times_ms()]})
                      + "\n")
            tel.flush()
            if comm is not None:
                net = (comm.frames, comm.bytes_sent)
                _print("WT_NET", {"step": step, "frames": net[0] - net0[0],
                                  "bytes": net[1] - net0[1]})
                net0 = net
            if eng.timing:
                gib = 2.0 ** 30
                _print("WT_MEM", {"step": step,
                                  "max_alloc_gib": round(torch.cuda.max_memory_allocated() / gib, 3),
                                  "reserved_gib": round(torch.cuda.memory_reserved() / gib, 3)})
            if spec.ckpt_every and (step + 1) % spec.ckpt_every == 0:
                waves.submit(step + 1, eng.state_dict())
            _print("WT_STEP", {"step": step, "ms": round(dt * 1e3, 3)})
            if _leaves_after(step, spec):
                # Test seam: this process leaves between steps (its kernels and
                # collectives are complete, its wave committed), without a done
                # marker, as a rank whose machine went away would.
                waves.wait()
                sys.stdout.flush()
                os._exit(17)
    except BaseException:
        try:
            waves.wait()  # a step finished before the failure still becomes a wave
        except Exception as e:  # noqa: BLE001 - the run's own error is the one reported
            _print("WT_WARN", str(e))
        raise
    waves.wait()
    tel.close()
    n_run = spec.steps - start
    _print("WT_TIMING", {"steps": n_run, "total_s": round(time.perf_counter() - t_run, 3),
                         "mean_step_ms": round((time.perf_counter() - t_run) * 1e3 / max(1, n_run),
                                               3)})
    if eng.last:
        with open(loss_path(spec, stage, peer), "w") as f:
            json.dump({"losses": loss_records(eng.losses)}, f, indent=1)
        if spec.stage_widths[-1] == 1:
            # a single last peer also writes the reference's file name
            # (src/wantrain/runtime/stage.py:3558-3571); wide last stages are
            # merged by the launcher or the coordinator
            with open(os.path.join(spec.out_dir, f"{spec.tag}_losses.json"), "w") as f:
                json.dump({"losses": loss_records(eng.losses)}, f, indent=1)
    if comm is not None:
        comm.close()
    if spec.world_size > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main(argv=None) -> int:
    from elysium_wan_b200.runtime.spec import JobSpec

    ap = argparse.ArgumentParser(prog="wantrain stage")
    ap.add_argument("--spec", required=True)
    ap.add_argument("--rank", type=int, required=True, help="stage index")
    ap.add_argument("--peer", type=int, default=0)
    ap.add_argument("--timeout", type=float, default=600.0)
    a = ap.parse_args(argv)
    rc = 1
    try:
        spec = JobSpec.load(a.spec).finalize()
        rc = run_stage(spec, a.rank, a.peer, a.timeout)
    except Exception as e:
        traceback.print_exc()
        msg = str(e).lower()
        # A neighbour that vanished surfaces as a transport error or timeout of
        # a collective / p2p op; the liveness judge keys on this phrase.
        if any(k in msg for k in ("connection", "closed", "reset", "timed out", "timeout",
                                  "broken pipe", "nccl", "gloo")):
            print(f"WT_ERROR peer connection lost: {e}", flush=True)
        rc = 1
    print(f"WT_DONE {rc}", flush=True)
    return rc


if __name__ == "__main__":
    sys.exit(main())
