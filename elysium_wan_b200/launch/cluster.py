"""A whole job on one machine: an in-process coordinator and worker agents as
real subprocesses (`python -m elysium_wan_b200 worker`), with host-side fault
injectors (kill a worker, freeze a stage). Used by the WAN demo and the chaos
tests; nothing here touches a GPU's state.

Reference: tests/helpers/cluster.py (LocalCluster with kill_worker /
kill_stage / freeze_stage) and examples/wan_cluster_demo.py.
"""

from __future__ import annotations

import os
import signal
import subprocess
import sys
import time

from elysium_wan_b200.control.coordinator import Coordinator, CoordinatorConfig

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

# Fast fault-tolerance timings for small runs (seconds).
FAST_FT = dict(heartbeat_timeout_s=4.0, reconnect_grace_s=3.0, stall_floor_s=30.0,
               strike_gap_s=2.0, first_step_timeout_s=120.0, exit_report_grace_s=3.0)


class LocalCluster:
    def __init__(self, workdir: str, regions: list, token: str = "demo-token", device: str = "cpu",
                 wan_links: dict | None = None, liveness: dict | None = None, max_heals: int = 3,
                 stage_timeout_s: float = 30.0, coord: dict | None = None,
                 worker_env: dict | None = None, worker_args: list | None = None,
                 sequential: bool = False):
        self.workdir = os.path.abspath(workdir)
        os.makedirs(self.workdir, exist_ok=True)
        cfg = CoordinatorConfig(state_dir=os.path.join(self.workdir, "coordinator"), token=token,
                                wait_workers_s=120.0, liveness=dict(FAST_FT, **(liveness or {})),
                                wan_links=wan_links or {}, max_heals=max_heals,
                                stage_timeout_s=stage_timeout_s, poll_s=0.2,
                                min_workers=len(regions), **(coord or {}))
        self.coord = Coordinator("127.0.0.1", 0, cfg).start()
        self.token = token
        self.workers: list = []
        env = dict(os.environ)
        env["PYTHONPATH"] = ROOT + os.pathsep + env.get("PYTHONPATH", "")
        env["WANTRAIN_COORD_TOKEN"] = token
        # worker_env: extra variables for every worker, or a list with one dict per worker;
        # worker_args: one list of extra `wantrain worker` flags per worker
        per = worker_env if isinstance(worker_env, list) else [worker_env or {}] * len(regions)
        for i, region in enumerate(regions):
            name = f"w{i}"
            log = open(os.path.join(self.workdir, f"{name}.log"), "w")
            cmd = [sys.executable, "-m", "elysium_wan_b200", "worker", "--coordinator",
                   f"127.0.0.1:{self.coord.port}", "--coordinator-id", self.coord.id, "--name", name,
                   "--workdir", os.path.join(self.workdir, name), "--device", device, "--region",
                   region, "--no-bench"] + list((worker_args or [[]] * len(regions))[i])
            p = subprocess.Popen(cmd, stdout=log, stderr=subprocess.STDOUT, env={**env, **per[i]},
                                 start_new_session=True)
            self.workers.append((name, p, log))
            if sequential:
                # registration order = list order (placement takes workers in
                # that order; the last ones are the spares)
                deadline = time.time() + 120.0
                while len(self.coord.nodes) < i + 1 and time.time() < deadline and p.poll() is None:
                    time.sleep(0.1)

    def node_of(self, name: str):
        for nid, n in self.coord.nodes.items():
            if n.info.name == name:
                return nid
        return None

    def worker_of_slot(self, slot) -> str | None:
        nid = self.coord.slot_node.get(slot)
        return self.coord.nodes[nid].info.name if nid else None

    def kill_worker(self, name: str):
        """SIGKILL the agent (its stage dies with it): a worker machine lost."""
        for n, p, _ in self.workers:
            if n == name and p.poll() is None:
                os.killpg(p.pid, signal.SIGKILL)
                p.wait()

    def freeze_worker(self, name: str):
        for n, p, _ in self.workers:
            if n == name and p.poll() is None:
                os.killpg(p.pid, signal.SIGSTOP)

    def _stage_pid(self, name: str) -> int | None:
        try:
            with open(os.path.join(self.workdir, name, "stage.pid")) as f:
                return int(f.read().strip())
        except (OSError, ValueError):
            return None

    def kill_stage(self, name: str):
        """SIGKILL the worker's stage process group; the agent survives and
        reports the exit (no done marker): a stage killed from outside."""
        pid = self._stage_pid(name)
        if pid:
            try:
                os.killpg(pid, signal.SIGKILL)
            except ProcessLookupError:
                pass

    def freeze_stage(self, name: str):
        """SIGSTOP the worker's stage: alive and heartbeating (its agent runs),
        but no progress anywhere."""
        pid = self._stage_pid(name)
        if pid:
            try:
                os.killpg(pid, signal.SIGSTOP)
            except ProcessLookupError:
                pass

    def sever_control(self, name: str):
        """Close the coordinator's side of a worker's control connection (a
        control-plane blip); the agent dials back with its node id."""
        nid = self.node_of(name)
        if nid is not None:
            self.coord.nodes[nid].ch.close()

    def run(self, job):
        return self.coord.run_job(job)

    def close(self):
        self.coord.stop()
        time.sleep(0.3)
        for _, p, log in self.workers:
            if p.poll() is None:
                try:
                    os.killpg(p.pid, signal.SIGKILL)
                except ProcessLookupError:
                    pass
            p.wait()
            log.close()
