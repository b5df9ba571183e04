"""Worker agent: one per machine (or per GPU on a B200 box).

Reference: WorkerAgent (src/wantrain/worker/agent.py:403-1301). The agent
dials the coordinator, answers the CHALLENGE with an HMAC'd HELLO carrying its
measured capabilities, heartbeats every second, and supervises one stage
subprocess (`python -m elysium_wan_b200.runtime.stage_main`). It turns the
stage's WT_* stdout markers into PROGRESS / TELEM_STEP messages, answers
PROBE (a row of the link matrix) and MEASURE (one path in full), ships every
checkpoint wave to the coordinator (CKPT, files with sha256), ships the stage's
per-step telemetry file (TELEMETRY) and reports EXIT {rc, done_marker, log
tail} and, from the last stage, RESULT {losses}. It
obeys ABORT (kill the stage's process group), RESTORE (write shipped wave
files), RELEASE and SHUTDOWN, and reconnects with backoff when the control
connection drops.
"""

from __future__ import annotations

import hashlib
import json
import os
import shutil
import signal
import subprocess
import sys
import threading
import time
import traceback

from elysium_wan_b200.fault_tolerance import checkpoint as ckpt
from elysium_wan_b200.transport.control import Channel, body_sha256, control_dial, token_mac, write_body

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _die_with_parent():
    """Child-side: receive SIGKILL when the agent dies (Linux prctl), so a dead
    worker machine takes its stage with it."""
    try:
        import ctypes

        ctypes.CDLL("libc.so.6", use_errno=True).prctl(1, signal.SIGKILL)  # PR_SET_PDEATHSIG
    except Exception:
        pass


class StageProcess:
    """One stage subprocess in its own process group, stdout read line by line."""

    def __init__(self, cmd: list, env: dict, on_line, log_path: str):
        self.log = open(log_path, "a")
        self.p = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, env=env,
                                  text=True, bufsize=1, start_new_session=True,
                                  preexec_fn=_die_with_parent)
        self.tail: list = []
        self.done_marker = False
        self.t = threading.Thread(target=self._read, args=(on_line,), daemon=True)
        self.t.start()

    def _read(self, on_line):
        for line in self.p.stdout:
            if self.log is not None:
                # a log that cannot be written (disk full, file gone) never
                # stops the pump: the stage would block on a full pipe and its
                # markers would stop reaching the coordinator
                try:
                    self.log.write(line)
                    self.log.flush()
                except (OSError, ValueError) as e:
                    print(f"stage log not written from here on: {e}", file=sys.stderr, flush=True)
                    self.log = None
            line = line.rstrip("\n")
            self.tail = (self.tail + [line])[-40:]
            if line.startswith("WT_DONE"):
                self.done_marker = True
            try:
                on_line(line)
            except Exception:
                traceback.print_exc()

    def alive(self) -> bool:
        return self.p.poll() is None

    def kill(self):
        if self.p.poll() is None:
            try:
                os.killpg(self.p.pid, signal.SIGKILL)
            except ProcessLookupError:
                pass
        self.p.wait()
        self.t.join(timeout=5)
        self._close_log()

    def wait(self) -> int:
        rc = self.p.wait()
        self.t.join(timeout=10)
        self._close_log()
        return rc

    def _close_log(self):
        try:
            if self.log is not None:
                self.log.close()
        except OSError:
            pass


class WorkerAgent:
    def __init__(self, coordinator: str, coordinator_id: str = "", token: str | None = None,
                 name: str | None = None, workdir: str = "worker", device: str = "cpu",
                 region: str = "default", wan_profile: str | None = None, declare: dict | None = None,
                 no_bench: bool = True, advertise_host: str = "127.0.0.1", heartbeat_s: float = 1.0,
                 probe_port: int | None = None):
        host, _, port = coordinator.rpartition(":")
        self.addr = (host or "127.0.0.1", int(port))
        # the coordinator this agent trusts: the flag, else $WANTRAIN_COORD_ID
        self.coordinator_id = coordinator_id or os.environ.get("WANTRAIN_COORD_ID", "")
        self.token = token if token is not None else os.environ.get("WANTRAIN_COORD_TOKEN", "")
        self.name = name or f"worker-{os.getpid()}"
        self.workdir = os.path.abspath(workdir)
        os.makedirs(self.workdir, exist_ok=True)
        self.device = device
        self.region = region
        self.wan_profile = wan_profile
        from elysium_wan_b200.resources.links import load_emulation

        # the region-pair link model this worker's probes are shaped by (WAN emulation)
        self.emu = load_emulation(region, wan_profile)
        self.declare = declare or {}
        self.no_bench = no_bench
        self.advertise_host = advertise_host
        self.heartbeat_s = heartbeat_s
        self.ch: Channel | None = None
        self.stage: StageProcess | None = None
        self.assign: dict | None = None
        self.stop = threading.Event()
        self.lock = threading.Lock()
        self.node_id = None
        # Link probe server (round trip and bandwidth from other workers).
        self.probe_port = None
        if probe_port is not None:
            from elysium_wan_b200.resources.links import serve_echo

            self._probe_srv, self.probe_port = serve_echo("0.0.0.0", probe_port)

    # ----------------------------------------------------------------- connection
    def _caps(self) -> dict:
        from elysium_wan_b200.resources.probe import measure

        caps = measure(self.device, bench=not self.no_bench)
        if os.environ.get("WANTRAIN_DEVICE_CLASS"):
            # an operator-chosen device class (e.g. an architecture class for a
            # fleet of different boards that compute alike)
            caps["device_class"] = os.environ["WANTRAIN_DEVICE_CLASS"]
        caps.update(self.declare)
        caps.update(name=self.name, region=self.region, host=self.advertise_host,
                    wan_profile=self.wan_profile, pid=os.getpid(), probe_port=self.probe_port)
        return caps

    def _connect(self):
        ch = control_dial(*self.addr)
        hdr, _ = ch.recv()
        if hdr.get("kind") != "CHALLENGE":
            raise ConnectionError(f"expected CHALLENGE, got {hdr.get('kind')}")
        cid = hdr.get("coordinator_id", "")
        if self.coordinator_id and cid != self.coordinator_id:
            raise ConnectionError(f"coordinator id {cid} is not the expected {self.coordinator_id}")
        ch.send("HELLO", caps=self._caps(), node_id=self.node_id,
                mac=token_mac(self.token, hdr["nonce"], cid))
        hdr, _ = ch.recv()
        if hdr.get("kind") != "WELCOME":
            raise PermissionError(f"coordinator refused: {hdr}")
        self.node_id = hdr["node_id"]
        self.ch = ch

    def send(self, kind: str, body: bytes = b"", **fields):
        ch = self.ch
        if ch is None:
            return
        try:
            ch.send(kind, body, **fields)
        except OSError:
            pass

    def run(self):
        backoff = 0.2
        hb = threading.Thread(target=self._heartbeat, daemon=True)
        hb.start()
        while not self.stop.is_set():
            try:
                self._connect()
                backoff = 0.2
                self._serve()
            except (ConnectionError, OSError):
                pass
            except PermissionError as e:
                print(f"WORKER refused: {e}", flush=True)
                return 2
            self.ch = None
            if self.stop.is_set():
                break
            time.sleep(backoff)
            backoff = min(5.0, backoff * 2)
        self._kill_stage()
        return 0

    def _heartbeat(self):
        while not self.stop.is_set():
            st = self.stage
            self.send("HEARTBEAT", stage_alive=(st.alive() if st else None), t=time.time())
            self.stop.wait(self.heartbeat_s)

    # ----------------------------------------------------------------- messages
    def _serve(self):
        from elysium_wan_b200.transport.control import Spilled

        while not self.stop.is_set():
            # restored checkpoint parts stream into the workdir's filesystem
            self.ch.spill_dir = os.path.join(self.workdir, ".spill")
            hdr, body = self.ch.recv()
            kind = hdr["kind"]
            handler = getattr(self, f"_on_{kind.lower()}", None)
            try:
                if handler is None:
                    self.send(f"{kind}_ACK", ok=False, why="unknown message")
                    continue
                handler(hdr, body)
            finally:
                if isinstance(body, Spilled):
                    body.discard()

    def _on_probe(self, hdr, body):
        """PROBE {targets: [[host, port, region], ...], self_index}: one row of
        the coordinator's probe matrix (round trip and upload rate to every
        other worker, shaped by this worker's WAN emulation). Without targets:
        this worker's capabilities again. Runs in a thread: the control
        channel keeps serving (heartbeats) meanwhile."""
        if "targets" not in hdr:
            self.send("PROBE_RESULT", caps=self._caps())
            return
        from elysium_wan_b200.resources.links import probe_row

        def run():
            try:
                row = probe_row(hdr["targets"], int(hdr["self_index"]),
                                secs=float(hdr.get("secs", 0.25)), flows=int(hdr.get("flows", 1)),
                                emu=self.emu)
                self.send("PROBE_RESULT", ok=True, row=row)
            except Exception as e:
                self.send("PROBE_RESULT", ok=False, why=repr(e))

        threading.Thread(target=run, daemon=True).start()

    def _on_measure(self, hdr, body):
        """MEASURE {host, port, region, target}: the full measurement of one
        path to another worker's probe server (round trip, up, down, both at
        once, duplex). Without a host: this device's capabilities with the
        matmul bench."""
        if "host" not in hdr:
            from elysium_wan_b200.resources.probe import measure

            self.send("MEASURE_RESULT", caps=measure(self.device, bench=True))
            return
        from elysium_wan_b200.resources.links import measure_pair

        def run():
            try:
                r = measure_pair(hdr["host"], int(hdr["port"]), flows=int(hdr.get("flows", 2)),
                                 secs=float(hdr.get("secs", 0.5)), emu=self.emu,
                                 region=hdr.get("region"))
                self.send("MEASURE_RESULT", ok=True, target=hdr.get("target"), **r)
            except Exception as e:
                self.send("MEASURE_RESULT", ok=False, target=hdr.get("target"), why=repr(e))

        threading.Thread(target=run, daemon=True).start()

    def _on_fit(self, hdr, body):
        from elysium_wan_b200.resources.fit import measure as fit_measure
        from elysium_wan_b200.runtime.spec import JobSpec

        try:
            spec = JobSpec.from_dict(hdr["spec"]).finalize()
            r = fit_measure(spec, hdr["stage"], self.device)
            self.send("FIT_RESULT", ok=True, **r)
        except Exception as e:
            self.send("FIT_RESULT", ok=False, why=repr(e))

    def _on_profile(self, hdr, body):
        from elysium_wan_b200.resources.profile import profile_stage
        from elysium_wan_b200.runtime.spec import JobSpec

        try:
            spec = JobSpec.from_dict(hdr["spec"]).finalize()
            self.send("PROFILE_RESULT", ok=True, **profile_stage(spec, hdr["stage"], self.device))
        except Exception as e:
            self.send("PROFILE_RESULT", ok=False, why=repr(e))

    def _run_dir(self, run_id: str) -> str:
        if not ckpt.safe_name(run_id):
            raise ValueError(f"refused run id {run_id!r}")
        d = os.path.join(self.workdir, run_id)
        os.makedirs(d, exist_ok=True)
        return d

    def _on_assign(self, hdr, body):
        self._kill_stage()
        run_id, attempt = hdr["run_id"], hdr["attempt"]
        stage, peer = hdr["stage"], hdr["peer"]
        d = self._run_dir(run_id)
        spec = dict(hdr["spec"])
        spec["out_dir"] = d
        if self.device != "cpu" and spec.get("device", "cpu").startswith("cuda"):
            spec["device"] = self.device
        sp = os.path.join(d, f"spec-a{attempt}-r{stage}p{peer}.json")
        with open(sp, "w") as f:
            json.dump(spec, f)
        env = dict(os.environ)
        from elysium_wan_b200.utils.determinism import PINNED_ENV

        env.update(PINNED_ENV)
        env.setdefault("CUDA_MODULE_LOADING", "EAGER")
        env["PYTHONPATH"] = ROOT + os.pathsep + env.get("PYTHONPATH", "")
        # Shared WAN budgets of this run and attempt: every stage process on
        # this host paces through the same bucket files (a host-wide path, so
        # agents of one host share them; a new attempt starts fresh buckets).
        import tempfile

        env["EWB_PACER_DIR"] = os.path.join(tempfile.gettempdir(), f"ewb-pacers-{os.getuid()}",
                                            f"{run_id}-a{attempt}")
        cmd = [sys.executable, "-m", "elysium_wan_b200.runtime.stage_main", "--spec", sp,
               "--rank", str(stage), "--peer", str(peer), "--timeout", str(hdr.get("timeout", 120))]
        self.assign = dict(hdr, spec_path=sp, dir=d)
        log = os.path.join(d, f"stage-a{attempt}-r{stage}p{peer}.log")
        self.stage = StageProcess(cmd, env, self._on_stage_line, log)
        # The stage's process id (its own process group), for host-side fault
        # injection by test harnesses.
        try:
            with open(os.path.join(self.workdir, "stage.pid"), "w") as f:
                f.write(str(self.stage.p.pid))
        except OSError:
            pass
        self.send("ASSIGN_ACK", ok=True, run_id=run_id, attempt=attempt)
        threading.Thread(target=self._supervise, args=(self.stage, dict(self.assign)), daemon=True).start()

    def _on_stage_line(self, line: str):
        a = self.assign or {}
        tag, _, rest = line.partition(" ")
        if tag == "WT_STEP":
            self.send("PROGRESS", step=json.loads(rest)["step"], attempt=a.get("attempt"))
        elif tag == "WT_TELEM":
            self.send("TELEM_STEP", telem=json.loads(rest), attempt=a.get("attempt"))
        elif tag == "WT_WAVE":
            w = json.loads(rest)
            self._ship_wave(w["dir"], a)
        elif tag == "WT_METRIC":
            self.send("METRIC", metric=json.loads(rest), attempt=a.get("attempt"))

    def _ship_wave(self, wave_dir: str, a: dict):
        """Send every file of a committed wave (wave.json last) to the
        coordinator, which files it under the slot of this connection."""
        step = ckpt._step_of(os.path.basename(os.path.normpath(wave_dir)))
        if step is None:
            return
        names = sorted(os.listdir(wave_dir), key=lambda n: n == "wave.json")
        for n in names:
            self.ch and self.ch.send_file("CKPT", os.path.join(wave_dir, n), step=step, name=n,
                                          run_id=a["run_id"], attempt=a.get("attempt"),
                                          last=(n == "wave.json"))

    def _supervise(self, proc: StageProcess, a: dict):
        rc = proc.wait()
        if self.stage is not proc:
            return
        spec = a["spec"]
        tel = os.path.join(a["dir"], f"{spec['tag']}_rank{a['stage']}p{a['peer']}_telemetry.jsonl")
        if os.path.exists(tel) and self.ch is not None:
            # the stage's per-step telemetry file, whole, before EXIT so the
            # coordinator has it when it sees the stage finish (reference:
            # worker/agent.py:1053-1067)
            try:
                self.ch.send_file("TELEMETRY", tel, run_id=a["run_id"], attempt=a["attempt"])
            except OSError:
                pass
        self.send("EXIT", rc=rc, done_marker=proc.done_marker, tail="\n".join(proc.tail[-20:]),
                  run_id=a["run_id"], attempt=a["attempt"], stage=a["stage"], peer=a["peer"])
        if rc == 0 and a["stage"] == spec["stages"] - 1:
            p = os.path.join(a["dir"], f"{spec['tag']}_losses_r{a['stage']}p{a['peer']}.json")
            if os.path.exists(p):
                with open(p) as f:
                    self.send("RESULT", losses=json.load(f)["losses"], run_id=a["run_id"],
                              attempt=a["attempt"], stage=a["stage"], peer=a["peer"])

    def _kill_stage(self):
        st = self.stage
        self.stage = None
        if st is not None:
            st.kill()

    def _on_abort(self, hdr, body):
        self._kill_stage()
        self.send("ABORT_ACK", ok=True)

    def _on_restore(self, hdr, body):
        """RESTORE: one file of a wave for this worker's next slot. The path is
        built here from checked parts (plain run id, tag and file name; integer
        slot and step), under <run dir>/waves/<tag>/r<R>p<P>/; the files land in
        a staging directory that is validated and renamed into place when the
        last one (wave.json) arrives."""
        run_id, tag, name = hdr.get("run_id"), hdr.get("tag"), hdr.get("name")
        stage, peer, step = hdr.get("stage"), hdr.get("peer"), hdr.get("step")
        ok = all(ckpt.safe_name(x) for x in (run_id, tag, name)) and \
            all(type(v) is int and v >= 0 for v in (stage, peer, step)) and \
            body_sha256(body) == hdr.get("sha256")
        if not ok:
            self.send("RESTORE_ACK", ok=False, why="refused: malformed restore part")
            return
        d = self._run_dir(run_id)
        final = ckpt.wave_dir(d, tag, stage, peer, step)
        staging = final + ".restore"
        os.makedirs(staging, exist_ok=True)
        write_body(body, os.path.join(staging, name))
        if not hdr.get("last"):
            return
        try:
            ckpt.validate_wave(staging)
        except ValueError as e:
            shutil.rmtree(staging, ignore_errors=True)
            self.send("RESTORE_ACK", ok=False, why=str(e), step=step)
            return
        if os.path.isdir(final):
            shutil.rmtree(final, ignore_errors=True)
        os.rename(staging, final)
        self.send("RESTORE_ACK", ok=True, step=step)

    def _on_release(self, hdr, body):
        """RELEASE {run_id}: the job is over; stop any stage and drop the
        assignment, so this worker is idle for the next job."""
        self._kill_stage()
        self.assign = None
        self.send("RELEASE_ACK", ok=True, run_id=hdr.get("run_id"))

    def _on_shutdown(self, hdr, body):
        self._kill_stage()
        self.stop.set()
        self.send("SHUTDOWN_ACK", ok=True)
        if self.ch:
            self.ch.close()
