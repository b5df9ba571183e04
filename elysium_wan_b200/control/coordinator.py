"""Coordinator: runs one job over registered worker agents.

Reference lifecycle (src/wantrain/coordinator/coordinator.py:316-2420):
register -> measure -> plan -> fit-check -> profile -> solve -> launch ->
monitor -> heal / restart -> complete. This coordinator keeps that lifecycle
and its message kinds:

  * register: agents dial in, answer the HMAC CHALLENGE (HELLO with
    capabilities), get WELCOME + a node id; a reconnect with the same node id
    rebinds the slot's channel.
  * plan: a job is {"spec": JobSpec} or {"plan": {...}, "stages": N}
    (scheduler/fleetplan.py). Workers are placed in rank order grouped by
    region; the rest are spares. Hops between regions get the worker's WAN
    link profile (the CPU/gloo configuration emulates it in the transport).
  * route (PROBE, MEASURE; with probing on): each worker in turn measures a
    row of the link matrix (round trip and upload rate to every other
    worker); a chain of 3+ single-peer stages is ordered through it for the
    fastest slowest hop, then the least total round trip
    (scheduler/routing.py). Each chosen hop is then measured in full; a hop
    far below its probe re-routes with the measured figures (reference
    :813-950). The matrix and the order go to rationale.json.
  * profile (PROFILE): every slot times F, B and W of one microbatch on its
    own node; the zero-bubble schedule and the peers' ownership weights are
    solved from those costs, and a cut the job did not pin is refined by the
    measured stage rates (reference :1591-1700). fit-check (FIT) is optional.
  * launch: ASSIGN to every slot, last rank first, with a fresh rendezvous
    port per attempt (a heal relaunches every slot, so NCCL / gloo groups are
    always new).
  * monitor: HEARTBEAT / PROGRESS / EXIT into SlotStates judged by the
    LivenessJudge every poll_s.
  * heal: ABORT all, pick a spare for the convicted slot, resume from the
    newest wave every slot holds (shipped CKPT files, sha256-checked), RESTORE
    that slot's wave to the spare, relaunch with resume=true.
  * stalled: restart in place from the common wave.
  * rebalance (`_maybe_recut`, reference :2194-2400): each stage's WT_TELEM
    summaries fill a per-slot window; at every new common wave the measured
    F + B + W per microbatch re-cut the chain (scheduler/rebalance.py) when
    the slowest stage shrinks by `recut_min_gain` and the saving over the
    remaining steps beats `recut_cost_s`: ABORT, convert the common wave to
    the new cut through the logical form (fault_tolerance/logical.py) under a
    new tag, RESTORE every slot, relaunch.
  * re-plan (`_reschedule_plan`, reference :2194 via zero_bubble.replan):
    when no re-cut pays, the zero-bubble order is re-solved from the same
    measured costs and the run relaunches from the wave with it (the cut and
    the ownership stay, so no bit changes).
  * slow slot (`_watch_slow`, reference :2406): a slot whose compute per
    microbatch stays above `slow_ratio` x its own baseline for `slow_runs`
    summaries is healed onto a spare, or, with none, re-cut away from.
  * complete: RESULT losses of the last stage -> runs/<id>/losses.json and
    result.json; every slot's worker gets RELEASE (idle for the next job) and
    its stage's telemetry file arrives as TELEMETRY before its EXIT.
"""

from __future__ import annotations

import collections
import copy
import hashlib
import json
import math
import os
import socket
import statistics
import threading
import time
import uuid
from dataclasses import dataclass, field

from elysium_wan_b200.fault_tolerance import checkpoint as ckpt
from elysium_wan_b200.fault_tolerance.liveness import LivenessJudge, SlotState
from elysium_wan_b200.fault_tolerance.replacement import find_replacement
from elysium_wan_b200.resources.node import NodeInfo, mixed_fleet
from elysium_wan_b200.runtime.spec import JobSpec

# The fit loop (`Coordinator._fit_loop`): remedies tried before a job that does
# not fit is refused, and how far an overshooting stage's planning memory
# drops per unit of excess (the analytic model misses by a per-layer amount,
# so one re-cut usually clears it).
FIT_ATTEMPTS = 4
MEM_FEEDBACK = 1.25
from elysium_wan_b200.transport.control import (Channel, Spilled, body_sha256, check_mac,
                                                control_listen, new_nonce, write_body)


@dataclass
class CoordinatorConfig:
    state_dir: str = "coordinator_state"
    token: str = ""
    wait_workers_s: float = 120.0
    poll_s: float = 0.25
    max_heals: int = 3
    max_restarts: int = 2
    no_probe: bool = True
    route: bool = True     # with probing on: order a chain of 3+ workers through the probe matrix
    probe_secs: float = 0.25  # upload seconds per pair in a probe-matrix row
    probe_disagree: float = 0.5  # a full measurement below this x its probe re-routes
    no_fit_check: bool = True
    profile: bool = True   # measure F/B/W per slot before launch and solve the schedule from them
    profile_timeout_s: float = 300.0
    group_by: str = "region"
    allow_shared_hosts: bool = True
    any_region: bool = True
    zb_mem_mode: str = "auto"
    replacement_match: str = "any"
    keep_workers: bool = False
    stage_timeout_s: float = 60.0
    liveness: dict = field(default_factory=dict)
    wan_links: dict = field(default_factory=dict)  # {"regionA|regionB": {bw_mbps, latency_ms}}
    job_timeout_s: float = 3600.0
    min_workers: int = 0  # wait for at least this many (slots + spares) before placing
    # rebalance from telemetry
    recut: bool = True
    recut_min_gain: float = 0.05      # the slowest stage must shrink by this fraction
    recut_cost_s: float = 60.0        # what a re-cut costs (abort, convert, relaunch)
    max_replans: int = 2
    replan_min_summaries: int = 4     # per slot, in the current attempt
    replan: bool = True               # re-solve the zero-bubble order from telemetry
    replan_min_gain: float = 0.10     # a re-solved order must be this much shorter ...
    replan_cost_s: float = 30.0       # ... and save twice this over the remaining steps
    telem_window: int = 8
    watch_slow: bool = True
    slow_ratio: float = 1.3
    slow_runs: int = 3


@dataclass
class Job:
    spec: JobSpec | None = None
    plan: dict | None = None
    stages: int | None = None


@dataclass
class RunResult:
    ok: bool
    run_id: str
    losses_path: str | None
    attempts: int
    heals: int
    restarts: int
    why: str = ""
    run_dir: str = ""


class _Node:
    def __init__(self, info: NodeInfo, ch: Channel):
        self.info = info
        self.ch = ch
        self.connected = True
        self.disconnected_at = None
        self.last_heartbeat = time.time()
        self.stage_alive = None
        self.dead = False


def _size(n: float) -> str:
    return f"{n / 2**30:.2f} GiB" if n >= 2**30 else f"{n / 2**20:.1f} MiB"


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class Coordinator:
    def __init__(self, host: str = "127.0.0.1", port: int = 28000, cfg: CoordinatorConfig | None = None):
        self.host, self.port = host, port
        self.cfg = cfg or CoordinatorConfig()
        self.id = uuid.uuid4().hex[:16]
        self.nodes: dict[str, _Node] = {}
        self.order: list = []  # node ids in registration order
        self.lock = threading.RLock()
        self.stop_ev = threading.Event()
        self.sock = None
        self.slots: dict = {}  # (stage, peer) -> SlotState
        self.slot_node: dict = {}  # (stage, peer) -> node id
        self.results: dict = {}
        self.run_id = None
        self.attempt = 0
        self.store = None
        self.events: list = []
        self.on_progress = None  # callback(slot, step, node_id)
        self._pending_ckpt: dict = {}
        self.link_memory = None
        self.link_results: dict = {}
        self.replies: dict = {}  # (result kind, node id) -> fields
        self.plan_rationale: dict | None = None
        self.run_dir: str | None = None
        # rebalance state (per run)
        self.telem: dict = {}          # slot -> deque of this attempt's summaries
        self.telem_all: dict = {}      # slot -> compute ms of every summary of this attempt
        self.replans: list = []
        self.replan_checked = -1
        self.slot_base: dict = {}
        self.slot_hist: dict = {}
        self.slow_noted = None
        self._next: tuple | None = None  # (kind, payload) decided by the monitor

    # ----------------------------------------------------------------- server
    def start(self):
        self.sock = control_listen(self.host, self.port)
        self.port = self.sock.getsockname()[1]
        os.makedirs(self.cfg.state_dir, exist_ok=True)
        from elysium_wan_b200.scheduler.linkmemory import LinkMemory

        self.link_memory = LinkMemory(self.cfg.state_dir)
        print(f"COORDINATOR_ID {self.id}", flush=True)
        threading.Thread(target=self._accept_loop, daemon=True).start()
        return self

    def stop(self):
        self.stop_ev.set()
        with self.lock:
            for n in self.nodes.values():
                if n.connected and not self.cfg.keep_workers:
                    try:
                        n.ch.send("SHUTDOWN")
                    except OSError:
                        pass
        try:
            self.sock.close()
        except OSError:
            pass

    def _accept_loop(self):
        while not self.stop_ev.is_set():
            try:
                s, _ = self.sock.accept()
            except OSError:
                return
            threading.Thread(target=self._handshake, args=(Channel(s),), daemon=True).start()

    def _handshake(self, ch: Channel):
        nonce = new_nonce()
        try:
            ch.send("CHALLENGE", nonce=nonce, coordinator_id=self.id)
            hdr, _ = ch.recv()
            if hdr.get("kind") != "HELLO" or not check_mac(self.cfg.token, nonce, self.id, hdr.get("mac", "")):
                ch.send("REJECT", why="bad token or protocol")
                ch.close()
                return
            nid = self._register(hdr, ch)
            ch.send("WELCOME", node_id=nid, coordinator_id=self.id)
        except (OSError, ConnectionError, ValueError):
            ch.close()
            return
        self._conn_loop(nid, ch)

    def _register(self, hdr: dict, ch: Channel) -> str:
        with self.lock:
            nid = hdr.get("node_id")
            if nid and nid in self.nodes and not self.nodes[nid].dead:
                n = self.nodes[nid]
                down = None if n.disconnected_at is None else time.time() - n.disconnected_at
                n.ch, n.connected, n.disconnected_at = ch, True, None
                n.last_heartbeat = time.time()
                self._sync_slot(nid)
                self.events.append(("reconnected", nid, {"after_s": down}))
                return nid
            caps = hdr.get("caps", {})
            nid = f"n{len(self.order)}-{caps.get('name', 'worker')}"
            self.nodes[nid] = _Node(NodeInfo.from_caps(nid, caps), ch)
            self.order.append(nid)
            return nid

    def _slot_of(self, nid):
        for s, n in self.slot_node.items():
            if n == nid:
                return s
        return None

    def _sync_slot(self, nid):
        s = self._slot_of(nid)
        if s is not None and s in self.slots:
            n = self.nodes[nid]
            st = self.slots[s]
            st.connected, st.disconnected_at = n.connected, n.disconnected_at
            st.last_heartbeat, st.stage_alive = n.last_heartbeat, n.stage_alive

    def _conn_loop(self, nid: str, ch: Channel):
        while not self.stop_ev.is_set():
            # large bodies (checkpoint parts) stream into the store's filesystem
            ch.spill_dir = os.path.join(self.store.root, ".spill") if self.store is not None else None
            try:
                hdr, body = ch.recv()
            except (OSError, ConnectionError, ValueError):
                with self.lock:
                    n = self.nodes.get(nid)
                    if n is not None and n.ch is ch:
                        n.connected = False
                        n.disconnected_at = time.time()
                        self._sync_slot(nid)
                return
            try:
                self._dispatch(nid, hdr, body)
            finally:
                if isinstance(body, Spilled):
                    body.discard()  # a body nobody took

    def _dispatch(self, nid: str, hdr: dict, body):
        kind = hdr["kind"]
        with self.lock:
            n = self.nodes[nid]
            slot = self._slot_of(nid)
            st = self.slots.get(slot) if slot is not None else None
            current = hdr.get("attempt") in (None, self.attempt)
            if kind == "HEARTBEAT":
                n.last_heartbeat = time.time()
                n.stage_alive = hdr.get("stage_alive")
                self._sync_slot(nid)
            elif kind == "PROGRESS" and st is not None and current:
                if st.add_progress(int(hdr["step"]), time.time(), self._final_step):
                    if self.on_progress:
                        self.on_progress(slot, int(hdr["step"]), nid)
            elif kind == "EXIT" and st is not None and hdr.get("attempt") == self.attempt:
                st.exit_code = int(hdr["rc"])
                st.done_marker = bool(hdr["done_marker"])
                st.log_tail = hdr.get("tail", "")
            elif kind == "RESULT" and hdr.get("attempt") == self.attempt:
                self.results[(hdr["stage"], hdr["peer"])] = hdr["losses"]
            elif kind == "CKPT" and self.store is not None and hdr.get("run_id") == self.run_id \
                    and hdr.get("attempt") == self.attempt:
                # The wave belongs to the slot of the connection that sent it;
                # only a validated integer step and a plain file name are taken
                # from the message (reference: checkpoint.py:727-745). A part of
                # an earlier attempt may belong to an abandoned timeline.
                if slot is not None and body_sha256(body) == hdr.get("sha256"):
                    r, q = slot
                    try:
                        self.store.stage_part(self.run_id, r, q, hdr.get("step"), hdr.get("name"),
                                              body)
                        if hdr.get("last"):
                            self.store.commit_staged(self.run_id, self.ckpt_tag, r, q,
                                                     hdr.get("step"))
                    except (ValueError, OSError) as e:
                        self.events.append(("ckpt_refused", nid, str(e)))
            elif kind == "TELEMETRY" and slot is not None and current and self.run_dir:
                # rank and peer come from the connection's slot, never from the
                # message (reference: coordinator/coordinator.py:594-604)
                if body_sha256(body) == hdr.get("sha256"):
                    r, q = slot
                    path = os.path.join(self.run_dir, f"telemetry_r{r}p{q}_a{self.attempt}.jsonl")
                    try:
                        write_body(body, path)
                    except OSError:
                        pass
            elif kind == "TELEM_STEP":
                self.events.append(("telem", nid, hdr.get("telem")))
                if slot is not None and current and isinstance(hdr.get("telem"), dict):
                    self.telem.setdefault(
                        slot, collections.deque(maxlen=self.cfg.telem_window)).append(hdr["telem"])
                    # every summary's compute of this attempt, in arrival order:
                    # the slow-slot baseline must not depend on when the monitor polls
                    from elysium_wan_b200.scheduler.rebalance import stage_compute_ms

                    self.telem_all.setdefault(slot, []).append(stage_compute_ms(hdr["telem"]))
                    if self.run_dir:
                        try:
                            with open(os.path.join(self.run_dir, "telem_steps.jsonl"), "a") as f:
                                f.write(json.dumps({"slot": list(slot), "attempt": self.attempt,
                                                    "telem": hdr["telem"]}) + "\n")
                        except OSError:
                            pass
            elif kind in ("PROFILE_RESULT", "FIT_RESULT", "PROBE_RESULT", "RELEASE_ACK"):
                self.replies[(kind, nid)] = {k: v for k, v in hdr.items() if k != "kind"}
            elif kind == "MEASURE_RESULT" and "target" in hdr:
                self.link_results[(nid, hdr.get("target"))] = {k: v for k, v in hdr.items()
                                                              if k != "kind"}
            else:
                self.events.append((kind, nid, {k: v for k, v in hdr.items() if k != "kind"}))

    # ----------------------------------------------------------------- job
    def wait_for_workers(self, n: int, timeout: float) -> list:
        t0 = time.time()
        while time.time() - t0 < timeout:
            with self.lock:
                live = [nid for nid in self.order if self.nodes[nid].connected and not self.nodes[nid].dead]
            if len(live) >= n:
                return live
            time.sleep(0.1)
        raise TimeoutError(f"only {len(live)} of {n} workers registered in {timeout:.0f}s")

    def _spec_for(self, job: Job) -> JobSpec:
        if job.spec is not None:
            return job.spec
        from elysium_wan_b200.scheduler.fleetplan import build_spec, plan_job

        with self.lock:
            fleet = [self.nodes[n].info for n in self.order if not self.nodes[n].dead]
        if job.stages is None and "stages" not in job.plan:
            # plan mode: depth, widths, layout and microbatches from the fleet
            spec, self.plan_rationale = plan_job(job.plan, fleet)
            return spec
        return build_spec(job.plan, job.stages, fleet)

    def _place(self, spec: JobSpec, live: list) -> list:
        """Slots in rank order take workers grouped by region (stable), the rest
        are spares. group_by any / model / series runs the node selector
        (one device class, remembered-dead hosts skipped, remembered path
        verdicts ranked) and keeps its choice first."""
        infos = [self.nodes[n].info for n in live]
        if self.cfg.group_by in ("any", "model", "series"):
            from elysium_wan_b200.scheduler.selection import SelectionPolicy, select_nodes

            pol = SelectionPolicy(group_by=self.cfg.group_by, same_region=not self.cfg.any_region,
                                  distinct_hosts=not self.cfg.allow_shared_hosts)
            sel = select_nodes(infos, spec.world_size, pol, self.link_memory)
            if not sel.ok:
                raise ValueError(sel.reason)
            return [n.node_id for n in sel.chosen] + [n.node_id for n in sel.spares]
        why = mixed_fleet(infos)
        if why:
            raise ValueError(why)
        if self.cfg.group_by == "region":
            regions = []
            for i in infos:
                if i.region not in regions:
                    regions.append(i.region)
            live = sorted(live, key=lambda n: regions.index(self.nodes[n].info.region))
        return live

    def _probe_links(self, spec: JobSpec, timeout: float = 30.0) -> dict:
        """Each pipeline hop measured by its upstream worker against the
        downstream worker's probe server; results go to the link memory."""
        asked = []
        for j in range(spec.stages - 1):
            a, b = self.slot_node[(j, 0)], self.slot_node[(j + 1, 0)]
            bi = self.nodes[b].info
            port = bi.caps.get("probe_port")
            if not port:
                continue
            # measured with the data plane's own flow count: a hop's rate over
            # one flow says little about `p2p_streams` flows (reference:
            # coordinator.py:1013-1017)
            self.nodes[a].ch.send("MEASURE", host=bi.host, port=int(port), region=bi.region,
                                  target=b, flows=max(1, int(spec.p2p_streams or 1)))
            asked.append((j, a, b))
        out = {}
        end = time.time() + timeout
        for j, a, b in asked:
            while (a, b) not in self.link_results and time.time() < end:
                time.sleep(0.05)
            r = self.link_results.get((a, b))
            if r and r.get("ok"):
                ai, bi = self.nodes[a].info, self.nodes[b].info
                mbps = min(r["up_mbps"], r["down_mbps"])
                if self.link_memory is not None:
                    self.link_memory.record_path(ai.host, bi.host, mbps, r["rtt_ms"],
                                                 self.run_id or "probe")
                out[f"{j}->{j + 1}"] = r
        return out

    def _probe_matrix(self, nids: list, timeout: float = 60.0, flows: int = 1):
        """(rtt, bw) over `nids`, symmetric: each worker in turn measures its
        round trip and upload rate to every other one's probe server (one row
        at a time: concurrent bulk probes would measure each other), then each
        pair takes its slower direction (reference: coordinator.py:813-857).
        None when a worker has no probe server or a row does not come back."""
        from elysium_wan_b200.scheduler.routing import symmetrize

        infos = [self.nodes[n].info for n in nids]
        if not all(i.caps.get("probe_port") for i in infos):
            return None
        targets = [[i.host, int(i.caps["probe_port"]), i.region] for i in infos]
        rtt, bw = [], []
        for k, nid in enumerate(nids):
            with self.lock:
                self.replies.pop(("PROBE_RESULT", nid), None)
            self.nodes[nid].ch.send("PROBE", targets=targets, self_index=k,
                                    secs=self.cfg.probe_secs, flows=flows)
            end = time.time() + timeout
            while ("PROBE_RESULT", nid) not in self.replies and time.time() < end:
                time.sleep(0.05)
            r = self.replies.get(("PROBE_RESULT", nid))
            if not r or not r.get("ok"):
                return None
            rtt.append(r["row"]["rtt_ms"])
            bw.append(r["row"]["bw_mbps"])
        return symmetrize(rtt, bw)

    def _route_chain(self, spec: JobSpec, live: list):
        """Order the chain's workers through the probed link matrix (max
        bottleneck rate, then min total round trip; scheduler/routing.py).
        Only a chain of single-peer stages over three or more workers is
        routed, and only an order clearly better than the placement's
        (`route_gain`) replaces it. -> (live, note or None)."""
        from elysium_wan_b200.scheduler.routing import chain_key, order_chain, route_gain

        n = spec.world_size
        if spec.stages < 3 or n != spec.stages or len(live) < n:
            return live, None
        chosen = live[:n]
        m = self._probe_matrix(chosen, flows=max(1, int(spec.p2p_streams or 1)))
        if m is None:
            return live, None
        rtt, bw = m
        order = order_chain(rtt, bw)
        ident = list(range(n))
        moved = order != ident and route_gain(ident, order, bw, rtt)
        note = {"probe_bw_mbps": [[None if not math.isfinite(x) else round(x, 1) for x in row]
                                  for row in bw],
                "probe_rtt_ms": [[None if not math.isfinite(x) else round(x, 3) for x in row]
                                 for row in rtt],
                "placed": [self.nodes[x].info.name for x in chosen],
                "order": [self.nodes[chosen[i]].info.name for i in (order if moved else ident)],
                "bottleneck_mbps": chain_key(order if moved else ident, bw, rtt)[0],
                "rerouted": moved, "matrix": (rtt, bw), "nids": chosen}
        if moved:
            live = [chosen[i] for i in order] + live[n:]
        return live, note

    def _memory_order(self, spec: JobSpec, live: list) -> list:
        """An unrouted chain on cards of different memory: the rank that needs
        the most (live activation graphs, the embedding on rank 0, logits and
        head on the last) takes the largest card (reference:
        coordinator.py:1023-1026 via placement.memory_order). Equal cards keep
        the placement's order."""
        from elysium_wan_b200.scheduler.placement import memory_order

        n = spec.world_size
        infos = [self.nodes[x].info for x in live[:n]]
        mems = [i.memory_bytes() for i in infos]
        if len(infos) < n or not all(mems) or min(mems) == max(mems):
            return live
        mo = memory_order(spec, infos)
        if mo is None:
            return live
        return [live[i] for i in mo] + live[n:]

    def _reroute_on_disagreement(self, spec: JobSpec, route: dict, measured: dict):
        """A hop whose full measurement is far below its probe (the probe was
        misled: a burst allowance, a shaper that kicks in late) re-routes the
        chain with the measured figures in the matrix (reference:
        coordinator.py:871-920). -> the new order (indices into the routed
        workers), or None when nothing changes."""
        from elysium_wan_b200.scheduler.routing import order_chain, route_gain

        rtt, bw = route["matrix"]
        chosen = route["nids"]
        cur = [chosen.index(self.slot_node[(j, 0)]) for j in range(spec.stages)]
        misled = False
        for j in range(spec.stages - 1):
            h = measured.get(f"{j}->{j + 1}")
            if h is None:
                continue
            a, b = cur[j], cur[j + 1]
            got = min(h["up_mbps"], h["down_mbps"])
            if bw[a][b] > 0 and got < self.cfg.probe_disagree * bw[a][b]:
                misled = True
            bw[a][b] = bw[b][a] = got
            rtt[a][b] = rtt[b][a] = h["rtt_ms"]
        if not misled:
            return None
        order = order_chain(rtt, bw)
        if order == cur or not route_gain(cur, order, bw, rtt):
            return None
        return order

    def _links(self, spec: JobSpec):
        links = []
        for j in range(spec.stages):
            link = {"latency_ms": 0.0, "bw_mbps": 0.0, "jitter_ms": 0.0, "jitter_seed": j}
            if j + 1 < spec.stages:
                a = self.nodes[self.slot_node[(j, 0)]].info
                b = self.nodes[self.slot_node[(j + 1, 0)]].info
                if a.region != b.region:
                    key = "|".join(sorted([a.region, b.region]))
                    link.update(self.cfg.wan_links.get(key, self.cfg.wan_links.get("*", {})))
            links.append(link)
        spec.links = links

    def run_job(self, job: Job) -> RunResult:
        if job.spec is None and job.stages is None and "stages" not in (job.plan or {}):
            # plan mode plans on the fleet: let the expected workers register first
            self.wait_for_workers(max(1, self.cfg.min_workers), self.cfg.wait_workers_s)
        spec = self._spec_for(job)
        cut_given = spec.partition is not None
        spec.zb_mem_mode = spec.zb_mem_mode or self.cfg.zb_mem_mode
        spec.finalize()
        self.run_id = time.strftime("%Y%m%d-%H%M%S") + "-" + uuid.uuid4().hex[:6]
        run_dir = os.path.join(self.cfg.state_dir, "runs", self.run_id)
        os.makedirs(run_dir, exist_ok=True)
        self.run_dir = run_dir
        self.store = ckpt.CheckpointStore(os.path.join(self.cfg.state_dir, "store"))
        self.ckpt_tag = spec.tag
        live = self.wait_for_workers(max(spec.world_size, self.cfg.min_workers),
                                     self.cfg.wait_workers_s)
        live = self._place(spec, live)
        slots = spec.slots()
        self.slot_node = {s: live[i] for i, s in enumerate(slots)}
        route = None
        if not self.cfg.no_probe and self.cfg.route:
            live, route = self._route_chain(spec, live)
            self.slot_node = {s: live[i] for i, s in enumerate(slots)}
        if route is None and spec.stages > 1 and spec.world_size == spec.stages:
            live = self._memory_order(spec, live)
            self.slot_node = {s: live[i] for i, s in enumerate(slots)}
        measured = {} if self.cfg.no_probe else self._probe_links(spec)
        for _ in range(2):  # a misled probe re-routes (twice at most), then re-measures
            order = None if route is None else self._reroute_on_disagreement(spec, route, measured)
            if order is None:
                break
            live = [route["nids"][i] for i in order] + live[spec.world_size:]
            self.slot_node = {s: live[i] for i, s in enumerate(slots)}
            route.update(order=[self.nodes[x].info.name for x in live[:spec.world_size]],
                         rerouted=True, remeasured=route.get("remeasured", 0) + 1)
            measured = self._probe_links(spec)
        spares = live[len(slots):]
        if route is not None:
            route.pop("matrix", None)
            route.pop("nids", None)
        self._links(spec)
        spec.finalize()
        schedule = None
        if spec.stages > 1 and self.cfg.profile and not spec.resume:
            schedule = self._zero_bubble(spec, slots, refine=not cut_given)
        admission = self._admit(spec, slots)
        if admission is not None and not admission["ok"]:
            why = "admission refused: " + "; ".join(admission["reasons"])
            return RunResult(False, self.run_id, None, 0, 0, 0, why, run_dir)
        fit_notes = None
        if not self.cfg.no_fit_check:
            fits, why, fit_notes = self._fit_loop(spec, slots, cut_given)
            if not fits:
                return RunResult(False, self.run_id, None, 0, 0, 0, why, run_dir)
        self._final_step = spec.steps - 1
        with open(os.path.join(run_dir, "spec.json"), "w") as f:
            f.write(spec.to_json())
        with open(os.path.join(run_dir, "rationale.json"), "w") as f:
            json.dump({"placement": {f"{s[0]}:{s[1]}": self.slot_node[s] for s in slots},
                       "spares": spares, "links": spec.links, "measured_links": measured,
                       "admission": admission, "schedule": schedule, "route": route,
                       "plan": self.plan_rationale, "fit": fit_notes},
                      f, indent=1)
        heals = restarts = 0
        resume_step = None
        self.replans, self.replan_checked = [], -1
        self.slot_base, self.slot_hist, self.slow_noted = {}, {}, None
        t_start = time.time()
        why = ""
        while True:
            if resume_step is not None:
                # the run continues from resume_step: newer waves in the store
                # belong to the abandoned timeline
                gone = self.store.drop_after(self.run_id, spec.tag, resume_step)
                if gone:
                    self.events.append(("waves_dropped", None, {"after": resume_step,
                                                                "waves": gone}))
            self._launch(spec, resume_step)
            verdict = self._monitor(spec, t_start)
            if verdict.kind == "done":
                losses = self._collect(spec, run_dir)
                res = RunResult(True, self.run_id, losses, self.attempt + 1, heals, restarts, "",
                                run_dir)
                break
            self._abort_all()
            if verdict.kind == "convict" and heals < self.cfg.max_heals:
                heals += 1
                dead = self.slot_node[verdict.slot]
                if self.link_memory is not None:
                    di = self.nodes[dead].info
                    self.link_memory.record_dead(f"{di.name}@{di.host}", verdict.why, self.run_id,
                                                 host=di.host)
                with self.lock:
                    self.nodes[dead].dead = True
                    # Any registered, live worker that holds no slot is a spare
                    # (including workers that joined after placement).
                    busy = set(self.slot_node.values())
                    spares = [n for n in self.order if n not in busy and not self.nodes[n].dead
                              and self.nodes[n].connected]
                    cands = [self.nodes[n].info for n in spares]
                rep = find_replacement(self.nodes[dead].info, cands, self.cfg.replacement_match)
                if rep is None:
                    res = RunResult(False, self.run_id, None, self.attempt + 1, heals, restarts,
                                    f"no spare for {verdict.slot}: {verdict.why}", run_dir)
                    break
                spares.remove(rep.node_id)
                self.slot_node[verdict.slot] = rep.node_id
                resume_step = self._resume_point(spec)
                self._restore(spec, verdict.slot, rep.node_id, resume_step)
                self.events.append(("heal", verdict.slot, {"from": dead, "to": rep.node_id,
                                                           "step": resume_step, "why": verdict.why}))
            elif verdict.kind == "stalled" and restarts < self.cfg.max_restarts:
                restarts += 1
                resume_step = self._resume_point(spec)
                self.events.append(("restart", None, {"step": resume_step, "why": verdict.why}))
            elif verdict.kind == "recut":
                new_spec, note = self._next[1]
                got = self._apply_recut(spec, new_spec, note, run_dir)
                if got is None:  # nothing to resume from: continue on the current cut
                    resume_step = self._resume_point(spec)
                else:
                    spec, resume_step = got
            elif verdict.kind == "reschedule":
                new_spec, note = self._next[1]
                resume_step = self._resume_point(spec)
                if new_spec.mb_owner != spec.mb_owner and resume_step:
                    # the steps before the resume point ran under the old table
                    new_spec.ownership_log = list(spec.ownership_log) + \
                        [[resume_step, spec.mb_owner]]
                    new_spec.finalize()
                spec = new_spec
                rec = {"step": resume_step, "reschedule": True, "note": note,
                       "owner_changed": bool(spec.ownership_log and
                                             spec.ownership_log[-1][0] == resume_step)}
                self.replans.append(rec)
                self.events.append(("reschedule", None, rec))
                with open(os.path.join(run_dir, "spec.json"), "w") as f:
                    f.write(spec.to_json())
            elif verdict.kind == "slow_heal":
                slot = verdict.slot
                with self.lock:
                    busy = set(self.slot_node.values())
                    spares = [n for n in self.order if n not in busy and not self.nodes[n].dead
                              and self.nodes[n].connected]
                    cands = [self.nodes[n].info for n in spares]
                old_nid = self.slot_node[slot]
                rep = find_replacement(self.nodes[old_nid].info, cands, self.cfg.replacement_match)
                resume_step = self._resume_point(spec)
                if rep is not None:
                    heals += 1
                    self.slot_node[slot] = rep.node_id
                    self._restore(spec, slot, rep.node_id, resume_step)
                    self.events.append(("heal", slot, {"from": old_nid, "to": rep.node_id,
                                                       "step": resume_step, "why": verdict.why}))
            else:
                why = verdict.why
                res = RunResult(False, self.run_id, None, self.attempt + 1, heals, restarts, why, run_dir)
                break
            self.attempt += 1
        released = self._release_all()
        with open(os.path.join(run_dir, "result.json"), "w") as f:
            json.dump({"ok": res.ok, "run_id": res.run_id, "attempts": res.attempts, "heals": res.heals,
                       "restarts": res.restarts, "why": res.why, "losses": res.losses_path,
                       "events": [list(map(str, e)) for e in self.events
                                  if e[0] in ("heal", "restart", "recut", "reschedule")],
                       "replans": self.replans, "released": released},
                      f, indent=1)
        return res

    def _release_all(self, timeout: float = 10.0) -> list:
        """RELEASE every worker that held a slot (its stage is stopped and its
        assignment dropped, so it is idle for the next job; reference:
        coordinator.py:1895-1905). -> names of the workers that acknowledged."""
        with self.lock:
            nids = [n for n in dict.fromkeys(self.slot_node.values())
                    if self.nodes[n].connected and not self.nodes[n].dead]
            for n in nids:
                self.replies.pop(("RELEASE_ACK", n), None)
        asked = []
        for n in nids:
            try:
                self.nodes[n].ch.send("RELEASE", run_id=self.run_id)
                asked.append(n)
            except OSError:
                pass
        end = time.time() + timeout
        while time.time() < end and not all(("RELEASE_ACK", n) in self.replies for n in asked):
            time.sleep(0.05)
        return [self.nodes[n].info.name for n in asked if ("RELEASE_ACK", n) in self.replies]

    def _ask_slots(self, kind: str, result: str, spec, slots, timeout: float) -> dict:
        """Send `kind` (PROFILE / FIT) for every slot to its node at once and
        collect the `result` replies. -> {slot: fields}; a missing reply is
        {"ok": False, "why": "timeout"}."""
        with self.lock:
            for s in slots:
                self.replies.pop((result, self.slot_node[s]), None)
        body = spec.to_dict()
        for s in slots:
            self.nodes[self.slot_node[s]].ch.send(kind, spec=body, stage=s[0], peer=s[1])
        t0 = time.time()
        while time.time() - t0 < timeout:
            with self.lock:
                if all((result, self.slot_node[s]) in self.replies for s in slots):
                    break
            time.sleep(0.05)
        with self.lock:
            return {s: self.replies.get((result, self.slot_node[s]), {"ok": False, "why": "timeout"})
                    for s in slots}

    def _zero_bubble(self, spec, slots, refine: bool) -> dict:
        """Profile every slot on its own node (F, B, W of one microbatch),
        re-cut by the measured stage rates when the job did not pin a cut and
        it shortens the slowest stage by 5% (reference: coordinator.py:1591-
        1700), then solve the zero-bubble schedule and the peers' ownership
        weights from the measured costs. A failed profile keeps the analytic
        schedule."""
        from elysium_wan_b200.scheduler import rebalance as rb

        def profile():
            got = self._ask_slots("PROFILE", "PROFILE_RESULT", spec, slots,
                                  self.cfg.profile_timeout_s)
            bad = [f"{s}: {r.get('why')}" for s, r in got.items() if not r.get("ok")]
            if bad:
                raise RuntimeError("; ".join(bad))
            out = []
            for r in range(spec.stages):
                out.append([{"t_f": got[(r, p)]["F"], "t_b": got[(r, p)]["B"],
                             "t_w": got[(r, p)]["W"]} for p in range(spec.stage_widths[r])])
            return out

        refined = None
        try:
            profiles = profile()
            if refine:
                res = rb.refined_partition(spec, profiles, None, 0.05)
                if res is not None:
                    refined = {"from": spec.partition, "to": res[0]}
                    spec.partition = res[0]
                    spec.stage_costs = None
                    spec.reschedule()
                    profiles = profile()
        except RuntimeError as e:
            self.events.append(("profile_failed", None, {"why": str(e)}))
            return {"source": "analytic", "reason": str(e)}
        # each peer's weight is its measured rate; the stage's cost per
        # microbatch is its peers' combined rate
        weights = [[1.0 / max(1e-9, p["t_f"] + p["t_b"] + p["t_w"]) for p in row]
                   for row in profiles]
        costs = []
        for row, wr in zip(profiles, weights):
            share = sum(wr)
            costs.append([sum(p[k] * w for p, w in zip(row, wr)) / share / len(row)
                          for k in ("t_f", "t_b", "t_w")])
        spec.stage_costs = costs
        spec.peer_weights = [[w / max(wr) for w in wr] for wr in weights]
        spec.mb_owner = None
        spec.schedule_order = None
        spec.finalize()
        return {"source": "profiled", "partition_refined": refined,
                "costs_ms": [[round(x * 1e3, 3) for x in c] for c in costs],
                "peer_weights": [[round(w, 3) for w in row] for row in spec.peer_weights]}

    def _fit_check(self, spec, slots):
        """Every slot builds its real slice on its node and holds the
        schedule's peak in-flight microbatches (resources/fit.py). -> (why a
        fit could not run or None, {stage: overshoot}) where an overshoot is
        the worst slot's {"peak", "budget", "base", "oom"} in bytes: a peak
        above the node's memory less its reserve, or an out-of-memory fit
        (whose demand is unknown: the peak counts as the whole device)."""
        from elysium_wan_b200.scheduler.admission import vram_reserve

        got = self._ask_slots("FIT", "FIT_RESULT", spec, slots, self.cfg.profile_timeout_s)
        over: dict = {}
        for s in slots:
            r = got[s]
            if not r.get("ok"):
                return f"fit of slot {s} failed: {r.get('why')}", {}
            mem = self.nodes[self.slot_node[s]].info.memory_bytes()
            budget = mem - vram_reserve(mem) if mem else None
            oom = not r.get("fits")
            peak = float(r.get("peak_bytes") or 0)
            if oom:
                peak = max(peak, mem or 0.0)
            if not oom and (budget is None or peak <= budget):
                continue
            if budget is None:
                return f"slot {s} does not fit: peak {int(peak)} bytes", {}
            prev = over.get(s[0])
            if prev is None or peak - budget > prev["peak"] - prev["budget"]:
                over[s[0]] = {"peak": peak, "budget": budget,
                              "base": float(r.get("base_bytes") or 0), "oom": oom}
        return None, over

    def _fit_loop(self, spec, slots, cut_given: bool):
        """The fit check with feedback (reference behaviour: coordinator.py
        :1500-1570, FIT_ATTEMPTS, `calibrated_budget`, `shrink_for_overshoot`).
        The memory models are analytic, the fit is measured; a stage that
        overshoots its node's budget is answered in this order, one remedy per
        attempt, the fit measured again after each:

        1. a stage that keeps F's tensors recomputes them instead;
        2. the schedule's activation budget of the stage is calibrated: the
           model's in-flight activations are scaled by what the fit really
           held beyond the stage's resident state, and the zero-bubble order
           is solved again under the budget that leaves (fewer microbatches
           in flight there; the cut keeps its balance);
        3. unless the job pinned its cut, the stage plans with less memory
           (its budget less MEM_FEEDBACK x the excess) and the chain is cut
           again by the memory model, moving layers off it.

        -> (fits, why, notes)."""
        from elysium_wan_b200.scheduler import rebalance as rb
        from elysium_wan_b200.scheduler.planner import default_schedule

        notes: list = []
        caps: dict = {}
        shrunk: dict = {}
        why = ""
        for attempt in range(FIT_ATTEMPTS):
            bad, over = self._fit_check(spec, slots)
            if bad:
                return False, bad, notes
            if not over:
                return True, "", notes
            why = "; ".join(f"stage {r} peaks at {_size(o['peak'])} of a {_size(o['budget'])} "
                            "budget" for r, o in sorted(over.items()))
            if attempt == FIT_ATTEMPTS - 1:
                break
            keep = [r for r in sorted(over) if not spec.recomputes(r)]
            if keep:
                spec.recompute_stages = [spec.recomputes(r) or r in keep
                                         for r in range(spec.stages)]
                spec.reschedule()
                notes.append(f"{why}: stages {keep} recompute")
                continue
            fresh = [r for r in sorted(over) if r not in caps]
            if fresh:
                for r in fresh:
                    o = over[r]
                    caps[r] = rb.calibrated_budget(spec, r, o["peak"], o["budget"], o["base"],
                                                   oom=o["oom"], feedback=MEM_FEEDBACK)
                spec.schedule_order = default_schedule(spec, rb.budget_list(spec, caps))
                spec.finalize()
                notes.append(f"{why}: the schedule holds at most " + ", ".join(
                    f"{_size(caps[r])} of activations on stage {r}" for r in fresh))
                continue
            if cut_given:
                break
            for r, o in over.items():
                shrunk[r] = max(0.0, min(shrunk.get(r, o["budget"]),
                                         o["budget"] - MEM_FEEDBACK * (o["peak"] - o["budget"])))
            budgets = [shrunk.get(r, self._stage_budget(r)) for r in range(spec.stages)]
            new = rb.memory_partition(spec, budgets)
            if new is None:
                break
            notes.append(f"{why}: re-cut {spec.partition} -> {new}")
            spec.partition, caps = new, {}
            spec.stage_costs = None
            spec.reschedule()
        return False, f"does not fit after {len(notes)} remedies: {why}", notes

    def _stage_budget(self, r: int) -> float:
        """The smallest memory budget among stage r's nodes (inf when unknown)."""
        from elysium_wan_b200.scheduler.admission import vram_reserve

        out = math.inf
        for (st, _p), nid in self.slot_node.items():
            if st == r:
                mem = self.nodes[nid].info.memory_bytes()
                if mem:
                    out = min(out, mem - vram_reserve(mem))
        return out

    def _admit(self, spec, slots) -> dict | None:
        """Admission of a job with wide stages (scheduler/admission.py) on the
        nodes placed in its slots; None when every stage has width 1."""
        from elysium_wan_b200.scheduler import admission as ad

        if all(w == 1 for w in spec.stage_widths):
            return None
        infos = [self.nodes[self.slot_node[s]].info for s in slots]
        ok, reasons, pred = ad.admit(spec, ad.devices_from_nodes(infos))
        return {"ok": ok, "reasons": [r.text() for r in reasons],
                "exposed_s": {str(k): v["exposed_s"] for k, v in pred.items()}}

    # ------------------------------------------------------------ rebalance
    def _windows(self) -> dict:
        with self.lock:
            return {slot: list(w) for slot, w in self.telem.items()}

    def _maybe_rebalance(self, spec):
        """Once per new common wave: ("recut", (new spec, note)) when the
        measured stage costs call for another cut and it pays, else None."""
        recut = self.cfg.recut and os.environ.get("WANTRAIN_RECUT", "on") != "off"
        if not (recut or self.cfg.replan):
            return None
        if len(self.replans) >= self.cfg.max_replans or self.store is None:
            return None
        windows = self._windows()
        slots = spec.slots()
        # the first summary of an attempt holds its warm-up
        windows = {s: w[1:] for s, w in windows.items()}
        if any(len(windows.get(s, ())) < self.cfg.replan_min_summaries for s in slots):
            return None
        step = self._resume_point(spec)
        final = spec.steps
        if step is None or step <= self.replan_checked or step >= final:
            return None
        self.replan_checked = step
        got = self._recut_plan(spec, windows, step, final) if recut else None
        if got is None and self.cfg.replan:
            got = self._reschedule_plan(spec, windows, step, final)
        return got

    def _reschedule_plan(self, spec, windows, step, final):
        """A re-plan from the window's measured F / B / W, the cut kept: on a
        chain of width-1 stages the zero-bubble order is re-solved (no bit
        changes); with a wide stage the ownership is re-solved too (each
        peer's share of the microbatches from its measured rate,
        `rebalance.replan_ownership`), and the run records the old table in
        `ownership_log` from the resume step on. Applied when it is
        `replan_min_gain` shorter and saves more than twice `replan_cost_s`
        over the remaining steps."""
        from elysium_wan_b200.scheduler import rebalance as rb

        owners = None
        try:
            profiles = rb.profiles_from_telemetry(spec, windows)
            hops = rb.hops_from_telemetry(spec, windows)
            if any(w > 1 for w in spec.stage_widths):
                got = rb.replan_ownership(spec, profiles, self.cfg.replan_min_gain, hops)
                self.events.append(("replan_eval", None, {"step": step, "why": got["why"]}))
                res = None
                if got["decision"]:
                    res = got["schedule_order"], got["pred_cur_s"], got["pred_new_s"]
                    owners = got
            else:
                res = rb.replan_schedule(spec, profiles, self.cfg.replan_min_gain, hops)
        except ValueError as e:
            self.events.append(("reschedule_skipped", None, {"step": step, "why": str(e)}))
            return None
        if res is None:
            return None
        order, cur, new = res
        cost = float(os.environ.get("WANTRAIN_REPLAN_COST_S", self.cfg.replan_cost_s))
        gain = (cur - new) * max(0, final - step)
        note = (f"re-solved order: {cur * 1e3:.1f} -> {new * 1e3:.1f} ms per step predicted, "
                f"{gain:.1f} s over {final - step} steps against 2 x {cost:.1f} s")
        self.events.append(("reschedule_eval", None, {"step": step, "note": note}))
        if gain <= 2 * cost:
            return None
        d = spec.to_dict()
        d.update(schedule_order=order, stage_costs=rb.stage_costs_from_profiles(
            profiles, spec.peer_weights), resume=False, resume_step=None)
        if owners is not None:
            d.update(peer_weights=owners["peer_weights"], mb_owner=owners["mb_owner"],
                     stage_costs=owners["stage_costs"])
            if owners["owner_changed"]:
                note += f"; peer weights {spec.peer_weights} -> {owners['peer_weights']}"
        nspec = JobSpec.from_dict(d)
        nspec.finalize()
        return "reschedule", (nspec, note)

    def _recut_plan(self, spec, windows, step, final, why: str | None = None):
        from elysium_wan_b200.scheduler import rebalance as rb

        refusal = rb.recut_refusal(spec)
        if refusal is not None:
            self.events.append(("recut_refused", None, {"step": step, "why": refusal}))
            return None
        try:
            profiles = rb.profiles_from_telemetry(spec, windows)
        except ValueError as e:
            self.events.append(("recut_skipped", None, {"step": step, "why": str(e)}))
            return None
        res = rb.refined_partition(spec, profiles, None, self.cfg.recut_min_gain)
        if res is None:
            return None
        new_part, before, after = res
        cost = float(os.environ.get("WANTRAIN_RECUT_COST_S", self.cfg.recut_cost_s))
        pays, saving = rb.recut_pays(before, after, spec.microbatches, final - step, cost)
        note = (f"re-cut {spec.partition} -> {new_part}: slowest stage {before * 1e3:.1f} -> "
                f"~{after * 1e3:.1f} ms per microbatch, ~{saving:.1f} s saved over {final - step} "
                f"steps against {cost:.1f} s" + (f" ({why})" if why else ""))
        self.events.append(("recut_eval", None, {"step": step, "note": note, "pays": pays}))
        if not pays:
            return None
        d = spec.to_dict()
        cuts = sum(1 for r in self.replans if r.get("recut"))
        d.update(partition=[list(x) for x in new_part], tag=f"{spec.tag.split('.cut')[0]}.cut{cuts + 1}",
                 schedule_order=None, mb_owner=None, resume=False, resume_step=None)
        new = JobSpec.from_dict(d)
        new.finalize()
        return "recut", (new, note)

    def _watch_slow(self, spec):
        """("slow", (slot, why)) for a slot that computes `slow_ratio` x its own
        baseline per microbatch for `slow_runs` summaries in a row and has a
        spare to move to; without a spare, a re-cut away from it (or None)."""
        from elysium_wan_b200.scheduler import rebalance as rb

        if not self.cfg.watch_slow or self.store is None:
            return None
        windows = self._windows()
        with self.lock:
            series = {slot: list(v) for slot, v in self.telem_all.items()}
        for slot, xs in series.items():
            hist = xs[2:]  # the attempt's first two summaries hold its warm-up
            if len(hist) >= self.cfg.slow_runs and slot not in self.slot_base:
                self.slot_base[slot] = statistics.median(hist[: self.cfg.slow_runs])
            if hist:
                self.slot_hist[slot] = hist
        slow = rb.slow_slots(self.slot_hist, self.slot_base, self.cfg.slow_ratio, self.cfg.slow_runs)
        if not slow:
            return None
        slot, ratio = max(slow, key=lambda x: x[1])
        why = f"slot {slot} computes {ratio:.2f}x its baseline per microbatch"
        step = self._resume_point(spec)
        if step is None or step >= spec.steps:
            return None
        with self.lock:
            busy = set(self.slot_node.values())
            spares = [n for n in self.order if n not in busy and not self.nodes[n].dead
                      and self.nodes[n].connected]
        if spares and sum(1 for e in self.events if e[0] == "heal") < self.cfg.max_heals:
            self.slot_base, self.slot_hist, self.slow_noted = {}, {}, None
            return "slow", (slot, why)
        if self.slow_noted == (slot, step) or len(self.replans) >= self.cfg.max_replans:
            return None
        self.slow_noted = (slot, step)
        recent = {s: w[-self.cfg.slow_runs:] for s, w in windows.items()}
        got = self._recut_plan(spec, recent, step, spec.steps, why)
        if got is not None:
            self.slot_base, self.slot_hist, self.slow_noted = {}, {}, None
        return got

    def _apply_recut(self, old: JobSpec, new: JobSpec, note: str, run_dir: str):
        """Abort, convert the common wave of every slot to `new`'s cut (a new
        tag, in the coordinator's store), ship each slot its wave. -> (new spec,
        resume step), or None when no common wave exists."""
        from elysium_wan_b200.fault_tolerance import logical

        step = self._resume_point(old)  # run_job has aborted every slot
        if step is None:
            self.replans.append({"recut": False, "why": "no common wave"})
            return None
        root = os.path.join(self.store.root, self.run_id)
        v_old, v_new = copy.copy(old), copy.copy(new)
        v_old.out_dir = v_new.out_dir = root
        logical.convert(v_old, v_new, step)
        rec = {"step": step, "recut": True, "from": old.partition, "to": new.partition,
               "tag": new.tag, "note": note}
        self.replans.append(rec)
        self.events.append(("recut", None, rec))
        with open(os.path.join(run_dir, "spec.json"), "w") as f:
            f.write(new.to_json())
        for s in new.slots():
            self._restore(new, s, self.slot_node[s], step)
        self._final_step = new.steps - 1
        return new, step

    def _resume_point(self, spec) -> int | None:
        return self.store.common_step(self.run_id, spec)

    def _restore(self, spec, slot, nid, step):
        """Ship the slot's wave at `step` from the store to its new worker.
        The wave is validated first (a step that does not validate is refused),
        and pinned so that pruning cannot remove it while it is shipped."""
        if step is None:
            return
        stage, peer = slot
        self.store.pinned.add(step)
        src = ckpt.wave_dir(os.path.join(self.store.root, self.run_id), spec.tag, stage, peer, step)
        meta = ckpt.validate_wave(src)  # raises ValueError: no heal from a damaged wave
        ch = self.nodes[nid].ch
        names = sorted(meta["files"]) + ["wave.json"]
        for n in names:
            # streamed from disk; the wave's own manifest already holds each
            # file's sha256 (validated above), wave.json's is computed
            sha = meta["files"][n]["sha256"] if n in meta["files"] else None
            extra = {"sha256": sha} if sha else {}
            ch.send_file("RESTORE", os.path.join(src, n), run_id=self.run_id, tag=spec.tag,
                         stage=stage, peer=peer, step=step, name=n, last=(n == "wave.json"),
                         **extra)

    def _launch(self, spec: JobSpec, resume_step):
        a = copy.deepcopy(spec)
        a.port_base = _free_port()
        a.resume = resume_step is not None
        a.resume_step = resume_step
        start = 0 if resume_step is None else resume_step
        with self.lock:
            self.results = {}
            self.slots = {}
            self.telem = {}
            self.telem_all = {}
            # a slot's baseline belongs to the node that runs it in this attempt
            self.slot_base, self.slot_hist, self.slow_noted = {}, {}, None
            for s in spec.slots():
                nid = self.slot_node[s]
                n = self.nodes[nid]
                self.slots[s] = SlotState(slot=s, node_id=nid, launched=True, connected=n.connected,
                                          last_heartbeat=time.time(), started_at=time.time(),
                                          start_step=start)
        for s in reversed(spec.slots()):
            self.nodes[self.slot_node[s]].ch.send(
                "ASSIGN", spec=a.to_dict(), stage=s[0], peer=s[1], run_id=self.run_id,
                attempt=self.attempt, timeout=self.cfg.stage_timeout_s)

    def _monitor(self, spec, t_start):
        from elysium_wan_b200.fault_tolerance.liveness import Verdict

        judge = LivenessJudge(final_step=spec.steps - 1, **self.cfg.liveness)
        while True:
            time.sleep(self.cfg.poll_s)
            with self.lock:
                v = judge.judge(list(self.slots.values()))
                if v.kind == "done":
                    last = spec.stages - 1
                    want = {(last, p) for p in range(spec.stage_widths[last])}
                    if not want <= set(self.results):
                        if time.time() - max(st.started_at for st in self.slots.values()) < 30:
                            continue
                    return v
                if v.kind in ("convict", "stalled", "failed"):
                    return v
            nxt = self._watch_slow(spec) or self._maybe_rebalance(spec)
            if nxt is not None:
                self._next = nxt
                kind, payload = nxt
                if kind in ("recut", "reschedule"):
                    return Verdict(kind, None, payload[1])
                return Verdict("slow_heal", payload[0], payload[1])
            if time.time() - t_start > self.cfg.job_timeout_s:
                from elysium_wan_b200.fault_tolerance.liveness import Verdict

                return Verdict("failed", None, "job timeout")

    def _abort_all(self):
        # the channels are picked under the lock and written to outside it: a
        # send to an agent that is slow to read must not hold up the readers
        with self.lock:
            chans = [self.nodes[nid].ch for nid in dict.fromkeys(self.slot_node.values())
                     if self.nodes[nid].connected and not self.nodes[nid].dead]
        for ch in chans:
            try:
                ch.send("ABORT")
            except (OSError, ConnectionError):
                pass
        time.sleep(0.5)

    def _collect(self, spec, run_dir) -> str:
        recs = []
        for losses in self.results.values():
            recs += losses
        recs.sort(key=lambda r: (r["step"], r["mb"]))
        p = os.path.join(run_dir, "losses.json")
        with open(p, "w") as f:
            json.dump({"losses": recs}, f, indent=1)
        return p

