"""Failure detection: convict a dead worker quickly, and only the right one.

Same verdict semantics as the reference's LivenessJudge
(src/wantrain/fault_tolerance/liveness.py:1-344):
  S1  an agent's control connection is gone past the reconnect grace;
  S2  a slot's stage process ended without its done marker (killed from
      outside) -- convicts at once; a heartbeat that says "stage gone" gets
      exit_report_grace_s for the explaining exit report first;
  S3  a slot exited with "peer connection lost" while another is silent: the
      silent one is the suspect;
  S4  no optimizer step fleet-wide for max(stall_floor_s, stall_steps x median
      step) (first_step_timeout_s before any step), judged only while some
      slot still owes a step; after the final step, quiet is shutdown,
      bounded by shutdown_limit_s.
Heartbeat silence is a first strike; conviction needs a second look at least
strike_gap_s later. Two or more convictions at once mean the network or the
coordinator, not a worker: "failed", no heal. A stage that raised (exit code
with the done marker, no lost peer) is deterministic: "failed". Everyone alive
with a lost peer or no progress: "stalled" (restart in place).

On the B200 box the stages talk over NCCL; a dead rank surfaces to its peers
as a collective error or timeout, which the stage reports as a lost peer.
"""

from __future__ import annotations

import statistics
import time
from dataclasses import dataclass, field

STALL_FLOOR_S = 90.0
STALL_STEPS = 6
STRIKE_GAP_S = 8.0
HEARTBEAT_TIMEOUT_S = 15.0
RECONNECT_GRACE_S = 30.0
SHUTDOWN_LIMIT_S = 600.0
PEER_LOST = "peer connection lost"
DONE_MARKER = "WT_DONE"


@dataclass
class SlotState:
    slot: tuple
    node_id: str
    launched: bool = False
    connected: bool = True
    disconnected_at: float | None = None
    last_heartbeat: float = 0.0
    stage_alive: bool | None = None
    exit_code: int | None = None
    done_marker: bool = False
    log_tail: str = ""
    progress: list = field(default_factory=list)  # [(step, t)]
    suspect_at: float | None = None
    started_at: float = 0.0
    gone_since: float | None = None
    peer_lost_at: float | None = None
    start_step: int = 0

    def last_step(self):
        return self.progress[-1][0] if self.progress else None

    def add_progress(self, step: int, t: float, final_step: int | None) -> bool:
        """Only steps of this attempt, strictly increasing, count as progress."""
        if step < self.start_step or (final_step is not None and step > final_step):
            return False
        if self.progress and step <= self.progress[-1][0]:
            return False
        self.progress.append((step, t))
        return True

    @property
    def lost_peer(self) -> bool:
        return self.exit_code not in (None, 0) and PEER_LOST in self.log_tail

    @property
    def running(self) -> bool:
        return self.exit_code is None


@dataclass
class Verdict:
    kind: str  # ok | suspect | convict | stalled | failed | done
    slot: tuple | None = None
    why: str = ""
    slots: list = field(default_factory=list)


def median_step_s(states):
    pts = sorted((s, t) for st in states for (s, t) in st.progress)
    gaps = [(t1 - t0) / (s1 - s0) for (s0, t0), (s1, t1) in zip(pts, pts[1:]) if s1 > s0 and t1 > t0]
    return statistics.median(gaps[-12:]) if len(gaps) >= 3 else None


def last_progress_at(states):
    ts = [t for st in states for (_, t) in st.progress]
    if ts:
        return max(ts)
    started = [st.started_at for st in states if st.launched and st.started_at]
    return max(started) if started else None


class LivenessJudge:
    def __init__(self, heartbeat_timeout_s=HEARTBEAT_TIMEOUT_S, reconnect_grace_s=RECONNECT_GRACE_S,
                 stall_floor_s=STALL_FLOOR_S, stall_steps=STALL_STEPS, strike_gap_s=STRIKE_GAP_S,
                 first_step_timeout_s=600.0, exit_report_grace_s=10.0, final_step=None,
                 shutdown_limit_s=SHUTDOWN_LIMIT_S):
        self.heartbeat_timeout_s = heartbeat_timeout_s
        self.reconnect_grace_s = reconnect_grace_s
        self.stall_floor_s = stall_floor_s
        self.stall_steps = stall_steps
        self.strike_gap_s = strike_gap_s
        self.first_step_timeout_s = first_step_timeout_s
        self.exit_report_grace_s = exit_report_grace_s
        self.final_step = final_step
        self.shutdown_limit_s = shutdown_limit_s

    # ----------------------------------------------------------------- signals
    def _killed(self, st: SlotState, now: float):
        """S2: the stage ended without its done marker (or vanished unexplained)."""
        if st.exit_code is None:
            if st.stage_alive is False and st.launched and st.connected:
                st.gone_since = st.gone_since if st.gone_since is not None else now
                if now - st.gone_since > self.exit_report_grace_s:
                    return "the stage process is gone and no exit was reported"
            else:
                st.gone_since = None
            return None
        if st.exit_code != 0 and not st.done_marker:
            return (f"the stage process died with code {st.exit_code} and no done marker "
                    f"(killed from outside: OOM killer, reboot, restart)")
        return None

    def _disconnected_too_long(self, st: SlotState, now: float):
        """S1: a closed control connection that did not come back in the grace."""
        if st.running and not st.connected and st.disconnected_at is not None \
                and now - st.disconnected_at > self.reconnect_grace_s:
            return (f"worker unreachable: control connection lost {now - st.disconnected_at:.0f}s "
                    f"ago and not re-established")
        return None

    def _silent(self, st: SlotState, now: float):
        if st.connected and st.last_heartbeat and now - st.last_heartbeat > self.heartbeat_timeout_s:
            return f"no heartbeat for {now - st.last_heartbeat:.0f}s"
        return None

    def _shutting_down(self, launched) -> bool:
        f = self.final_step
        return f is not None and all(st.exit_code == 0 or st.last_step() == f or st.start_step > f
                                     for st in launched)

    def _strike(self, st: SlotState, why: str, now: float) -> Verdict:
        if st.suspect_at is None:
            st.suspect_at = now
            return Verdict("suspect", st.slot, f"first strike: {why}")
        if now - st.suspect_at >= self.strike_gap_s:
            return Verdict("convict", st.slot,
                           f"{why}; still failing {now - st.suspect_at:.0f}s after the first strike")
        return Verdict("suspect", st.slot, f"awaiting second strike: {why}")

    # ----------------------------------------------------------------- verdict
    def judge(self, states, now: float | None = None) -> Verdict:
        now = time.time() if now is None else now
        launched = [st for st in states if st.launched]
        if not launched:
            return Verdict("ok")
        if all(st.exit_code == 0 for st in launched):
            return Verdict("done")

        convicted = [(st, w) for st in launched if (w := self._killed(st, now))]
        convicted += [(st, w) for st in launched if (w := self._disconnected_too_long(st, now))]
        if len(convicted) == 1:
            return Verdict("convict", convicted[0][0].slot, convicted[0][1])
        if len(convicted) > 1:
            names = ", ".join(str(s.slot) for s, _ in convicted)
            return Verdict("failed", None,
                           f"{len(convicted)} slots failed at once ({names}): a network or "
                           f"coordinator problem, not one dead worker", [s.slot for s, _ in convicted])

        waiting = [st for st in launched if st.running and not st.connected]
        if waiting:
            since = now - (waiting[0].disconnected_at or now)
            return Verdict("suspect", waiting[0].slot,
                           f"control connection lost {since:.0f}s ago; waiting up to "
                           f"{self.reconnect_grace_s:.0f}s for the worker to reconnect",
                           [w.slot for w in waiting])

        crashed = [st for st in launched
                   if st.exit_code not in (None, 0) and st.done_marker and PEER_LOST not in st.log_tail]
        if crashed:
            st = crashed[0]
            return Verdict("failed", st.slot, f"slot {st.slot} raised (exit {st.exit_code}); this is "
                                              f"the run, not the hardware. Log tail: {st.log_tail[-300:]}")

        peer_lost = any(st.lost_peer for st in launched)
        silent = [st for st in launched if st.running]
        step_s = median_step_s(launched)
        seen = last_progress_at(launched)
        limit = self.first_step_timeout_s if step_s is None else max(self.stall_floor_s,
                                                                      self.stall_steps * step_s)
        if self._shutting_down(launched):
            ts = [t for st in launched for (_, t) in st.progress] + \
                 [st.started_at for st in launched if st.started_at]
            quiet = now - max(ts) if ts else 0.0
            if not (peer_lost and silent) and quiet > self.shutdown_limit_s:
                return Verdict("failed", None,
                               f"shutdown exceeded {self.shutdown_limit_s:.0f}s after the final step",
                               [st.slot for st in launched])
            stalled = False
        else:
            stalled = seen is not None and now - seen > limit
        suspects = silent if peer_lost else (launched if stalled else [])
        if not suspects:
            for st in launched:
                if st.running and (w := self._silent(st, now)):
                    return self._strike(st, w, now)
            for st in launched:
                st.suspect_at = None
            return Verdict("ok")
        unreachable = [(st, w) for st in suspects if st.running and (w := self._silent(st, now))]
        if len(unreachable) == 1:
            return self._strike(unreachable[0][0], unreachable[0][1], now)
        if len(unreachable) > 1:
            return Verdict("suspect", None, f"{len(unreachable)} slots unreachable at once; waiting "
                                            f"for the reconnect grace before judging",
                           [s.slot for s, _ in unreachable])
        for st in suspects:
            st.suspect_at = None
        if peer_lost:
            lost = []
            for st in launched:
                if st.lost_peer:
                    st.peer_lost_at = st.peer_lost_at if st.peer_lost_at is not None else now
                    lost.append(st.peer_lost_at)
            if silent and now - min(lost) <= self.exit_report_grace_s:
                return Verdict("suspect", None,
                               f"a stage lost its peer; waiting up to {self.exit_report_grace_s:.0f}s "
                               f"for the silent slots' exit reports", [st.slot for st in silent])
        why = ("a stage lost its peer while every worker is alive" if peer_lost else
               f"no optimizer step fleet-wide for {now - (seen or now):.0f}s (limit {limit:.0f}s) "
               f"while every worker is alive")
        return Verdict("stalled", None, why, [st.slot for st in launched])
