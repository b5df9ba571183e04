"""Failure detection for one attempt of a job: which slot, if any, is dead.

The verdicts and their rules are the reference's public behaviour
(src/wantrain/fault_tolerance/liveness.py:1-344, semantics only): kinds ok,
suspect, convict, stalled, failed and done, from four signals --

  S1  an agent's control connection stays closed past the reconnect grace;
  S2  a stage process ended without its done marker (killed from outside), or
      a heartbeat says the process is gone and no exit report explains it
      within the exit-report grace;
  S3  a stage ended on a lost peer while another slot is silent: the silent
      slot is the suspect;
  S4  no optimizer step anywhere for max(stall floor, stall steps x median
      step time) (the first-step timeout before any step), judged only while
      some slot still owes a step; after the final step quiet is shutdown,
      bounded by the shutdown limit.

Heartbeat silence alone never convicts on first sight: it is a strike, and a
conviction needs a second look at least the strike gap later. Hard evidence
(S1, S2) against two or more slots at once points at the network or the
coordinator: the job fails, nobody is healed. A stage that raised an error of
its own (exit code with the done marker, no lost peer) is deterministic and
fails the job. Everyone alive but a lost peer or no progress is a stall
(restart in place).

This module is built as a decision table. `judge()` first reduces the slots to
facts (`_Facts`: per-slot evidence plus fleet-wide quantities), then walks
`RULES` in order; the first rule whose test holds produces the verdict. The
only memory the judge keeps between calls (first-strike times, when a stage
was first reported gone, when a lost peer was first seen) lives in the judge,
keyed by slot, so the slot records the coordinator fills hold reported facts
only. On the B200 box stages talk over NCCL: a dead rank reaches its peers as
a collective error or timeout, which the stage reports as a lost peer.
"""

from __future__ import annotations

import statistics
import time
from dataclasses import dataclass, field
from typing import Callable

PEER_LOST = "peer connection lost"
DONE_MARKER = "WT_DONE"

# Defaults of the judge's clocks (seconds unless named otherwise).
HEARTBEAT_TIMEOUT_S = 15.0
RECONNECT_GRACE_S = 30.0
STALL_FLOOR_S = 90.0
STALL_STEPS = 6
STRIKE_GAP_S = 8.0
SHUTDOWN_LIMIT_S = 600.0


@dataclass
class SlotState:
    """What the coordinator has been told about one slot of this attempt."""

    slot: tuple
    node_id: str
    launched: bool = False
    started_at: float = 0.0
    start_step: int = 0  # first step this attempt runs (a resume starts later)
    # control connection of the slot's agent
    connected: bool = True
    disconnected_at: float | None = None
    last_heartbeat: float = 0.0
    stage_alive: bool | None = None  # the agent's last word on its stage process
    # the stage's exit report
    exit_code: int | None = None
    done_marker: bool = False
    log_tail: str = ""
    progress: list = field(default_factory=list)  # [(step, time)] strictly increasing

    def add_progress(self, step: int, t: float, final_step: int | None) -> bool:
        """Record a finished step; only steps of this attempt, in increasing
        order and not past the final step, count."""
        last = self.progress[-1][0] if self.progress else self.start_step - 1
        if step <= last or (final_step is not None and step > final_step):
            return False
        self.progress.append((step, t))
        return True

    def last_step(self):
        return self.progress[-1][0] if self.progress else None

    @property
    def running(self) -> bool:
        return self.exit_code is None

    @property
    def ended_on_lost_peer(self) -> bool:
        return self.exit_code not in (None, 0) and PEER_LOST in self.log_tail


@dataclass
class Verdict:
    kind: str  # ok | suspect | convict | stalled | failed | done
    slot: tuple | None = None
    why: str = ""
    slots: list = field(default_factory=list)


def median_step_s(states) -> float | None:
    """Median seconds per step over the fleet's recent progress reports (the
    last 12 gaps), None until three gaps exist."""
    points = sorted(p for st in states for p in st.progress)
    rates = []
    for (s0, t0), (s1, t1) in zip(points, points[1:]):
        if s1 > s0 and t1 > t0:
            rates.append((t1 - t0) / (s1 - s0))
    return statistics.median(rates[-12:]) if len(rates) >= 3 else None


def last_progress_at(states) -> float | None:
    """Time of the newest step report, else of the newest launch."""
    stamps = [t for st in states for _, t in st.progress]
    if not stamps:
        stamps = [st.started_at for st in states if st.launched and st.started_at]
    return max(stamps) if stamps else None


@dataclass
class _Evidence:
    st: SlotState
    hard: str | None = None  # S1 / S2: convicts without a second look
    reconnecting: bool = False  # connection down, still inside the grace
    quiet: str | None = None  # heartbeat silence: a strike
    raised: bool = False  # the stage's own error (deterministic)


@dataclass
class _Facts:
    now: float
    launched: list
    ev: list  # _Evidence per launched slot
    all_clean: bool = False
    peer_lost: bool = False
    step_s: float | None = None
    last_seen: float | None = None
    limit: float = 0.0
    past_final: bool = False
    stalled: bool = False
    quiet_since_final: float = 0.0

    @property
    def hard(self):
        return [e for e in self.ev if e.hard]

    @property
    def reconnecting(self):
        return [e for e in self.ev if e.reconnecting]

    @property
    def raised(self):
        return [e for e in self.ev if e.raised]

    @property
    def running(self):
        return [e for e in self.ev if e.st.running]

    @property
    def suspects(self):
        """S3: the running slots when a stage lost its peer; S4: everyone
        when the fleet stalled; else nobody."""
        if self.peer_lost:
            return self.running
        return list(self.ev) if self.stalled else []

    @property
    def silent_suspects(self):
        return [e for e in self.suspects if e.st.running and e.quiet]


@dataclass(frozen=True)
class Rule:
    name: str
    holds: Callable  # (judge, facts) -> bool
    verdict: Callable  # (judge, facts) -> Verdict


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
        # memory between calls, keyed by slot
        self.first_strike: dict = {}
        self.gone_since: dict = {}
        self.peer_lost_seen: dict = {}

    # ------------------------------------------------------------ evidence
    def _evidence(self, st: SlotState, now: float) -> _Evidence:
        e = _Evidence(st)
        if st.running:
            gone = st.stage_alive is False and st.connected
            if gone:
                since = self.gone_since.setdefault(st.slot, now)
                if now - since > self.exit_report_grace_s:
                    e.hard = "the stage process is gone and no exit was reported"
            else:
                self.gone_since.pop(st.slot, None)
            if not st.connected and st.disconnected_at is not None:
                down = now - st.disconnected_at
                if down > self.reconnect_grace_s:
                    e.hard = e.hard or (f"worker unreachable: control connection lost {down:.0f}s "
                                        f"ago and not re-established")
                else:
                    e.reconnecting = True
            elif not st.connected:
                e.reconnecting = True
            if st.connected and st.last_heartbeat and \
                    now - st.last_heartbeat > self.heartbeat_timeout_s:
                e.quiet = f"no heartbeat for {now - st.last_heartbeat:.0f}s"
        elif st.exit_code != 0:
            if not st.done_marker:
                e.hard = (f"the stage process died with code {st.exit_code} and no done marker "
                          f"(killed from outside: OOM killer, reboot, restart)")
            elif not st.ended_on_lost_peer:
                e.raised = True
        return e

    def _facts(self, states, now: float) -> _Facts:
        launched = [st for st in states if st.launched]
        f = _Facts(now, launched, [self._evidence(st, now) for st in launched])
        if not launched:
            return f
        f.all_clean = all(st.exit_code == 0 for st in launched)
        f.peer_lost = any(st.ended_on_lost_peer for st in launched)
        f.step_s = median_step_s(launched)
        f.last_seen = last_progress_at(launched)
        f.limit = self.first_step_timeout_s if f.step_s is None else \
            max(self.stall_floor_s, self.stall_steps * f.step_s)
        fin = self.final_step
        f.past_final = fin is not None and all(
            st.exit_code == 0 or st.last_step() == fin or st.start_step > fin for st in launched)
        if f.past_final:
            stamps = [t for st in launched for _, t in st.progress] + \
                [st.started_at for st in launched if st.started_at]
            f.quiet_since_final = now - max(stamps) if stamps else 0.0
        else:
            f.stalled = f.last_seen is not None and now - f.last_seen > f.limit
        return f

    # ------------------------------------------------------------ verdicts
    def _strike(self, e: _Evidence, now: float) -> Verdict:
        first = self.first_strike.get(e.st.slot)
        if first is None:
            self.first_strike[e.st.slot] = now
            return Verdict("suspect", e.st.slot, f"first strike: {e.quiet}")
        if now - first >= self.strike_gap_s:
            return Verdict("convict", e.st.slot,
                           f"{e.quiet}; still failing {now - first:.0f}s after the first strike")
        return Verdict("suspect", e.st.slot, f"awaiting second strike: {e.quiet}")

    def _clear_strikes(self, evs):
        for e in evs:
            self.first_strike.pop(e.st.slot, None)

    def _healthy(self, f: _Facts) -> Verdict:
        for e in f.running:
            if e.quiet:
                return self._strike(e, f.now)
        self._clear_strikes(f.ev)
        return Verdict("ok")

    def _awaiting_exit_reports(self, f: _Facts) -> bool:
        if not (f.peer_lost and f.running):
            return False
        seen = [self.peer_lost_seen.setdefault(e.st.slot, f.now)
                for e in f.ev if e.st.ended_on_lost_peer]
        return f.now - min(seen) <= self.exit_report_grace_s

    def judge(self, states, now: float | None = None) -> Verdict:
        now = time.time() if now is None else now
        f = self._facts(states, now)
        for rule in RULES:
            if rule.holds(self, f):
                return rule.verdict(self, f)
        raise AssertionError("the last rule always holds")


def _one_hard(j, f):
    e = f.hard[0]
    return Verdict("convict", e.st.slot, e.hard)


def _many_hard(j, f):
    slots = [e.st.slot for e in f.hard]
    return Verdict("failed", None, f"{len(slots)} slots failed at once "
                                   f"({', '.join(map(str, slots))}): a network or coordinator "
                                   f"problem, not one dead worker", slots)


def _reconnect_wait(j, f):
    e = f.reconnecting[0]
    down = f.now - (e.st.disconnected_at or f.now)
    return Verdict("suspect", e.st.slot,
                   f"control connection lost {down:.0f}s ago; waiting up to "
                   f"{j.reconnect_grace_s:.0f}s for the worker to reconnect",
                   [x.st.slot for x in f.reconnecting])


def _deterministic(j, f):
    st = f.raised[0].st
    return Verdict("failed", st.slot, f"slot {st.slot} raised (exit {st.exit_code}); this is the "
                                      f"run, not the hardware. Log tail: {st.log_tail[-300:]}")


def _shutdown_overdue(j, f):
    return Verdict("failed", None, f"shutdown exceeded {j.shutdown_limit_s:.0f}s after the final "
                                   f"step", [st.slot for st in f.launched])


def _several_silent(j, f):
    return Verdict("suspect", None, f"{len(f.silent_suspects)} slots unreachable at once; waiting "
                                    f"for the reconnect grace before judging",
                   [e.st.slot for e in f.silent_suspects])


def _exit_report_wait(j, f):
    j._clear_strikes(f.suspects)
    return Verdict("suspect", None, f"a stage lost its peer; waiting up to "
                                    f"{j.exit_report_grace_s:.0f}s for the silent slots' exit "
                                    f"reports", [e.st.slot for e in f.running])


def _stalled(j, f):
    j._clear_strikes(f.suspects)
    why = ("a stage lost its peer while every worker is alive" if f.peer_lost else
           f"no optimizer step fleet-wide for {f.now - (f.last_seen or f.now):.0f}s "
           f"(limit {f.limit:.0f}s) while every worker is alive")
    return Verdict("stalled", None, why, [st.slot for st in f.launched])


# The decision table, walked top to bottom; the first rule that holds decides.
RULES = (
    Rule("nothing launched", lambda j, f: not f.launched, lambda j, f: Verdict("ok")),
    Rule("every stage exited cleanly", lambda j, f: f.all_clean, lambda j, f: Verdict("done")),
    Rule("S1/S2 against one slot", lambda j, f: len(f.hard) == 1, _one_hard),
    Rule("S1/S2 against several slots", lambda j, f: len(f.hard) > 1, _many_hard),
    Rule("connection down inside the grace", lambda j, f: bool(f.reconnecting), _reconnect_wait),
    Rule("a stage raised its own error", lambda j, f: bool(f.raised), _deterministic),
    Rule("shutdown past its limit",
         lambda j, f: f.past_final and not (f.peer_lost and f.running)
         and f.quiet_since_final > j.shutdown_limit_s, _shutdown_overdue),
    Rule("no S3/S4 suspects", lambda j, f: not f.suspects, lambda j, f: j._healthy(f)),
    Rule("one suspect is silent", lambda j, f: len(f.silent_suspects) == 1,
         lambda j, f: j._strike(f.silent_suspects[0], f.now)),
    Rule("several suspects are silent", lambda j, f: len(f.silent_suspects) > 1, _several_silent),
    Rule("a lost peer, exit reports pending", lambda j, f: j._awaiting_exit_reports(f),
         _exit_report_wait),
    Rule("everyone alive, no progress", lambda j, f: True, _stalled),
)
