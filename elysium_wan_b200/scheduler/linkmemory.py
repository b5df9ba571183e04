"""Memory across runs: how the network path between two machines measured, and
which machines recently failed.

Behaviour of the reference's link memory (src/wantrain/scheduler/linkmemory.py
:52-176, semantics only): a path is graded from its readings -- good when
every reading clears the bandwidth floor, variable when only some do, slow
when none does or its round trip is too long -- and a slow path is ranked
down and named by node selection, never refused; a machine that failed is
avoided for a time-to-live, because a dead host fails against every peer; a
run counts once per path however often its measurement is replayed.

Structure here: the memory is a journal of readings. Each path keeps one
`Reading` per run (the newest runs, at most `KEEP_RUNS`), and everything the
selector asks for (latest rate, slowest and fastest run, the grade) is
derived from that list when asked. Failed machines are `Sighting`s that
expire by age when read. Both live in one JSON document under the
coordinator's state directory, rewritten through a temporary file in the same
directory and an atomic rename.
"""

from __future__ import annotations

import ipaddress
import json
import os
import tempfile
import threading
import time
from dataclasses import asdict, dataclass, field

FLOOR_MBPS = 100.0  # a reading below this rate is slow
MAX_RTT_MS = 80.0  # a path whose latest round trip is longer is slow
DEAD_TTL_S = 6 * 3600.0  # how long a failed machine is avoided
KEEP_RUNS = 50  # readings kept per path
GRADE_RANK = {"good": 0, "variable": 1, "slow": 2}  # selection sorts by this
FILE_NAME = "links.json"


def _ends(a: str, b: str) -> tuple:
    return tuple(sorted((a, b)))


def shares_subnet(addresses) -> str | None:
    """The /24 network that two of the IPv4 addresses share (one LAN, or two
    port forwards through one gateway), else None. Reported with a
    selection, not scored."""
    nets = set()
    for a in addresses:
        try:
            ip = ipaddress.IPv4Address((a or "").strip())
        except ValueError:
            continue
        net = str(ipaddress.IPv4Network(f"{ip}/24", strict=False).network_address)[:-2]
        if net in nets:
            return net
        nets.add(net)
    return None


@dataclass(frozen=True)
class Reading:
    run_id: str
    mbps: float  # slower direction
    rtt_ms: float
    at: float


@dataclass
class PathHistory:
    ends: tuple
    readings: list = field(default_factory=list)  # oldest first, one per run

    @property
    def samples(self) -> int:
        return len(self.readings)

    @property
    def latest(self) -> Reading:
        return self.readings[-1]

    @property
    def mbps(self) -> float:
        return self.latest.mbps

    @property
    def rtt_ms(self) -> float:
        return self.latest.rtt_ms

    @property
    def slowest_mbps(self) -> float:
        return min(r.mbps for r in self.readings)

    @property
    def fastest_mbps(self) -> float:
        return max(r.mbps for r in self.readings)

    def grade(self) -> str:
        if self.rtt_ms > MAX_RTT_MS or self.fastest_mbps < FLOOR_MBPS:
            return "slow"
        return "good" if self.slowest_mbps >= FLOOR_MBPS else "variable"


def verdict(history: PathHistory | None) -> str | None:
    """The grade of a remembered path; None for a path never measured."""
    return None if history is None or not history.readings else history.grade()


@dataclass(frozen=True)
class Sighting:
    node_key: str
    host: str | None
    reason: str
    at: float
    run_id: str


class LinkMemory:
    def __init__(self, state_dir: str | None = None, dead_ttl_s: float = DEAD_TTL_S):
        self.state_dir = state_dir
        self.dead_ttl_s = dead_ttl_s
        self._lock = threading.Lock()
        self._paths: dict = {}  # ends -> PathHistory
        self._dead: dict = {}  # node_key -> Sighting
        if state_dir:
            os.makedirs(state_dir, exist_ok=True)
            self._read()

    # ------------------------------------------------------------ storage
    def _read(self):
        try:
            with open(os.path.join(self.state_dir, FILE_NAME)) as f:
                doc = json.load(f)
        except (OSError, ValueError):
            return
        for row in doc.get("paths", []) if isinstance(doc, dict) else []:
            try:
                h = PathHistory(_ends(*row["ends"]), [Reading(**r) for r in row["readings"]])
            except (KeyError, TypeError, ValueError):
                continue
            if h.readings:
                self._paths[h.ends] = h
        for row in doc.get("dead", []) if isinstance(doc, dict) else []:
            try:
                s = Sighting(**row)
            except TypeError:
                continue
            self._dead[s.node_key] = s

    def _write(self):
        if not self.state_dir:
            return
        doc = {"paths": [{"ends": list(h.ends), "readings": [asdict(r) for r in h.readings]}
                         for h in self._paths.values()],
               "dead": [asdict(s) for s in self._dead.values()]}
        fd, tmp = tempfile.mkstemp(prefix=".links-", dir=self.state_dir)
        with os.fdopen(fd, "w") as f:
            json.dump(doc, f)
        os.replace(tmp, os.path.join(self.state_dir, FILE_NAME))

    # ------------------------------------------------------------ paths
    def record_path(self, a: str, b: str, mbps: float, rtt_ms: float, run_id: str) -> PathHistory:
        """Add this run's reading of the path (a second reading from the same
        run is ignored)."""
        with self._lock:
            h = self._paths.setdefault(_ends(a, b), PathHistory(_ends(a, b)))
            if any(r.run_id == run_id for r in h.readings):
                return h
            h.readings = (h.readings + [Reading(run_id, float(mbps), float(rtt_ms), time.time())])
            h.readings = h.readings[-KEEP_RUNS:]
            self._write()
            return h

    def path(self, a: str, b: str) -> PathHistory | None:
        return self._paths.get(_ends(a, b))

    def paths(self) -> dict:
        return dict(self._paths)

    # ------------------------------------------------------------ failed machines
    def _live_sightings(self, now: float) -> dict:
        return {k: s for k, s in self._dead.items() if now - s.at < self.dead_ttl_s}

    def record_dead(self, node_key: str, reason: str, run_id: str, host: str | None = None):
        with self._lock:
            now = time.time()
            self._dead = self._live_sightings(now)
            self._dead[node_key] = Sighting(node_key, host, reason[:300], now, run_id)
            self._write()

    def dead_keys(self) -> set:
        return set(self._live_sightings(time.time()))
