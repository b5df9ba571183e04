"""Link memory: what earlier runs measured on the path between two machines,
and which machines recently proved dead.

Parity: src/wantrain/scheduler/linkmemory.py (`PathRecord` :52, `verdict`
:66, `LinkMemory` :92 with `record_path`, `path`, `record_dead`,
`dead_keys`). A slow path is ranked down and named, never refused; a dead
host is remembered for a TTL because it fails against every peer. Stored as
two JSON files under the coordinator's state directory (atomic replace).
"""

from __future__ import annotations

import json
import os
import re
import threading
import time
from dataclasses import asdict, dataclass, field

SLOW_PATH_MBPS = 100.0
SLOW_PATH_RTT_MS = 80.0
DEAD_HOST_TTL_S = 6 * 3600.0
PENALTY = {"good": 0, "variable": 1, "slow": 2}


def path_key(a: str, b: str) -> str:
    return "|".join(sorted((a, b)))


def subnet24(ip: str | None) -> str | None:
    m = re.fullmatch(r"(\d{1,3}\.\d{1,3}\.\d{1,3})\.\d{1,3}", (ip or "").strip())
    return m.group(1) if m else None


def shares_subnet(ips) -> str | None:
    """The /24 two of the addresses share, if any (one LAN, or two forwards
    through one gateway): reported with the selection, not scored."""
    seen = set()
    for n in (subnet24(i) for i in ips):
        if n is None:
            continue
        if n in seen:
            return n
        seen.add(n)
    return None


@dataclass
class PathRecord:
    a: str
    b: str
    mbps: float  # slower direction of the latest reading
    rtt_ms: float
    measured_at: float
    run_id: str
    samples: int = 1
    run_ids: list = field(default_factory=list)
    worst_mbps: float = 0.0
    best_mbps: float = 0.0


def verdict(p: PathRecord | None) -> str | None:
    """good (every reading clears the floor), variable (some do), slow (none
    does, or the round trip is too long); None when never measured."""
    if p is None:
        return None
    if p.rtt_ms > SLOW_PATH_RTT_MS or p.best_mbps < SLOW_PATH_MBPS:
        return "slow"
    return "variable" if p.worst_mbps < SLOW_PATH_MBPS else "good"


@dataclass
class DeadHost:
    node_key: str
    host: str | None
    reason: str
    at: float
    run_id: str


class LinkMemory:
    def __init__(self, state_dir: str | None = None, dead_ttl_s: float = DEAD_HOST_TTL_S):
        self.state_dir = state_dir
        self.dead_ttl_s = dead_ttl_s
        self._lock = threading.Lock()
        self._paths: dict[str, PathRecord] = {}
        self._dead: dict[str, DeadHost] = {}
        if state_dir:
            os.makedirs(state_dir, exist_ok=True)
            for r in self._load("link-memory.json"):
                p = PathRecord(**r)
                self._paths[path_key(p.a, p.b)] = p
            for r in self._load("dead-hosts.json"):
                d = DeadHost(**r)
                self._dead[d.node_key] = d

    def _load(self, name) -> list:
        try:
            with open(os.path.join(self.state_dir, name)) as f:
                rows = json.load(f)
            return rows if isinstance(rows, list) else []
        except (OSError, ValueError, TypeError):
            return []

    def _save(self, name, rows):
        if not self.state_dir:
            return
        path = os.path.join(self.state_dir, name)
        tmp = f"{path}.{os.getpid()}.tmp"
        with open(tmp, "w") as f:
            json.dump(rows, f, indent=1)
        os.replace(tmp, path)

    def record_path(self, a: str, b: str, mbps: float, rtt_ms: float, run_id: str) -> PathRecord:
        """One reading per run per path (a replay does not count twice); the
        range of readings rides along with the latest."""
        a, b = sorted((a, b))
        with self._lock:
            key = path_key(a, b)
            prev = self._paths.get(key)
            ids = list(prev.run_ids) if prev else []
            if prev and run_id in ids:
                return prev
            ids = (ids + [run_id])[-50:]
            rec = PathRecord(a, b, float(mbps), float(rtt_ms), time.time(), run_id, len(ids), ids,
                             min(prev.worst_mbps, mbps) if prev else mbps,
                             max(prev.best_mbps, mbps) if prev else mbps)
            self._paths[key] = rec
            self._save("link-memory.json", [asdict(p) for p in self._paths.values()])
            return rec

    def path(self, a: str, b: str) -> PathRecord | None:
        return self._paths.get(path_key(a, b))

    def paths(self) -> dict:
        return dict(self._paths)

    def record_dead(self, node_key: str, reason: str, run_id: str, host: str | None = None):
        now = time.time()
        with self._lock:
            self._dead = {k: d for k, d in self._dead.items() if now - d.at < self.dead_ttl_s}
            self._dead[node_key] = DeadHost(node_key, host, reason[:300], now, run_id)
            self._save("dead-hosts.json", [asdict(d) for d in self._dead.values()])

    def dead_keys(self) -> set:
        now = time.time()
        return {k for k, d in self._dead.items() if now - d.at < self.dead_ttl_s}
