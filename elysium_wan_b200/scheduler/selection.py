"""Node selection: which registered workers a job runs on.

Parity: src/wantrain/scheduler/selection.py (`SelectionPolicy` :45,
`distinct_addresses` :105, `candidate_fleets` :138, `select_nodes` :287).
Filters, in order: remembered-dead hosts, device type, GPU-name substring,
uplink floor (only while enough nodes remain), compute-capability window,
device memory floor, one device class per fleet (a pool that no single class
can field is refused as MIXED-FLEET). Candidates group by region (unless
any-region) and by GPU model or series; the best is ranked by the worst
remembered path verdict, then total speed, then the smallest memory. The
nodes not chosen are the spares fault tolerance draws from.

On one B200 box every worker shares an address, so `distinct_hosts` is off by
default here (the reference defaults it on for WAN fleets).
"""

from __future__ import annotations

import re
from dataclasses import dataclass, field

from elysium_wan_b200.scheduler.linkmemory import GRADE_RANK, LinkMemory, shares_subnet, verdict

MIN_UPLINK_MBPS = 200.0


def gpu_name(n) -> str:
    return str(n.caps.get("gpu_name") or n.caps.get("gpu") or n.device_class or "")


def gpu_series(name: str) -> str | None:
    """Consumer series of a device name ("RTX 40-series"), None otherwise."""
    m = re.search(r"\b(RTX|GTX)\s?(\d{2})\d{2}(?!\d)", name or "", re.I)
    return f"{m.group(1).upper()} {m.group(2)}-series" if m else None


def node_key(n) -> str:
    return f"{n.name}@{n.host}"


def cap_int(n) -> int:
    """Compute capability as an integer (sm_100 -> 1000), 0 if unknown."""
    cc = n.caps.get("compute_capability")
    if isinstance(cc, (list, tuple)) and len(cc) == 2:
        return int(cc[0]) * 100 + int(cc[1]) * 10
    return 0


@dataclass
class SelectionPolicy:
    group_by: str = "any"  # any | model | series | region
    same_region: bool = True
    distinct_hosts: bool = False
    min_vram_bytes: int = 0
    min_compute_cap: int = 0
    max_compute_cap: int = 0
    min_uplink_mbps: float = MIN_UPLINK_MBPS
    gpu: str | None = None
    devices: tuple | None = None


@dataclass
class Candidate:
    region: str
    group: str
    nodes: list

    def total_speed(self) -> float:
        return sum(n.speed() for n in self.nodes)

    def min_memory(self) -> float:
        return min((n.memory_bytes() or 0.0) for n in self.nodes)


@dataclass
class Selection:
    ok: bool
    chosen: list = field(default_factory=list)
    spares: list = field(default_factory=list)
    reason: str | None = None
    note: str | None = None
    alternatives: list = field(default_factory=list)


def _hop(a, b, memory):
    return None if memory is None else verdict(memory.path(a.host, b.host))


def _penalty(fleet, memory) -> int:
    return max([GRADE_RANK[v] for v in (_hop(a, b, memory) for a, b in zip(fleet, fleet[1:])) if v]
               or [0])


def _rank(n):
    return (-n.speed(), -(n.memory_bytes() or 0.0), n.node_id)


def distinct_addresses(nodes, n: int, distinct_hosts: bool, memory: LinkMemory | None) -> list:
    """The fastest n nodes (on distinct addresses when asked), avoiding pairs
    a previous run measured as not good (trying each node as the seed, fastest
    first); falls back to ignoring the memory."""
    order = sorted(nodes, key=_rank)

    def greedy(avoid, seed=None):
        hosts, out = set(), []
        for o in ([seed] if seed is not None else []) + [x for x in order if x is not seed]:
            if distinct_hosts and o.host in hosts:
                continue
            if avoid and any((_hop(p, o, memory) or "good") != "good" for p in out):
                continue
            hosts.add(o.host)
            out.append(o)
            if len(out) == n:
                break
        return out

    if memory is not None:
        # Seed with each node in speed order, so a fast node whose paths are
        # all bad does not spoil every fleet that would start from it.
        for seed in order:
            clean = greedy(True, seed)
            if len(clean) == n:
                return clean
    return greedy(False)


def _group_key(n, group_by: str) -> str:
    if group_by == "model":
        return gpu_name(n)
    if group_by == "series":
        return gpu_series(gpu_name(n)) or gpu_name(n)
    return "*"


def candidate_fleets(pool, n: int, policy: SelectionPolicy | None = None,
                     memory: LinkMemory | None = None, dead: set | None = None):
    """(candidates best first, reason when there are none)."""
    pol = policy or SelectionPolicy()
    if n < 1:
        return [], "a fleet needs at least one node"
    dead = set(dead or ()) | (memory.dead_keys() if memory else set())
    nodes = [x for x in pool if node_key(x) not in dead and x.alive]
    seen = len(nodes)
    if pol.devices:
        nodes = [x for x in nodes if x.device.split(":")[0] in pol.devices]
    if pol.gpu:
        nodes = [x for x in nodes if pol.gpu.lower() in gpu_name(x).lower()]
        if not nodes:
            return [], f'no registered node matches "{pol.gpu}" ({seen} seen)'
    fat = [x for x in nodes if float(x.caps.get("uplink_mbps") or 1e12) >= pol.min_uplink_mbps]
    if len(fat) >= n:
        nodes = fat
    if pol.min_compute_cap:
        ok = [x for x in nodes if cap_int(x) >= pol.min_compute_cap]
        if len(ok) < n:
            return [], (f"fewer than {n} nodes have compute capability "
                        f"sm_{pol.min_compute_cap // 10} or newer")
        nodes = ok
    if pol.max_compute_cap:
        ok = [x for x in nodes if cap_int(x) <= pol.max_compute_cap]
        if len(ok) < n:
            return [], (f"fewer than {n} nodes are within this runtime's kernels "
                        f"(sm_{pol.max_compute_cap // 10} at most)")
        nodes = ok
    if pol.min_vram_bytes:
        ok = [x for x in nodes if (x.memory_bytes() or 0) >= pol.min_vram_bytes]
        if len(ok) < n:
            return [], f"fewer than {n} nodes have {pol.min_vram_bytes / 2**30:.1f} GiB of memory"
        nodes = ok
    classes: dict = {}
    for x in nodes:
        classes.setdefault(x.device_class, []).append(x)
    if len(classes) > 1 and not any(
            len(distinct_addresses(g, n, pol.distinct_hosts, memory)) == n for g in classes.values()):
        counts = ", ".join(f"{k}: {len(v)}" for k, v in sorted(classes.items()))
        return [], (f"MIXED-FLEET: no single device class can field {n} nodes ({counts}); one "
                    f"job computes on one device class")
    regions: dict = {}
    for x in nodes:
        regions.setdefault(x.region if pol.same_region else "*", []).append(x)
    cands = []
    for region, group in regions.items():
        keyed: dict = {}
        for x in group:
            keyed.setdefault(f"{x.device_class}|{_group_key(x, pol.group_by)}", []).append(x)
        for key, same in keyed.items():
            picked = distinct_addresses(same, n, pol.distinct_hosts, memory)
            if len(picked) == n:
                cands.append(Candidate(region, key, picked))
    if not cands:
        where = "single region " if pol.same_region else ""
        return [], (f"no {where}group can field {n} nodes ({len(nodes)} eligible across "
                    f"{len(regions)} region(s))")
    cands.sort(key=lambda c: (_penalty(c.nodes, memory), -c.total_speed(), -c.min_memory(),
                              c.region, c.group))
    return cands, None


def select_nodes(pool, n: int, policy: SelectionPolicy | None = None,
                 memory: LinkMemory | None = None, dead: set | None = None) -> Selection:
    """Pick n workers that form a pipeline; the rest are spares."""
    cands, reason = candidate_fleets(pool, n, policy, memory, dead)
    if not cands:
        return Selection(ok=False, reason=reason, spares=list(pool))
    win = cands[0]
    chosen = list(win.nodes)
    ids = {x.node_id for x in chosen}
    spares = sorted([x for x in pool if x.node_id not in ids], key=_rank)
    notes = [f"{n} node(s) in {win.region}: " + ", ".join(f"{x.name}({x.device})" for x in chosen)]
    worst = None
    for a, b in zip(chosen, chosen[1:]):
        p = memory.path(a.host, b.host) if memory else None
        if p and (worst is None or p.slowest_mbps < worst.slowest_mbps):
            worst = p
    if worst is not None:
        v = verdict(worst)
        notes.append(f"{'WARNING: ' if v != 'good' else ''}a hop was measured at "
                     f"{worst.slowest_mbps:.0f}-{worst.fastest_mbps:.0f} Mbps, RTT {worst.rtt_ms:.0f} ms "
                     f"({v})")
    net = shares_subnet({x.host for x in chosen})
    if net and worst is None:
        notes.append(f"nodes share {net}.0/24 on different addresses")
    alts = [dict(region=c.region, group=c.group, nodes=[x.name for x in c.nodes],
                 total_tflops=round(c.total_speed(), 3)) for c in cands[1:4]]
    return Selection(ok=True, chosen=chosen, spares=spares, note="; ".join(notes),
                     alternatives=alts)
