"""Placement: bind a recipe (JobSpec) to measured nodes.

Reference behaviour (src/wantrain/scheduler/placement.py:31-114, semantics
only): one job computes on one device type (a mixed map is refused before
anything is placed); a stage's layer range is proportional to its measured
speed, a wide stage's speed being the sum of its replicas'; replicas own
microbatches in proportion to their speed (IWRR); the rank that needs the
most memory gets the card with the most memory; nodes that declared a WAN
emulation profile get the per-hop shim settings of their regions.

Structure here: `plan_placement` is a pure function from (spec, node groups,
emulation profiles) to a `Placement` record; `Placement.apply` writes it into
the spec and re-solves ownership and schedule; `place` does both and returns
the rationale. The memory need of a rank is this engine's own model: the
parameter state of its share of the layer list (fp32 master, gradient,
working copy and moments) plus the activations of the microbatches the
zero-bubble order keeps alive on it (scheduler/planner.py
`stage_memory_model`, S - r microbatches in flight on rank r).
"""

from __future__ import annotations

import copy
from dataclasses import asdict, dataclass, field

from elysium_wan_b200.resources.node import mixed_fleet
from elysium_wan_b200.runtime.spec import JobSpec, LinkCfg
from elysium_wan_b200.scheduler.partition import proportional_partition

STATE_BYTES_PER_PARAM = 4 + 4 + 2 + 8  # master, gradient, bf16 working copy, AdamW moments


def _entry_params(cfg, a: int, b: int) -> int:
    from elysium_wan_b200.models.gpt import entry_specs

    n = 0
    for e in range(a, b):
        for s in entry_specs(cfg, e):
            k = 1
            for x in s.shape:
                k *= x
            n += k
    return n


def rank_memory_need(spec: JobSpec) -> list:
    """Bytes each pipeline rank needs under an equal-speed cut: parameter
    state plus the activations of its in-flight microbatches."""
    from elysium_wan_b200.scheduler.planner import stage_memory_model

    S = spec.stages
    view = copy.copy(spec)
    view.partition = proportional_partition(spec.model, [1.0] * S)
    need = []
    for r, (a, b) in enumerate(view.partition):
        mem_f, _, _ = stage_memory_model(view, r)
        state = _entry_params(spec.model, a, b) * STATE_BYTES_PER_PARAM
        need.append(float(state + mem_f * (S - r)))
    return need


def memory_order(spec: JobSpec, nodes) -> list | None:
    """Node index per rank such that the k-th hungriest rank gets the k-th
    largest card (ties keep rank and node order); None when a node does not
    state its memory or the counts differ. Matching sorted needs to sorted
    capacities maximises the smallest capacity / need ratio."""
    if len(nodes) != spec.stages or any(not n.memory_bytes() for n in nodes):
        return None
    need = rank_memory_need(spec)
    ranks = sorted(range(spec.stages), key=lambda r: (-need[r], r))
    cards = sorted(range(len(nodes)), key=lambda i: (-nodes[i].memory_bytes(), i))
    out = [0] * spec.stages
    for r, i in zip(ranks, cards):
        out[r] = i
    return out


def _hop(src, dst, emulations):
    """Shim settings of the hop src -> dst from src's emulation profile; in
    shared-pacer mode also the budgets its frames share with other flows: the
    sender's and the receiver's NIC, and the uplink from src's region to
    dst's when they differ."""
    em = emulations[src.node_id]
    link = em.link_to(dst.region)
    cfg = LinkCfg(latency_ms=link.rtt_ms / 2.0, bw_mbps=link.mbps)
    if em.shared:
        dem = emulations.get(dst.node_id)
        if em.nic_mbps > 0:
            cfg.egress_key, cfg.egress_mbps = src.node_id, em.nic_mbps
        if dem is not None and dem.nic_mbps > 0:
            cfg.ingress_key, cfg.ingress_mbps = dst.node_id, dem.nic_mbps
        if src.region != dst.region and link.mbps > 0:
            cfg.uplink_key, cfg.uplink_mbps = f"{src.region}>{dst.region}", link.mbps
    return asdict(cfg)


def emulated_links(groups, emulations) -> list | None:
    """spec.links from the nodes' WAN emulation profiles, or None unless every
    node declared one. links[r] joins stage r and r + 1 (the last entry joins
    the last stage back to the first, as the JobSpec format has it)."""
    profiles = emulations or {}
    if not profiles or not all(getattr(e, "enabled", False) for e in profiles.values()):
        return None
    heads = [g[0] for g in groups]
    return [_hop(heads[r], heads[(r + 1) % len(heads)], profiles) for r in range(len(heads))]


def emulated_mesh_links(groups, emulations) -> list | None:
    """Per stage, the shim settings of the links among its replicas
    ({"p>q": link}, from p's emulation profile toward q's region), or None
    unless every node declared a profile."""
    profiles = emulations or {}
    if not profiles or not all(getattr(e, "enabled", False) for e in profiles.values()):
        return None
    return [{f"{p}>{q}": _hop(g[p], g[q], profiles) for p in range(len(g)) for q in range(len(g))
             if p != q} for g in groups]


@dataclass
class Placement:
    widths: list
    endpoints: list
    devices: list  # devices[stage][peer]
    stage_speed: list
    peer_weights: list
    partition: list | None  # None: keep the spec's
    links: list | None
    names: list = field(default_factory=list)
    mesh_links: list | None = None

    def apply(self, spec: JobSpec) -> JobSpec:
        spec.stage_widths = list(self.widths)
        spec.endpoints = self.endpoints
        one = {d for row in self.devices for d in row}
        if len(one) == 1:
            spec.device, spec.devices = next(iter(one)), None
        else:
            spec.devices = self.devices
        spec.peer_weights = self.peer_weights
        if self.partition is not None:
            spec.partition = self.partition
        if self.links is not None:
            spec.links = self.links
        if self.mesh_links is not None:
            spec.mesh_links = self.mesh_links
        return spec.reschedule()

    def rationale(self, spec: JobSpec) -> dict:
        return {"placement": self.names, "stage_tflops": [round(s, 4) for s in self.stage_speed],
                "partition": spec.partition,
                "layers_per_stage": [b - a for a, b in spec.partition],
                "devices": spec.devices or spec.device, "emulated_links": self.links}


def plan_placement(spec: JobSpec, groups, emulations=None, keep_partition: bool = False) -> Placement:
    """groups[r][p] is the NodeInfo that will hold slot (r, p)."""
    problem = mixed_fleet([n for g in groups for n in g])
    if problem is not None:
        raise ValueError(problem)
    if len(groups) != spec.stages:
        raise ValueError(f"{len(groups)} node groups for {spec.stages} stages")
    speed = [sum(n.speed() for n in g) for g in groups]
    fastest = [max(n.speed() for n in g) for g in groups]
    cut = None
    if not keep_partition and (spec.partition is None or len(set(speed)) > 1):
        cut = proportional_partition(spec.model, speed)
    return Placement(
        widths=[len(g) for g in groups],
        endpoints=[[[n.host, int(n.caps.get("data_port", 0)), int(n.caps.get("bind_port", 0))]
                    for n in g] for g in groups],
        devices=[[n.device for n in g] for g in groups],
        stage_speed=speed,
        peer_weights=[[n.speed() / top for n in g] for g, top in zip(groups, fastest)],
        partition=cut,
        links=emulated_links(groups, emulations),
        names=[[f"{n.name}({n.device})" for n in g] for g in groups],
        mesh_links=emulated_mesh_links(groups, emulations))


def place(spec: JobSpec, groups, emulations=None, keep_partition: bool = False) -> dict:
    """Bind `spec` to the node groups in place; returns the rationale printed
    with the plan."""
    p = plan_placement(spec, groups, emulations, keep_partition)
    p.apply(spec)
    return p.rationale(spec)
