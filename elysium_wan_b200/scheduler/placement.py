"""Placement: bind a recipe (JobSpec) to measured nodes.

Parity: src/wantrain/scheduler/placement.py (`rank_memory_weights` :31,
`memory_order` :52, `stage_speeds` :64, `emulated_links` :69, `place` :84).

- Rank order by memory need: rank 0 holds the deepest stack of live graphs
  (a microbatch lives from its F to its B, n_stages - rank intervals) plus the
  embedding's state, and the last rank holds the logits and the head's state,
  so the largest need gets the largest device.
- The layer cut is proportional to measured stage speed (the exact min-max
  program of `partition.assign_layers`); a wide stage's speed is the sum of
  its replicas', and microbatches are owned in proportion to replica speed
  (IWRR).
- A map that mixes device types is refused before anything is placed: one
  job computes on one device type so one oracle reproduces it.
"""

from __future__ import annotations

from dataclasses import asdict

from elysium_wan_b200.resources.node import mixed_fleet
from elysium_wan_b200.runtime.spec import JobSpec, LinkCfg
from elysium_wan_b200.scheduler.partition import proportional_partition
from elysium_wan_b200.scheduler.solve import stage_live_graphs

BYTES_PER_PARAM_ADAM = 16  # fp32 master 4 + fp32 gradient 4 + moments 8


def activation_graph_bytes(cfg, mb_size: int, n_layers: int = 1) -> float:
    """Activation bytes one microbatch keeps per block on this engine: the
    saved F tensors of `planner.act_bytes` (bf16 on GPUs)."""
    from elysium_wan_b200.scheduler.planner import act_bytes

    return float(n_layers * act_bytes(cfg, mb_size, "cuda")["saved"])


def rank_memory_weights(spec: JobSpec, k_inflight: int = 1) -> list:
    """Relative memory need per rank before layers are cut, in bytes."""
    m = spec.model
    S = spec.stages
    graph = activation_graph_bytes(m, spec.mb_size, max(1, m.n_layer // S))
    emb = m.vocab_size * m.d_model * BYTES_PER_PARAM_ADAM
    logits = 2 * spec.mb_size * m.seq_len * m.vocab_size * 4
    out = []
    for r in range(S):
        w = stage_live_graphs(S, r, k_inflight) * graph
        if r == 0:
            w += emb
        if r == S - 1:
            w += logits + (0 if m.tie_embeddings else emb)
        out.append(w)
    return out


def memory_order(spec: JobSpec, nodes, k_inflight: int = 1) -> list | None:
    """Node index per rank pairing the largest need with the largest memory;
    None when a node cannot state its memory or the counts differ."""
    if len(nodes) != spec.stages or any(not n.memory_bytes() for n in nodes):
        return None
    need = rank_memory_weights(spec, k_inflight)
    by_need = sorted(range(spec.stages), key=lambda r: (-need[r], r))
    by_mem = sorted(range(len(nodes)), key=lambda i: (-nodes[i].memory_bytes(), i))
    slot = dict(zip(by_need, by_mem))
    return [slot[r] for r in range(spec.stages)]


def stage_speeds(groups) -> list:
    """groups[r] = the nodes of stage r; a stage's speed is its replicas' sum."""
    return [sum(n.speed() for n in g) for g in groups]


def emulated_links(groups, emulations) -> list | None:
    """Per-hop WAN shim settings when every node declared an emulation profile
    ({node_id: obj with .enabled and .link_to(region) -> (rtt_ms, mbps)}).
    Hop r joins stage r and r+1; the last entry is the ring wrap."""
    if not emulations or any(e is None or not getattr(e, "enabled", False)
                             for e in emulations.values()):
        return None
    S = len(groups)
    out = []
    for r in range(S):
        a, b = groups[r][0], groups[(r + 1) % S][0]
        link = emulations[a.node_id].link_to(b.region)
        out.append(asdict(LinkCfg(latency_ms=link.rtt_ms / 2.0, bw_mbps=link.mbps)))
    return out


def place(spec: JobSpec, groups, emulations=None, keep_partition: bool = False) -> dict:
    """Fill endpoints, devices, peer weights, the partition and emulated links
    of `spec` in place; groups[r][p] is the NodeInfo holding slot (r, p).
    Returns the rationale dict printed with the plan."""
    mixed = mixed_fleet([n for g in groups for n in g])
    if mixed is not None:
        raise ValueError(mixed)
    if len(groups) != spec.stages:
        raise ValueError(f"{len(groups)} node groups for {spec.stages} stages")
    had_partition = spec.partition is not None
    spec.stage_widths = [len(g) for g in groups]
    spec.endpoints = [[[n.host, int(n.caps.get("data_port", 0)), int(n.caps.get("bind_port", 0))]
                       for n in g] for g in groups]
    devices = [[n.device for n in g] for g in groups]
    flat = {d for row in devices for d in row}
    if len(flat) == 1:
        spec.device, spec.devices = devices[0][0], None
    else:
        spec.devices = devices
    speeds = stage_speeds(groups)
    spec.peer_weights = [[n.speed() / max(m.speed() for m in g) for n in g] for g in groups]
    if not keep_partition and (not had_partition or len(set(speeds)) > 1):
        spec.partition = proportional_partition(spec.model, speeds)
    links = emulated_links(groups, emulations)
    if links is not None:
        spec.links = links
    spec.reschedule()
    return {
        "placement": [[f"{n.name}({n.device})" for n in g] for g in groups],
        "stage_tflops": [round(s, 4) for s in speeds],
        "partition": spec.partition,
        "layers_per_stage": [b - a for a, b in spec.partition],
        "devices": spec.devices or spec.device,
        "emulated_links": links,
    }
