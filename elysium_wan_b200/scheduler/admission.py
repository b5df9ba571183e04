"""Admission of wide stages (ZeRO-1 or pieces) and the exchange simulator.

Reference behaviour: src/wantrain/scheduler/admission.py (S1 stream test, S2
exposure test, device and host memory terms, one device class per stage:
`check_class` :214, `s1_loads` :311, memory and host terms :420-610) and
src/wantrain/scheduler/exchange_sim.py (`simulate_exchange` :664,
`predict_exchange` :747: need-first sharing of a peer's link between the
gradient reduce-scatter and the parameter all-gather). Restated here for one
process per GPU; a link is whatever carries the stage's exchange: NVLink
through NVSwitch on one box (measured 770 GB/s per direction), a NIC between
machines.

What a wide stage of width w exchanges per step, per peer (per direction):
  reduce-scatter  the fp32 gradient partial of every trainable element,
                  (w - 1) / w of it leaves the peer;
  all-gather      ZeRO-1: the fp32 master; pieces: the fp32 non-matrix
                  region and the bf16 matrix region, (w - 1) / w arrives.

- S1 (stream): spread over the step's microbatches, the exchange plus the
  pipeline boundary fit the link: (share + A) / c <= rate, with c the seconds
  one microbatch takes the peer.
- S2 (exposure): `simulate_exchange` walks the step's end: each unit's
  gradient can leave once its last W is done (units finish in reverse forward
  order), its shard steps AdamW, and its gathered parameters must arrive
  before the next step's first F reaches it; a link serves the transfer whose
  deadline is nearest (need-first). The exposed time (when F must wait) must
  stay within `epsilon` of one microbatch's compute.
- Memory: per peer device bytes (layout-dependent parameter state plus the
  in-flight activations) within the device less its reserve; with host AdamW
  moments, the host's RAM less its reserve.
- Class: every peer of a stage is the same device class (a fold over unequal
  devices would pace the whole stage to the slowest).
Every refusal is a `Reason` naming the stage, peer, link or host and its numbers.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

EPSILON = 0.03


@dataclass(frozen=True)
class Device:
    """One GPU (or CPU slot) as admission sees it; rates in bytes/s per direction."""

    name: str
    host: str = "localhost"
    device_class: str = "b200"
    vram_bytes: float = 178 * 2**30
    tflops: float = 1400.0
    link_Bps: float = 770e9


@dataclass(frozen=True)
class HostMem:
    name: str
    ram_bytes: float


@dataclass(frozen=True)
class Reason:
    kind: str  # class | S1 | S2 | MEM | MEM-HOST
    where: str
    value: float = 0.0
    bound: float = 0.0
    unit: str = ""

    def text(self) -> str:
        if not self.value and not self.bound:
            return f"{self.kind}: {self.where}"
        return f"{self.kind}: {self.where} {self.value:.4g} > {self.bound:.4g} {self.unit}".rstrip()


@dataclass
class StageTerms:
    """What one microbatch and one step cost a stage (from the model)."""

    params: int            # every element the stage holds
    trainable: int
    nonmatrix: int         # trainable elements outside the matrices (norms, biases, tables)
    units: list = field(default_factory=list)  # per forward-order entry: trainable elements
    flops_mb: float = 0.0  # F + B + W of one microbatch
    boundary_mb: float = 0.0  # pipeline boundary bytes of one microbatch per direction
    act_mb: float = 0.0    # activation bytes one in-flight microbatch holds


def vram_reserve(vram: float) -> float:
    return max(0.12 * vram, 2**30)


def host_reserve(ram: float) -> float:
    return max(0.10 * ram, 4 * 2**30)


def stage_terms(spec, stage: int) -> StageTerms:
    from elysium_wan_b200.models.gpt import entry_specs
    from elysium_wan_b200.scheduler.planner import stage_memory_model

    cfg = spec.model
    a, b = spec.partition[stage]
    units, params, trainable, nonmatrix = [], 0, 0, 0
    for e in range(a, b):
        n_unit = 0
        for s in entry_specs(cfg, e):
            n = math.prod(s.shape)
            params += n
            if s.frozen:
                continue
            trainable += n
            n_unit += n
            if not s.matrix or s.replicate:  # held whole by every pieces replica
                nonmatrix += n
        units.append(n_unit)
    T = spec.mb_size * cfg.seq_len
    flops_mb = 6.0 * trainable * T  # F + B + W of the GEMMs
    bdt = {"fp32": 4.0, "bf16": 2.0}.get(cfg.boundary_dtype, 1.0 + 4.0 / 128)
    boundary = T * cfg.d_model * bdt if stage < spec.stages - 1 else 0.0
    mem_f, _, _ = stage_memory_model(spec, stage)
    return StageTerms(params=params, trainable=trainable, nonmatrix=nonmatrix, units=units,
                      flops_mb=flops_mb, boundary_mb=boundary, act_mb=max(0.0, mem_f))


def exchange_bytes(terms: StageTerms, width: int, shard: str) -> tuple[float, float]:
    """(reduce-scatter bytes out, all-gather bytes in) per peer per step."""
    if width <= 1:
        return 0.0, 0.0
    f = (width - 1) / width
    rs = 4.0 * terms.trainable * f
    if shard == "pieces":
        ag = (4.0 * terms.nonmatrix + 2.0 * (terms.trainable - terms.nonmatrix)) * f
    else:
        ag = 4.0 * terms.trainable * f
    return rs, ag


def device_bytes(terms: StageTerms, width: int, shard: str, inflight: int,
                 host_moments: bool = False) -> float:
    """Per-peer device bytes: parameter state of the layout plus activations."""
    P, N, R = terms.params, terms.trainable, terms.nonmatrix
    work = 2.0 * P           # bf16 working copy of everything
    grad = 4.0 * N           # fp32 gradient (fold target)
    if shard == "pieces" and width > 1:
        master = 4.0 * (R + (N - R) / width) + 4.0 * (P - N)
        moments = 0.0 if host_moments else 8.0 * N / width
    else:
        master = 4.0 * P
        moments = 0.0 if host_moments else 8.0 * (N / width if width > 1 else N)
    return work + grad + master + moments + inflight * terms.act_mb


def check_class(stage: int, devs: list) -> list:
    classes = sorted({d.device_class for d in devs})
    if len(classes) > 1:
        return [Reason("class", f"stage {stage} peers {', '.join(d.name for d in devs)}: "
                       + " + ".join(classes))]
    return []


def s1(stage: int, terms: StageTerms, devs: list, shard: str, microbatches: int) -> list:
    """Each peer's link carries its share of the step's exchange, spread over
    the microbatches it computes, plus the boundary, at its compute pace."""
    w = len(devs)
    rs, ag = exchange_bytes(terms, w, shard)
    out = []
    mbs_per_peer = max(1, microbatches // max(1, w))
    for d in devs:
        c = terms.flops_mb / (d.tflops * 1e12)
        for name, xfer in (("out", rs), ("in", ag)):
            load = (xfer / mbs_per_peer + terms.boundary_mb) / c
            if load > d.link_Bps:
                out.append(Reason("S1", f"stage {stage} peer {d.name} link {name}", load,
                                  d.link_Bps, "B/s"))
    return out


def simulate_exchange(units: list, width: int, shard: str, link_Bps: float,
                      c_mb: float, w_share: float = 1.0 / 3.0, f_share: float = 1.0 / 3.0,
                      adam_Bps: float = 6.5e12, nonmatrix_frac: float = 0.0) -> dict:
    """The step boundary of one peer, need-first on its link.

    units: trainable elements per entry in forward order. The last
    microbatch's W visits the units in reverse order, taking w_share * c_mb in
    proportion to size; as a unit's W ends its gradient share (fp32, (w-1)/w)
    may leave. After the last W and the unit's AdamW (bytes at adam_Bps), its
    gathered parameters must arrive; the next step's first F needs unit u
    after the F of units before it (f_share * c_mb in proportion). Transfers
    are served earliest-deadline-first; a reduce-scatter's deadline is its
    unit's gather deadline. -> {"exposed_s", "end_s", "order"}."""
    if width <= 1 or not units:
        return {"exposed_s": 0.0, "end_s": 0.0, "order": []}
    f = (width - 1) / width
    total = float(sum(units)) or 1.0
    # W in reverse order: end time of each unit's last W
    t = 0.0
    w_end = [0.0] * len(units)
    for u in reversed(range(len(units))):
        t += w_share * c_mb * units[u] / total
        w_end[u] = t
    t_last_w = t
    # AdamW of the shard after the step's fold (one pass, all units)
    adam = sum(units) / width * 32.0 / adam_Bps
    # next step's F: unit u needed at
    need = [0.0] * len(units)
    tf = t_last_w + adam
    for u in range(len(units)):
        need[u] = tf
        tf += f_share * c_mb * units[u] / total
    per_elem_ag = 4.0 * nonmatrix_frac + (2.0 if shard == "pieces" else 4.0) * (1 - nonmatrix_frac)
    t_adam = t_last_w + adam
    # (deadline, ready, bytes, kind, unit): gradients first; a unit's gather
    # joins once its gradient has left and the optimizer has run
    pending = [(need[u], w_end[u], 4.0 * units[u] * f, "rs", u) for u in range(len(units))]
    link_t, exposed, order = 0.0, 0.0, []
    while pending:
        ready = [j for j in pending if j[1] <= link_t]
        if not ready:  # the link idles until the next transfer is ready
            link_t = min(j[1] for j in pending)
            continue
        j = min(ready, key=lambda x: (x[0], x[1]))  # nearest deadline first
        pending.remove(j)
        link_t += j[2] / link_Bps
        order.append((j[3], j[4]))
        if j[3] == "rs":
            pending.append((need[j[4]], max(link_t, t_adam), per_elem_ag * units[j[4]] * f, "ag",
                            j[4]))
        else:
            exposed = max(exposed, link_t - need[j[4]])
    return {"exposed_s": max(0.0, exposed), "end_s": link_t, "order": order}


def admit(spec, devices: list, hosts: dict | None = None, inflight: int | None = None,
          epsilon: float = EPSILON) -> tuple[bool, list, dict]:
    """Admission of every stage of `spec` placed on `devices` (slot order:
    devices[rank] for spec.slots()). -> (ok, reasons, predictions)."""
    reasons, pred = [], {}
    hosts = hosts or {}
    host_need: dict = {}
    slots = spec.slots()
    by_stage: dict = {}
    for i, (r, p) in enumerate(slots):
        by_stage.setdefault(r, []).append(devices[i])
    host_moments = spec.optimizer == "adamw-host"
    for r in range(spec.stages):
        devs = by_stage[r]
        w = len(devs)
        terms = stage_terms(spec, r)
        reasons += check_class(r, devs)
        if w > 1:
            reasons += s1(r, terms, devs, spec.shard, spec.microbatches)
            c = terms.flops_mb / (min(d.tflops for d in devs) * 1e12)
            sim = simulate_exchange(terms.units, w, spec.shard, min(d.link_Bps for d in devs), c,
                                    nonmatrix_frac=terms.nonmatrix / max(1, terms.trainable))
            pred[r] = sim
            if sim["exposed_s"] > epsilon * c:
                reasons.append(Reason("S2", f"stage {r} exposed exchange", sim["exposed_s"],
                                      epsilon * c, "s"))
        k = inflight if inflight is not None else max(1, spec.stages - r)
        need = device_bytes(terms, w, spec.shard, k, host_moments)
        for d in devs:
            if not d.vram_bytes:  # a host device: its memory is the host's
                continue
            cap = d.vram_bytes - vram_reserve(d.vram_bytes)
            if need > cap:
                reasons.append(Reason("MEM", f"stage {r} peer {d.name}", need, cap, "B"))
            if host_moments:
                n = terms.trainable / (w if w > 1 else 1)
                host_need[d.host] = host_need.get(d.host, 0.0) + 8.0 * n
    for h, need in host_need.items():
        hm = hosts.get(h)
        if hm is not None and need > hm.ram_bytes - host_reserve(hm.ram_bytes):
            reasons.append(Reason("MEM-HOST", f"host {h}", need,
                                  hm.ram_bytes - host_reserve(hm.ram_bytes), "B"))
    return not reasons, reasons, pred


def devices_from_nodes(infos: list, link_Bps: float | None = None) -> list:
    """Admission devices from registered nodes (NodeInfo): class, memory and
    speed as probed; the link rate measured between them when known, else
    the NVLink figure for GPUs and an unbounded one for host devices."""
    out = []
    for n in infos:
        gpu = str(getattr(n, "device", "cpu")).startswith("cuda")
        mem = n.memory_bytes() if gpu else None
        rate = link_Bps if link_Bps else (770e9 if gpu else float("inf"))
        measured = getattr(n, "tflops_bf16", None)
        tflops = float(measured) if measured else (1400.0 if gpu else 1.0)
        out.append(Device(name=n.name, host=n.host, device_class=n.device_class,
                          vram_bytes=mem or 0.0, tflops=tflops, link_Bps=rate))
    return out
