"""Zero-bubble pipeline schedules (Qi et al., "Zero Bubble Pipeline
Parallelism", ICLR 2024, arXiv:2401.10241).

The backward of a stage is split into B (input gradient, on the critical path)
and W (weight gradient, free to move anywhere after its B). A schedule is, per
stage, an order of (op, microbatch) with op in F / B / W.

Solver (same decision steps as the paper's automatic heuristic, which the
reference ports in src/wantrain/scheduler/zero_bubble.py:179-345, generalised
there and here to per-stage costs and per-hop communication):
  * warm-up: every stage runs F(0); stage j then runs as many extra F as fit
    its memory budget before the first B can come back from downstream
    (optionally allowing a bubble before that first B), never more than its
    upstream neighbour;
  * steady state, per microbatch: F where it does not starve the downstream
    stage's B (when `prioritize_b`), W to cover the wait for the next input
    (all of it, or only where the gap exceeds the worst stage's bubble unless
    `greedy_w`), W under memory pressure, then B from the last stage down;
  * tail: the remaining W.
The grid over the three binary choices keeps the shortest simulated makespan
that fits the memory budget; a warm-up family (k_j forwards then B W F) is the
fallback when no grid candidate fits or when it is shorter.

Memory model (reference convention): F allocates mem_f, B frees -mem_b, W frees
-mem_w, mem_f + mem_b + mem_w = 0. ZB-1p budgets p * mem_f (1F1B's activation
peak), ZB-2p twice that, "given" uses max_mem as is.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

F, B, W = "F", "B", "W"
OPS = (F, B, W)
_EPS = 1e-9


@dataclass
class ZBConfig:
    n_stages: int
    n_micro: int
    cost_f: list
    cost_b: list
    cost_w: list
    comm: list = field(default_factory=list)  # hop j -> j+1, len n_stages - 1
    mem_f: list = field(default_factory=list)
    mem_b: list = field(default_factory=list)
    mem_w: list = field(default_factory=list)
    max_mem: list | None = None

    def __post_init__(self):
        p = self.n_stages
        for name in ("cost_f", "cost_b", "cost_w"):
            if len(getattr(self, name)) != p:
                raise ValueError(f"{name} needs one entry per stage ({p})")
        if isinstance(self.comm, (int, float)):
            self.comm = [float(self.comm)] * max(0, p - 1)
        elif not self.comm:
            self.comm = [0.0] * max(0, p - 1)
        if len(self.comm) != max(0, p - 1):
            raise ValueError(f"comm needs one entry per hop ({p - 1})")
        if not self.mem_f:
            self.mem_f = [1.0] * p
            self.mem_b = [-0.5] * p
            self.mem_w = [-0.5] * p
        for a, b, c in zip(self.mem_f, self.mem_b, self.mem_w):
            if abs(a + b + c) > 1e-6 * max(1.0, abs(a)):
                raise ValueError("mem_f + mem_b + mem_w must be 0")

    def cost(self, op: str, s: int) -> float:
        return {F: self.cost_f, B: self.cost_b, W: self.cost_w}[op][s]

    def mem(self, op: str, s: int) -> float:
        return {F: self.mem_f, B: self.mem_b, W: self.mem_w}[op][s]

    def work(self, s: int) -> float:
        return self.n_micro * (self.cost_f[s] + self.cost_b[s] + self.cost_w[s])

    def with_budget(self, budget: list) -> "ZBConfig":
        return ZBConfig(self.n_stages, self.n_micro, self.cost_f, self.cost_b, self.cost_w,
                        self.comm, self.mem_f, self.mem_b, self.mem_w, max_mem=list(budget))


@dataclass
class Schedule:
    kind: str
    orders: list  # per stage: [(op, mb), ...]
    makespan: float
    bubble_rate: float
    params: dict = field(default_factory=dict)

    def as_spec_order(self) -> list:
        return [[[op, mb] for op, mb in order] for order in self.orders]


def bubble_rate(cfg: ZBConfig, makespan: float) -> float:
    if makespan <= 0:
        return 0.0
    useful = sum(cfg.work(s) for s in range(cfg.n_stages))
    return max(0.0, 1.0 - useful / (cfg.n_stages * makespan))


# --------------------------------------------------------------------------- simulator
def simulate(cfg: ZBConfig, orders):
    """Run per-stage orders under the dependencies (F(s,m) after F(s-1,m) +
    comm; B(s,m) after B(s+1,m) + comm, the last stage's B after its F; W after
    its B). Returns ({(op, stage, mb): end}, makespan). Raises on deadlock."""
    return simulate_slots(cfg, [[o] for o in orders], [[1.0] for _ in range(cfg.n_stages)])


def simulate_slots(cfg: ZBConfig, slot_orders, peer_weights):
    """Several peers per stage: peer q of stage s runs an op in
    cost * sum(weights) / weight[q] (its share of the stage's throughput)."""
    p = cfg.n_stages
    end: dict = {}
    slots = [(s, q) for s in range(p) for q in range(len(slot_orders[s]))]
    pos = dict.fromkeys(slots, 0)
    free = dict.fromkeys(slots, 0.0)
    start0: dict = {}
    left = sum(len(slot_orders[s][q]) for s, q in slots)

    def ready(op, s, mb):
        if op == F:
            if s == 0:
                return 0.0
            k = (F, s - 1, mb)
            return end[k] + cfg.comm[s - 1] if k in end else None
        if op == B:
            if s == p - 1:
                return end.get((F, s, mb))
            k = (B, s + 1, mb)
            return end[k] + cfg.comm[s] if k in end else None
        return end.get((B, s, mb))

    while left:
        moved = False
        for s, q in slots:
            order = slot_orders[s][q]
            scale = sum(peer_weights[s]) / peer_weights[s][q]
            while pos[(s, q)] < len(order):
                op, mb = order[pos[(s, q)]]
                r = ready(op, s, mb)
                if r is None:
                    break
                t0 = max(free[(s, q)], r)
                start0.setdefault((s, q), t0)
                free[(s, q)] = end[(op, s, mb)] = t0 + cfg.cost(op, s) * scale
                pos[(s, q)] += 1
                left -= 1
                moved = True
        if not moved:
            raise ValueError("schedule deadlocks: an op waits on one ordered after it")
    makespan = max(free[k] - start0.get(k, 0.0) for k in slots)
    return end, makespan


def stage_peak(cfg: ZBConfig, s: int, order) -> float:
    m = peak = 0.0
    for op, _ in order:
        m += cfg.mem(op, s)
        peak = max(peak, m)
    return peak


def peak_memory(cfg: ZBConfig, orders) -> list:
    return [stage_peak(cfg, s, o) for s, o in enumerate(orders)]


def _fits(cfg, orders, limit) -> bool:
    return all(pk <= lim + _EPS for pk, lim in zip(peak_memory(cfg, orders), limit))


def default_budget(cfg: ZBConfig) -> list:
    return cfg.max_mem or [cfg.mem_f[s] * cfg.n_micro * 3 for s in range(cfg.n_stages)]


# --------------------------------------------------------------------------- heuristic
class _Builder:
    """Incremental construction of per-stage orders with a running time model."""

    def __init__(self, cfg: ZBConfig, budget: list):
        p = cfg.n_stages
        self.cfg, self.p, self.budget = cfg, p, budget
        self.count = {F: [0] * p, B: [0] * p, W: [0] * p}
        self.clock = [0.0] * p  # when stage j becomes free
        self.memory = [0.0] * p
        self.bubble = [0.0] * p
        self.done: dict = {}  # (op, stage, mb) -> end time
        self.orders: list = [[] for _ in range(p)]

    def n(self, op, j):
        return self.count[op][j]

    def arrival(self, op, j, mb):
        """When the input of (op, j, mb) is available at stage j."""
        c = self.cfg
        if op == F and j > 0:
            return self.done[(F, j - 1, mb)] + c.comm[j - 1]
        if op == B and j < self.p - 1:
            return self.done[(B, j + 1, mb)] + c.comm[j]
        return 0.0

    def emit(self, j, op):
        c = self.cfg
        mb = self.count[op][j]
        cost = c.cost(op, j)
        unblocked = self.clock[j] + cost
        fin = unblocked
        if (op == F and j > 0) or (op == B and j < self.p - 1):
            fin = max(fin, self.arrival(op, j, mb) + cost)
        if self.count[F][j] > 0:
            self.bubble[j] += fin - unblocked
        self.clock[j] = fin
        self.done[(op, j, mb)] = fin
        self.memory[j] += c.mem(op, j)
        self.orders[j].append((op, mb))
        self.count[op][j] += 1

    def pending_w(self, j) -> bool:
        return self.count[W][j] < self.count[B][j]

    def w_until(self, j, t, greedy):
        """Fill the wait for an input arriving at t with W: every W that ends
        before t, then one more if the gap is a real bubble (or greedily)."""
        c = self.cfg
        while self.pending_w(j) and self.clock[j] + c.cost_w[j] <= t:
            self.emit(j, W)
        if self.pending_w(j) and self.clock[j] < t:
            if t - self.clock[j] > max(self.bubble) - self.bubble[j] or greedy:
                self.emit(j, W)

    def make_room(self, j, need):
        while self.memory[j] + need > self.budget[j] + _EPS:
            if not self.pending_w(j):
                raise ValueError("cannot fit memory")
            self.emit(j, W)


def _heuristic(cfg: ZBConfig, budget: list, bubble_before_first_b: bool, prioritize_b: bool,
               greedy_w: bool):
    p, nmb = cfg.n_stages, cfg.n_micro
    st = _Builder(cfg, budget)
    for i in range(nmb):
        if i == 0:
            for j in range(p):
                st.emit(j, F)
            # Warm-up: extra forwards per stage that fit memory and finish
            # before the first B returns from downstream.
            extra = [0] * p
            back = 0.0
            for j in range(p - 1, -1, -1):
                if j == p - 1:
                    back = st.done[(F, j, 0)] + cfg.cost_b[j]
                    continue
                mem, t = st.memory[j], st.clock[j]
                horizon = back + cfg.comm[j]
                while st.n(F, j) + extra[j] < nmb and mem + cfg.mem_f[j] <= budget[j] + _EPS:
                    if bubble_before_first_b:
                        if t + cfg.cost_f[j] > horizon:
                            break
                    elif t >= horizon:
                        break
                    mem += cfg.mem_f[j]
                    t += cfg.cost_f[j]
                    extra[j] += 1
                back = max(t, horizon) + cfg.cost_b[j]
            for j in range(1, p):
                # a stage never warms up deeper than the one feeding it
                while extra[j] > 0 and extra[j] >= extra[j - 1] and st.n(F, j) + extra[j] < nmb:
                    extra[j] -= 1
                extra[j] = min(extra[j], extra[j - 1])
            for j in range(p):
                for _ in range(extra[j]):
                    st.emit(j, F)
            for j in range(p - 1, -1, -1):
                st.emit(j, B)
            continue

        want_f = [0] * p
        for j in range(p):
            if st.n(F, j) >= nmb:
                continue
            if prioritize_b and j + 1 < p and st.n(F, j) >= st.n(F, j + 1) + 2:
                # Downstream already holds two of our forwards: run F only if it
                # does not delay the B that downstream will send back.
                downstream = st.clock[j + 1] + cfg.cost_f[j + 1] + cfg.cost_b[j + 1] + cfg.comm[j]
                if st.clock[j] >= downstream:
                    continue
                w_cost, k, mem = 0.0, 0, st.memory[j] + cfg.mem_f[j]
                while mem > budget[j] + _EPS and st.n(W, j) + k < st.n(B, j):
                    w_cost += cfg.cost_w[j]
                    mem += cfg.mem_w[j]
                    k += 1
                if st.clock[j] + cfg.cost_f[j] + w_cost <= downstream:
                    want_f[j] = 1
                    continue
                if downstream - st.clock[j] <= max(st.bubble) - st.bubble[j]:
                    continue
            want_f[j] = 1
        for j in range(p - 2, -1, -1):
            want_f[j] = min(want_f[j], want_f[j + 1])
        for j in range(p):
            if not want_f[j]:
                continue
            st.make_room(j, cfg.mem_f[j])
            if j > 0:
                st.w_until(j, st.arrival(F, j, st.n(F, j)), greedy_w)
            st.emit(j, F)
        for j in range(p - 1, -1, -1):
            st.make_room(j, cfg.mem_b[j])
            if j + 1 < p:
                st.w_until(j, st.arrival(B, j, st.n(B, j)), greedy_w)
            if j == 0 and st.n(F, j) == nmb:
                while st.pending_w(j):
                    st.emit(j, W)
            st.emit(j, B)
    for j in range(p):
        while st.n(W, j) < nmb:
            st.emit(j, W)
    return st.orders


def warmup_order(n_micro: int, k: int) -> list:
    """k forwards, then per microbatch B, W and the next F."""
    o = [(F, mb) for mb in range(k)]
    for i in range(n_micro):
        o += [(B, i), (W, i)]
        if k + i < n_micro:
            o.append((F, k + i))
    return o


def _warmup_family(cfg: ZBConfig, budget, mem_mode: str) -> Schedule:
    """Best schedule of the form 'k_j forwards, then B W F' with k_j
    non-increasing down the pipeline and within each stage's budget."""
    p, n = cfg.n_stages, cfg.n_micro
    largest, cap = [], n
    for s in range(p):
        lo, hi = 1, cap
        while lo < hi:
            mid = (lo + hi + 1) // 2
            if stage_peak(cfg, s, warmup_order(n, mid)) <= budget[s] + _EPS:
                lo = mid
            else:
                hi = mid - 1
        largest.append(lo)
        cap = lo
    g_max = max(1, math.ceil((largest[0] - 1) / max(1, p - 1)))
    gaps = sorted({g for e in range(g_max.bit_length() + 1) for g in (2 ** e, 3 * 2 ** e // 2)}
                  | {g_max})
    best = None
    for g in (x for x in gaps if 1 <= x <= g_max):
        warm = [min(largest[j], 1 + g * (p - 1 - j)) for j in range(p)]
        orders = [warmup_order(n, k) for k in warm]
        _, ms = simulate(cfg, orders)
        if best is None or ms < best[1] - 1e-12:
            best = (orders, ms, warm)
    orders, ms, warm = best
    if not _fits(cfg, orders, budget):
        raise ValueError(f"no warm-up schedule fits the memory budget (warm-ups {warm})")
    return Schedule("zb", orders, ms, bubble_rate(cfg, ms),
                    dict(degraded=True, warmups=warm, mem_mode=mem_mode))


def _check_one_microbatch(cfg, budget):
    for s in range(cfg.n_stages):
        need = max(0.0, cfg.mem_f[s], cfg.mem_f[s] + cfg.mem_b[s])
        if need > budget[s] + _EPS:
            raise ValueError(f"stage {s} cannot fit one microbatch: needs {need:.0f}, "
                             f"budget {budget[s]:.0f}")


def zero_bubble(cfg: ZBConfig, mem_mode: str = "1p") -> Schedule:
    """Automatic zero-bubble schedule: grid search over the heuristic's three
    choices plus the warm-up family; shortest simulated makespan that fits."""
    if mem_mode in ("1p", "2p"):
        # 1F1B's activation peak is p microbatches; with recompute B (not F)
        # allocates the larger share, so the unit is the larger of the two.
        k = 1 if mem_mode == "1p" else 2
        unit = max(max(cfg.mem_f), max(f + b for f, b in zip(cfg.mem_f, cfg.mem_b)))
        cfg = cfg.with_budget([k * cfg.n_stages * unit] * cfg.n_stages)
    budget = default_budget(cfg)
    _check_one_microbatch(cfg, budget)
    if cfg.n_stages == 1:
        o = [[(F, m) for m in range(cfg.n_micro)] + [(B, m) for m in range(cfg.n_micro)]
             + [(W, m) for m in range(cfg.n_micro)]]
        if not _fits(cfg, o, budget):
            return _warmup_family(cfg, budget, mem_mode)
        _, ms = simulate(cfg, o)
        return Schedule("zb", o, ms, bubble_rate(cfg, ms), dict(mem_mode=mem_mode, degraded=False))
    best = None
    for a in (True, False):
        for pb in (True, False):
            for gw in (True, False):
                try:
                    orders = _heuristic(cfg, budget, a, pb, gw)
                except ValueError:
                    continue
                if not _fits(cfg, orders, budget):
                    continue
                _, ms = simulate(cfg, orders)
                if best is None or ms < best[1] - 1e-12:
                    best = (orders, ms, dict(allow_bubble_before_first_b=a, prioritize_b=pb,
                                             no_bubble_greedy=gw))
    fallback = _warmup_family(cfg, budget, mem_mode)
    if best is None or fallback.makespan < best[1] - 1e-12:
        return fallback
    orders, ms, choice = best
    return Schedule("zb", orders, ms, bubble_rate(cfg, ms), dict(choice, mem_mode=mem_mode,
                                                                  degraded=False))


def one_f_one_b(cfg: ZBConfig) -> Schedule:
    """1F1B (W right after its B) for comparison: stage j warms up p - j forwards."""
    p, n = cfg.n_stages, cfg.n_micro
    orders = [warmup_order(n, min(n, p - j)) for j in range(p)]
    _, ms = simulate(cfg, orders)
    return Schedule("1f1b", orders, ms, bubble_rate(cfg, ms), {})


def iwrr(n: int, weights) -> list:
    """Interleaved weighted round robin: owner of each of n microbatches, peer
    of weight w receiving w / sum(weights) of them, interleaved; equal weights
    give plain round robin (mb % width). Ties go to the lower index."""
    w = [float(x) for x in weights]
    if any(x <= 0 for x in w):
        raise ValueError(f"peer weights must be positive, got {weights}")
    count = [0] * len(w)
    out = []
    for _ in range(n):
        q = min(range(len(w)), key=lambda i: ((count[i] + 1) / w[i], i))
        count[q] += 1
        out.append(q)
    return out


def comm_seconds(boundary_bytes: float, mbps: float, rtt_ms: float) -> float:
    """One boundary transfer across a hop: one-way latency + bytes at rate."""
    rate = boundary_bytes * 8 / (mbps * 1e6) if mbps and math.isfinite(mbps) and mbps > 0 else 0.0
    return max(0.0, rtt_ms) / 2000.0 + rate


def slot_orders(stage_order: list, owners: list, width: int) -> list:
    """Split a stage's aggregate order into one order per peer by microbatch
    ownership (owners[mb] = peer), keeping the relative order."""
    out = [[] for _ in range(width)]
    for op, mb in stage_order:
        out[owners[mb]].append((op, mb))
    return out


def in_flight_peak(order) -> int:
    """Most microbatches one slot's order holds between an F and its B."""
    live = peak = 0
    for op, _mb in order:
        if op == F:
            live += 1
            peak = max(peak, live)
        elif op == B:
            live -= 1
    return peak


def selective_recompute(spec, force=frozenset(), budget_bytes: list | None = None) -> list | None:
    """Per stage, whether it recomputes under a recomputing spec (None when
    nothing changes).

    Without `budget_bytes` (the reference's rule, selective_recompute in
    src/wantrain/scheduler/zero_bubble.py:607, RUNTIME-I25): a stage
    recomputes only where some slot's order holds more than one microbatch
    between an F and its B, or it is in `force`.

    This engine recomputes layer by layer (B re-runs one layer's forward just
    before that layer's backward), so even one microbatch in flight needs less
    memory recomputed. With `budget_bytes` (activation bytes each stage may
    hold) the rule is memory's: a stage keeps F's saved tensors when its
    in-flight peak of them fits its budget, else it recomputes. The math is the
    same either way, so the bits are too."""
    if not spec.recompute or spec.schedule_order is None:
        return None
    out = []
    for r, slots in enumerate(spec.schedule_order):
        peak = max((in_flight_peak([(op, mb) for op, mb in order]) for order in slots),
                   default=0)
        if budget_bytes is None:
            need = peak > 1
        else:
            from elysium_wan_b200.scheduler.planner import act_bytes

            a, b = spec.partition[r]
            blocks = sum(1 for e in range(a, b) if 1 <= e <= spec.model.n_layer)
            m = act_bytes(spec.model, spec.mb_size, spec.device_for(r))
            need = peak * blocks * (m["saved"] + m["boundary"]) > budget_bytes[r]
        out.append(need or r in force)
    return None if all(out) else out
