"""Contiguous partition of the flat layer list [Embed, Block x n, Head] over
pipeline stages.

Per-entry cost model (FLOPs per token up to a constant, the reference's
model in src/wantrain/scheduler/partition.py:164-198): a block costs
h * (72 h + 12 s) (its GEMMs plus causal attention), the head 6 h V, the
embedding 3 h. `assign_layers` is an exact min-max dynamic program over
contiguous ranges with per-stage speeds and an optional memory predicate.
"""

from __future__ import annotations


def layer_costs(cfg) -> list:
    h, s, V, n = cfg.d_model, cfg.seq_len, cfg.vocab_size, cfg.n_layer
    f_ratio = cfg.ff / (4 * h)
    block = h * (24 * h + 48 * h * f_ratio + 12 * s)
    return [3.0 * h] + [float(block)] * n + [6.0 * h * V]


def assign_layers(costs: list, speeds: list, fits=None) -> list:
    """[(start, end)] per stage minimising max(cost of range / stage speed).
    fits(stage, start, end) -> bool can veto ranges (memory)."""
    n, S = len(costs), len(speeds)
    if S > n:
        raise ValueError(f"{S} stages for {n} layers")
    pre = [0.0]
    for c in costs:
        pre.append(pre[-1] + c)
    INF = float("inf")
    # best[k][i]: min over partitions of the first i entries into k stages
    best = [[INF] * (n + 1) for _ in range(S + 1)]
    arg = [[-1] * (n + 1) for _ in range(S + 1)]
    best[0][0] = 0.0
    for k in range(1, S + 1):
        for i in range(k, n - (S - k) + 1):
            for j in range(k - 1, i):
                if best[k - 1][j] == INF:
                    continue
                if fits is not None and not fits(k - 1, j, i):
                    continue
                v = max(best[k - 1][j], (pre[i] - pre[j]) / speeds[k - 1])
                if v < best[k][i] - 1e-12:
                    best[k][i] = v
                    arg[k][i] = j
    if best[S][n] == INF:
        raise ValueError("no partition satisfies the memory predicate")
    out, i = [], n
    for k in range(S, 0, -1):
        j = arg[k][i]
        out.append((j, i))
        i = j
    return out[::-1]


def proportional_partition(cfg, speeds: list) -> list:
    return [list(r) for r in assign_layers(layer_costs(cfg), speeds)]


def even_blocks_partition(cfg, stages: int) -> list:
    """n_layer / stages blocks per stage, the embedding on the first and the
    head on the last (the BASELINE cuts: e.g. 8 stages of 6 layers)."""
    n = cfg.n_layer
    if n % stages:
        raise ValueError(f"{n} layers do not split evenly over {stages} stages")
    per = n // stages
    out = []
    for r in range(stages):
        lo = 0 if r == 0 else 1 + r * per
        hi = n + 2 if r == stages - 1 else 1 + (r + 1) * per
        out.append([lo, hi])
    return out


def stage_costs(cfg, partition) -> list:
    c = layer_costs(cfg)
    return [sum(c[a:b]) for a, b in partition]
