"""Chain routing: which machine holds which pipeline rank.

Reference behaviour: src/wantrain/scheduler/partition.py (`order_stages` :36,
`best_chain` :99) and the coordinator's probe-and-route loop
(src/wantrain/coordinator/coordinator.py `_probe_matrix` :813, `_route_chain`
:859). Rank r talks to rank r+1 only, so the chain should be the Hamiltonian
path through the measured link matrix whose slowest hop is fastest; among
those, the one with the least total round trip.

How it is solved here (not a branch-and-bound over orderings):
1. the best bottleneck is the largest link rate t for which the graph of
   links with rate >= t still has a Hamiltonian path. Path existence is a
   subset DP (`_reachable_ends`: for every subset, the set of nodes a path
   through exactly that subset can end on, as a bitmask), and it is monotone
   in t, so t is found by binary search over the distinct rates;
2. on that graph a Held-Karp DP over (subset, end node) finds the path of
   least total round trip.
Both are exact up to EXACT_MAX nodes (2^n * n^2 steps). Beyond that, a best
next hop from every start node is refined by segment reversals (2-opt) that
raise the (bottleneck, -total RTT) key.

A chain and its reverse carry the same hops; the returned order is the
direction whose first node has the lower index.
"""

from __future__ import annotations

import math

EXACT_MAX = 12


def chain_key(order: list, bw: list, rtt: list | None = None) -> tuple:
    """(bottleneck rate, -total round trip) of a chain: larger is better."""
    hops = list(zip(order, order[1:]))
    if not hops:
        return (math.inf, 0.0)
    return (min(bw[a][b] for a, b in hops),
            -sum(rtt[a][b] for a, b in hops) if rtt is not None else 0.0)


def symmetrize(rtt: list, bw: list) -> tuple[list, list]:
    """A hop carries both directions: its rate is the slower direction's, its
    round trip the longer one. None (unreachable) becomes 0 rate, inf RTT."""
    n = len(bw)
    r2 = [[0.0] * n for _ in range(n)]
    b2 = [[math.inf] * n for _ in range(n)]
    for i in range(n):
        for j in range(n):
            if i == j:
                continue
            bij, bji = bw[i][j], bw[j][i]
            rij, rji = rtt[i][j], rtt[j][i]
            b2[i][j] = min(0.0 if bij is None else float(bij), 0.0 if bji is None else float(bji))
            r2[i][j] = max(math.inf if rij is None else float(rij),
                           math.inf if rji is None else float(rji))
    return r2, b2


def _reachable_ends(n: int, adj: list) -> list:
    """ends[mask] = bitmask of nodes on which a path visiting exactly `mask`
    can end. adj[v] = bitmask of v's neighbours."""
    ends = [0] * (1 << n)
    for v in range(n):
        ends[1 << v] = 1 << v
    for mask in range(1, 1 << n):
        e = ends[mask]
        if not e:
            continue
        free = ~mask & ((1 << n) - 1)
        v = 0
        while e:
            if e & 1:
                nxt = adj[v] & free
                while nxt:
                    low = nxt & -nxt
                    ends[mask | low] |= low
                    nxt ^= low
            e >>= 1
            v += 1
    return ends


def _has_path(n: int, bw: list, t: float) -> bool:
    adj = [sum(1 << j for j in range(n) if j != i and bw[i][j] >= t) for i in range(n)]
    return _reachable_ends(n, adj)[(1 << n) - 1] != 0


def _min_rtt_path(n: int, bw: list, rtt: list | None, t: float) -> list:
    """Held-Karp over links with rate >= t: the path of least total RTT
    (ties: the first found in index order)."""
    full = (1 << n) - 1
    INF = math.inf
    cost = [[INF] * n for _ in range(1 << n)]
    par = [[-1] * n for _ in range(1 << n)]
    for v in range(n):
        cost[1 << v][v] = 0.0
    for mask in range(1, 1 << n):
        row = cost[mask]
        for v in range(n):
            c = row[v]
            if c == INF and not (mask == 1 << v):
                continue
            for w in range(n):
                if mask >> w & 1 or bw[v][w] < t:
                    continue
                c2 = c + (rtt[v][w] if rtt is not None else 0.0)
                m2 = mask | 1 << w
                if c2 < cost[m2][w]:
                    cost[m2][w] = c2
                    par[m2][w] = v
    # the Held-Karp table stores inf for paths through unreachable RTT; fall
    # back to any path of the right bottleneck
    end = min(range(n), key=lambda v: (cost[full][v], v))
    if cost[full][end] == INF:
        return _any_path(n, bw, t)
    order, mask, v = [], full, end
    while v != -1:
        order.append(v)
        pv = par[mask][v]
        mask ^= 1 << v
        v = pv
    return order[::-1]


def _any_path(n: int, bw: list, t: float) -> list:
    adj = [sum(1 << j for j in range(n) if j != i and bw[i][j] >= t) for i in range(n)]
    ends = _reachable_ends(n, adj)
    full = (1 << n) - 1
    v = next(v for v in range(n) if ends[full] >> v & 1)
    order, mask = [v], full
    while mask != 1 << v:
        mask ^= 1 << v
        v = next(u for u in range(n) if ends[mask] >> u & 1 and adj[u] >> v & 1)
        order.append(v)
    return order[::-1]


def _greedy(n: int, bw: list, rtt: list | None) -> list:
    best = None
    for s in range(n):
        order, used = [s], {s}
        while len(order) < n:
            a = order[-1]
            b = max((k for k in range(n) if k not in used),
                    key=lambda k: (bw[a][k], -(rtt[a][k] if rtt is not None else 0.0), -k))
            order.append(b)
            used.add(b)
        if best is None or chain_key(order, bw, rtt) > chain_key(best, bw, rtt):
            best = order
    improved = True
    while improved:  # 2-opt: reverse a segment while the key rises
        improved = False
        for i in range(n - 1):
            for j in range(i + 2, n + 1):
                cand = best[:i] + best[i:j][::-1] + best[j:]
                if chain_key(cand, bw, rtt) > chain_key(best, bw, rtt):
                    best, improved = cand, True
    return best


def order_chain(rtt: list | None, bw: list) -> list:
    """Node order for the chain: max bottleneck rate, then min total RTT.
    bw[i][j] / rtt[i][j] are symmetric numbers (see `symmetrize`)."""
    n = len(bw)
    if n <= 2:
        return list(range(n))
    if n > EXACT_MAX:
        order = _greedy(n, bw, rtt)
    else:
        rates = sorted({bw[i][j] for i in range(n) for j in range(n) if i != j})
        lo, hi = 0, len(rates) - 1  # rates[lo] always admits a path (complete graph)
        while lo < hi:
            mid = (lo + hi + 1) // 2
            if _has_path(n, bw, rates[mid]):
                lo = mid
            else:
                hi = mid - 1
        order = _min_rtt_path(n, bw, rtt, rates[lo])
    return order if order[0] < order[-1] else order[::-1]


def best_chain(n: int, edges) -> tuple[list, float]:
    """Max-bottleneck chain from undirected edges [(i, j, mbps), ...]; pairs
    not listed weigh 0. -> (order, bottleneck); 0 means no order connects
    every node over probed links."""
    w = [[0.0] * n for _ in range(n)]
    for i, j, mbps in edges:
        w[i][j] = w[j][i] = float(mbps)
    order = order_chain(None, w)
    return order, (chain_key(order, w)[0] if n > 1 else math.inf)


def route_gain(cur: list, new: list, bw: list, rtt: list | None, margin: float = 0.2) -> bool:
    """Whether `new` is clearly better than `cur`: a bottleneck higher by more
    than `margin`, or (bottleneck within the margin) a total RTT lower by more
    than `margin` and 1 ms. Measurement noise on equal links moves nothing."""
    (b0, r0), (b1, r1) = chain_key(cur, bw, rtt), chain_key(new, bw, rtt)
    if b1 > b0 * (1.0 + margin):
        return True
    if b1 >= b0 * (1.0 - margin) and math.isfinite(r0) and -r1 < -r0 * (1.0 - margin) \
            and (-r0) - (-r1) > 1.0:
        return True
    return False
