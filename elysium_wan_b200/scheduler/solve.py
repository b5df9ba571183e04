"""Schedule solvers: how many microbatches per step, how many in flight, and
how large a fleet one synchronous run keeps busy.

Parity: src/wantrain/scheduler/schedule.py (`fbw_costs` :15,
`solve_microbatches` :28, `solve_fleet_ceiling` :105, `stage_live_graphs`
:178, `solve_k_inflight` :195). The decisions are the same; the bubble is the
one this package's zero-bubble solver leaves, so the solver and the runtime
agree on what "bubble" means. None of these choices changes the trained
model (microbatching is a recipe pin only through `microbatches`, which the
caller adopts or not).
"""

from __future__ import annotations

import math

from elysium_wan_b200.scheduler.zero_bubble import ZBConfig, zero_bubble


def fbw_costs(d_model: int, seq_len: int) -> tuple:
    """Relative (F, B, W) cost of one layer per token.

    Transformer FLOP counts from Qi et al. 2023 ("Zero Bubble Pipeline
    Parallelism", Table 1): F = sbh(24h + 4s), B = sbh(24h + 8s), W = sbh(24h).
    The common factor sbh cancels in every ratio the solvers use."""
    h, s = float(d_model), float(seq_len)
    return (24 * h + 4 * s, 24 * h + 8 * s, 24 * h)


def _bubble(n_stages: int, m: int, f: float, b: float, w: float, comm: float) -> float:
    cfg = ZBConfig(n_stages, m, [f] * n_stages, [b] * n_stages, [w] * n_stages,
                   comm=[comm] * (n_stages - 1))
    # The solver runs against a ZB-2p budget: two pipeline depths of graphs.
    unit = max(max(cfg.mem_f), max(x + y for x, y in zip(cfg.mem_f, cfg.mem_b)))
    cfg = cfg.with_budget([2 * n_stages * unit] * n_stages)
    return zero_bubble(cfg, "given").bubble_rate


def solve_microbatches(n_stages: int, bubble_target: float = 0.05,
                       tokens_per_step_cap: int | None = None, mb_size: int = 1,
                       seq_len: int = 1024, floor: int | None = None, fbw: tuple | None = None,
                       comm_ratio: float = 0.0, cap: int = 1024) -> dict:
    """The smallest microbatch count M whose zero-bubble schedule idles at most
    `bubble_target` of the pipeline; the step's token budget caps M first.

    The bubble falls monotonically with M (fill and drain amortise), so the
    search doubles M until the target holds, then bisects down to the least M.
    Returns {microbatches, bubble, family, reason}."""
    lo = max(1, floor or 1)
    if n_stages < 2:
        return dict(microbatches=lo, bubble=0.0, family="none",
                    reason="one stage: there is no pipeline to fill")
    f, b, w = fbw or (1.0, 1.0, 1.0)
    b, w, f = b / f, w / f, 1.0
    top = cap
    if tokens_per_step_cap:
        top = max(1, min(cap, tokens_per_step_cap // max(1, mb_size * seq_len)))
    lo = min(lo, top)
    memo = {}

    def bub(m):
        if m not in memo:
            memo[m] = _bubble(n_stages, m, f, b, w, comm_ratio)
        return memo[m]

    hi = lo
    while bub(hi) > bubble_target and hi < top:
        hi = min(top, hi * 2)
    if bub(hi) <= bubble_target and hi > lo:
        left, right = max(lo, hi // 2), hi
        while left < right:
            mid = (left + right) // 2
            if bub(mid) <= bubble_target:
                right = mid
            else:
                left = mid + 1
        hi = left
    m, br = hi, bub(hi)
    reason = (f"{m} microbatches leave a {br:.1%} bubble across {n_stages} stages in the "
              f"zero-bubble schedule (target {bubble_target:.0%}; F:B:W = 1:{b:.2f}:{w:.2f}; "
              f"hop transfer {comm_ratio:.2f} x F)")
    if br > bubble_target and m == top and tokens_per_step_cap:
        reason = (f"{m} microbatches is all the {tokens_per_step_cap:,}-token step budget holds at "
                  f"mb_size={mb_size}, seq_len={seq_len}; the bubble stays at {br:.1%} (target "
                  f"{bubble_target:.0%}): a batch past the critical size costs convergence, a "
                  f"bubble only costs speed")
    return dict(microbatches=m, bubble=br, family="zb", reason=reason)


def solve_fleet_ceiling(batch_tokens: float, mb_tokens: int, util_target: float = 0.5,
                        fbw: tuple | None = None, w_fill_depth: int | None = None,
                        n_stages: int | None = None, intra_split: int = 1,
                        n_params: float | None = None, rtt_s: float | None = None,
                        flops_per_gpu: float | None = None) -> dict:
    """The most GPUs one synchronous run keeps `util_target` busy.

    Batch side: each chain pays fill and drain once per step, so a chain is
    busy M/(M + span) of the time; the batch (capped by the critical batch
    size, McCandlish et al. 2018) bounds the total M. Deferred W work banked
    during the fill shortens the effective span by 2*t_W/(t_F+t_B+t_W) of a
    microbatch slot (all of it when W fills the whole drain). Latency side
    (when n_params, rtt_s and flops_per_gpu are given): one update's
    6*N*B FLOPs cannot finish faster than the S*RTT chain."""
    f, b, w = fbw or fbw_costs(4096, 2048)
    slot = f + b + w
    stages = n_stages or 2
    share = 1.0
    if w_fill_depth is not None and stages > 1 and w_fill_depth < stages - 1:
        share = w_fill_depth / (stages - 1)
    span = (slot - 2.0 * w * share) / slot
    dividend = 1.0 / max(1e-9, span)
    u = util_target
    batch_side = max(1, intra_split) * dividend * (batch_tokens / max(1, mb_tokens)) * (1 - u) / u
    lat_side = None
    if n_params and rtt_s and flops_per_gpu:
        lat_side = 6.0 * n_params * batch_tokens / (flops_per_gpu * max(1, stages) * rtt_s * u)
    fleet = batch_side if lat_side is None else min(batch_side, lat_side)
    binding = "batch" if lat_side is None or batch_side <= lat_side else "latency"
    reason = (f"{int(fleet):,} GPUs is the most a {batch_tokens / 1e6:.1f}M-token batch keeps "
              f"{u:.0%} busy at {mb_tokens} tokens per microbatch"
              + (f" split over {intra_split} devices" if intra_split > 1 else "")
              + f"; banked W fills the drain for a {dividend:.2f}x dividend")
    if lat_side is not None:
        reason += f"; the S*RTT chain allows {int(lat_side):,} GPUs and the {binding} side binds"
    return dict(fleet_max=int(fleet), fleet_batch_side=int(batch_side),
                fleet_latency_side=None if lat_side is None else int(lat_side), binding=binding,
                zb_dividend=round(dividend, 2), reason=reason)


def stage_live_graphs(n_stages: int, rank: int, k_inflight: int) -> int:
    """Live activation graphs rank `rank` holds at peak: a microbatch lives
    from its F to its B, i.e. (n_stages - rank) schedule intervals (Qi et al.
    2024, controllable memory), plus one per extra in-flight microbatch."""
    return max(1, n_stages - rank) + max(0, (k_inflight or 1) - 1)


def solve_k_inflight(window_s: float, rtt_ms: float, boundary_bytes: float, link_mbps: float,
                     mem_slack_bytes: float | None = None, per_inflight_bytes: float | None = None,
                     cap: int = 16) -> dict:
    """In-flight microbatches that hide a hop's latency: while microbatch i's
    boundary travels (half the RTT plus its serialisation time), the stage
    computes i+1..i+k, so k = ceil(travel / window) + 1, capped by `cap` and
    by the memory left for the extra boundary buffers and graphs."""
    one_way = max(0.0, rtt_ms) / 2000.0
    xfer = boundary_bytes * 8.0 / (max(1e-9, link_mbps) * 1e6)
    need = one_way + xfer
    if window_s <= 0:
        return dict(k=1, reason="no compute-window estimate: k stays 1")
    k = max(1, math.ceil(need / window_s) + 1)
    reason = (f"k={k} covers {need * 1e3:.1f} ms ({one_way * 1e3:.1f} ms one way + "
              f"{xfer * 1e3:.1f} ms on the wire) with a {window_s * 1e3:.1f} ms compute window")
    if k > cap:
        k = cap
        reason = (f"k capped at {cap}: {need * 1e3:.1f} ms of travel against a "
                  f"{window_s * 1e3:.1f} ms window leaves the stage latency-bound")
    if mem_slack_bytes is not None and per_inflight_bytes:
        fits = max(1, int(mem_slack_bytes // per_inflight_bytes))
        if fits < k:
            reason = (f"k={fits}: memory holds no more ({per_inflight_bytes / 2**20:.0f} MiB per "
                      f"in-flight microbatch, {mem_slack_bytes / 2**30:.1f} GiB spare); latency "
                      f"wanted k={k}")
            k = fits
    return dict(k=k, reason=reason, latency_s=need, window_s=window_s)
