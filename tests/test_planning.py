"""Planning helpers: microbatch / in-flight solvers, shape advisor, precision
admission, placement, node selection with link memory, production flags.
Mirrors the reference's scheduler unit tests (tests/unit/test_schedule.py,
test_autoconfig.py, test_placement.py, test_selection.py in
virgiliolrf/elysium-wan): pure host logic, no device."""

import pytest

from elysium_wan_b200.models.config import make_config
from elysium_wan_b200.resources.node import NodeInfo
from elysium_wan_b200.runtime.spec import JobSpec
from elysium_wan_b200.scheduler import autoconfig, production, shape, solve
from elysium_wan_b200.scheduler.linkmemory import LinkMemory, verdict
from elysium_wan_b200.scheduler.placement import memory_order, place, rank_memory_need
from elysium_wan_b200.scheduler.selection import SelectionPolicy, select_nodes


def test_fbw_ratios():
    f, b, w = solve.fbw_costs(4096, 2048)
    assert w < f < b
    assert abs((b + w) - 2 * f) < 1e-9 * f  # B + W = 2F


def test_solve_microbatches_meets_target_and_is_minimal():
    r = solve.solve_microbatches(4, bubble_target=0.10, fbw=(1.0, 1.0, 1.0))
    m = r["microbatches"]
    assert r["bubble"] <= 0.10
    assert solve._bubble(4, m - 1, 1.0, 1.0, 1.0, 0.0) > 0.10 if m > 1 else True
    assert "bubble" in r["reason"]


def test_solve_microbatches_token_cap_binds():
    r = solve.solve_microbatches(8, bubble_target=0.001, tokens_per_step_cap=8 * 2048,
                                 mb_size=1, seq_len=2048)
    assert r["microbatches"] == 8
    assert "step budget" in r["reason"]


def test_single_stage_needs_no_fill():
    assert solve.solve_microbatches(1)["bubble"] == 0.0


def test_k_inflight():
    r = solve.solve_k_inflight(window_s=0.1, rtt_ms=100, boundary_bytes=10e6, link_mbps=1000)
    # 50 ms one way + 80 ms on the wire over a 100 ms window -> k = 3
    assert r["k"] == 3
    r2 = solve.solve_k_inflight(0.1, 100, 10e6, 1000, mem_slack_bytes=1e9, per_inflight_bytes=6e8)
    assert r2["k"] == 1 and "memory" in r2["reason"]


def test_live_graphs_deepest_at_rank0():
    assert [solve.stage_live_graphs(4, r, 1) for r in range(4)] == [4, 3, 2, 1]


def test_fleet_ceiling_latency_binds():
    r = solve.solve_fleet_ceiling(4e6, 2048, n_params=1e11, rtt_s=0.2, flops_per_gpu=1e15,
                                  n_stages=8)
    assert r["fleet_max"] == min(r["fleet_batch_side"], r["fleet_latency_side"])


def test_shape_advisor_prefers_largest_within_target():
    out = shape.advise(8, 160e9, tflops=1000, link_mbps=6e6)
    best = out["best"]
    assert out["met_target"]
    assert all(s.params <= best.params for s in out["fits"] if s.bubble <= 0.2)
    assert best.stage_bytes <= 160e9
    # A slow hop forces a smaller bubble-feasible shape or none at all.
    slow = shape.advise(8, 160e9, tflops=1000, link_mbps=50)
    assert slow["best"].bubble >= best.bubble


def test_precision_admission_policies():
    cfg = make_config("gpt15b")
    p = 6 * 12 * cfg.d_model ** 2
    fast = autoconfig.plan(cfg, p, 6, link_mbps=6e6, window_s=0.2, mem_budget_bytes=180e9)
    assert fast["chosen"]["boundary"] == "fp32"  # widest lossless rung on NVLink
    slow = autoconfig.plan(cfg, p, 6, link_mbps=1200, window_s=0.2, mem_budget_bytes=180e9)
    # 2048 x 5120 bf16 = 21 MB per microbatch -> 839 Mbps floor, 1678 with margin:
    # balanced takes the lossless bf16 rung at the floor and says so.
    assert slow["chosen"]["boundary"] == "bf16" and "WITHOUT" in slow["reason"]
    ll = autoconfig.plan(cfg, p, 6, link_mbps=1200, window_s=0.2, mem_budget_bytes=180e9,
                         policy="lossless")
    assert ll["chosen"] is None and "no lossless" in ll["reason"]
    bal = autoconfig.plan(cfg, p, 6, link_mbps=700, window_s=0.2, mem_budget_bytes=180e9)
    assert bal["chosen"]["boundary"] == "fp8_e4m3_b128" and "NO LOSSLESS" in bal["reason"]
    thr = autoconfig.plan(cfg, p, 6, link_mbps=1200, window_s=0.2, mem_budget_bytes=180e9,
                          policy="max_throughput")
    assert thr["chosen"]["boundary"] == "fp8_e4m3_b128"
    pinned = autoconfig.plan(cfg, p, 6, link_mbps=100, window_s=0.2, mem_budget_bytes=1e9,
                             boundary_override="bf16")
    assert "WARNING" in pinned["reason"] and "chosen" in pinned["report"]


def _nodes(n, vram=(180,), tf=1000.0, cls="cuda:B200", region="r0"):
    out = []
    for i in range(n):
        out.append(NodeInfo(node_id=f"n{i}", name=f"w{i}", host=f"10.0.0.{i + 1}", region=region,
                            device=f"cuda:{i}", device_class=cls,
                            vram_gb=vram[i % len(vram)], tflops_bf16=tf))
    return out


def test_memory_order_gives_rank0_the_biggest_card():
    spec = JobSpec(model=make_config("gpt0_6b"), stages=4, microbatches=8, mb_size=1)
    w = rank_memory_need(spec)
    assert w[0] == max(w[:-1])
    nodes = _nodes(4, vram=(80, 180, 96, 141))
    order = memory_order(spec, nodes)
    assert sorted(order) == [0, 1, 2, 3]
    big = max(range(4), key=lambda r: w[r])
    assert nodes[order[big]].vram_gb == 180


def test_place_cuts_by_speed():
    spec = JobSpec(model=make_config("cpu_plumbing"), stages=2, microbatches=4, mb_size=1,
                   device="cpu")
    nodes = _nodes(2, cls="cpu")
    for n in nodes:
        n.device = "cpu"
    nodes[0].tflops_bf16 = 3.0
    nodes[1].tflops_bf16 = 1.0
    why = place(spec, [[nodes[0]], [nodes[1]]])
    lay = why["layers_per_stage"]
    assert lay[0] >= lay[1]
    assert spec.schedule_order is not None


def test_selection_refuses_mixed_and_skips_dead(tmp_path):
    pool = _nodes(2, cls="cuda:B200") + _nodes(1, cls="cuda:H100")
    pool[2].node_id, pool[2].name = "n9", "w9"
    sel = select_nodes(pool, 3)
    assert not sel.ok and "MIXED-FLEET" in sel.reason
    mem = LinkMemory(str(tmp_path))
    pool = _nodes(4)
    mem.record_dead("w0@10.0.0.1", "heartbeat lost", "run1", host="10.0.0.1")
    sel = select_nodes(pool, 3, memory=mem)
    assert sel.ok and "n0" not in [n.node_id for n in sel.chosen]
    # the memory persists
    assert "w0@10.0.0.1" in LinkMemory(str(tmp_path)).dead_keys()


def test_link_memory_verdicts(tmp_path):
    mem = LinkMemory(str(tmp_path))
    mem.record_path("a", "b", 500, 20, "r1")
    assert verdict(mem.path("b", "a")) == "good"
    mem.record_path("a", "b", 30, 20, "r2")
    assert verdict(mem.path("a", "b")) == "variable"
    mem.record_path("a", "b", 30, 20, "r2")  # replay of the same run
    assert mem.path("a", "b").samples == 2
    mem.record_path("c", "d", 500, 200, "r1")
    assert verdict(mem.path("c", "d")) == "slow"


def test_selection_ranks_by_remembered_paths(tmp_path):
    mem = LinkMemory(str(tmp_path))
    pool = _nodes(3)
    pool[0].tflops_bf16 = 2000.0  # fastest, but its path to everyone is slow
    for o in ("10.0.0.2", "10.0.0.3"):
        mem.record_path("10.0.0.1", o, 10, 300, "r")
    sel = select_nodes(pool, 2, SelectionPolicy(), memory=mem)
    assert sel.ok and "n0" not in [n.node_id for n in sel.chosen]


def test_production_fields():
    f = production.spec_fields([1, 2], {"recompute": False, "lr": None})
    assert f["recompute"] is False and f["grad_sync"] == "fused" and "lr" not in f
    assert production.deviations(f) == ["recompute=False (production: True)"]
    assert production.spec_fields(wan=True)["wire_codec"] == "planes"


@pytest.mark.parametrize("policy", ["lossless", "balanced", "max_throughput"])
def test_choose_returns_reason(policy):
    cfg = make_config("gpt0_6b")
    rows = autoconfig.evaluate(cfg, 10**8, 4, 1, 2, 1e5, 0.05, 1e12)
    row, why = autoconfig.choose(rows, policy)
    assert row is not None and isinstance(why, str)


def test_link_probe_over_loopback_and_duplex_classes():
    from elysium_wan_b200.resources import links

    srv, port = links.serve_echo("127.0.0.1", 0)
    try:
        r = links.measure_pair("127.0.0.1", port, flows=2, secs=0.3)
    finally:
        srv.shutdown()
    assert r["rtt_ms"] > 0 and r["up_mbps"] > 0 and r["down_mbps"] > 0
    assert links.classify_duplex(100, 100, 190) == "full"
    assert links.classify_duplex(100, 100, 100) == "half"
    assert links.classify_duplex(100, 100, 150) == "shared"
    em = links.Emulation("us", {"eu": {"rtt_ms": 120, "mbps": 500}})
    assert em.link_to("eu").rtt_ms == 120 and em.link_to("us").mbps == 0.0


def test_wide_stage_admission_and_exchange_simulator():
    from elysium_wan_b200.models.config import make_config
    from elysium_wan_b200.runtime.spec import JobSpec
    from elysium_wan_b200.scheduler import admission as ad

    # the 0.6B config as 2 stages x 4 replicas on B200s: admitted, exposure tiny
    cfg = make_config("gpt15b", n_layer=20, d_model=1536, n_head=12)
    for shard in ("zero1", "pieces"):
        spec = JobSpec(model=cfg, stages=2, stage_widths=[4, 4], microbatches=16, mb_size=4,
                       shard=shard).finalize()
        ok, reasons, pred = ad.admit(spec, [ad.Device(f"g{i}") for i in range(8)])
        assert ok, [r.text() for r in reasons]
        assert 0 <= pred[0]["exposed_s"] < 1e-3
    # pieces moves the matrices as bf16: less all-gather than ZeRO-1, same reduce-scatter
    t = ad.stage_terms(spec, 0)
    rz, az = ad.exchange_bytes(t, 4, "zero1")
    rp, ap = ad.exchange_bytes(t, 4, "pieces")
    assert rz == rp and ap < az
    assert ad.device_bytes(t, 4, "pieces", 1) < ad.device_bytes(t, 4, "zero1", 1)
    # a slow link fails S1 (and S2), a small device fails MEM, mixed classes fail class
    ok, reasons, _ = ad.admit(spec, [ad.Device(f"g{i}", link_Bps=1e9) for i in range(8)])
    kinds = {r.kind for r in reasons}
    assert not ok and {"S1", "S2"} <= kinds
    ok, reasons, _ = ad.admit(spec, [ad.Device(f"g{i}", vram_bytes=8 * 2**30) for i in range(8)])
    assert not ok and any(r.kind == "MEM" for r in reasons)
    mixed = [ad.Device(f"g{i}") for i in range(7)] + [ad.Device("h", device_class="h100")]
    ok, reasons, _ = ad.admit(spec, mixed)
    assert not ok and reasons[0].kind == "class" and "h100" in reasons[0].text()
    # need-first: with a link too slow to hide the exchange, the first unit the
    # next forward needs gets its gather before later units' gradients
    sim = ad.simulate_exchange([10, 10, 10, 10], 2, "zero1", link_Bps=1.0, c_mb=30.0)
    assert sim["exposed_s"] > 0
    ags = [u for k, u in sim["order"] if k == "ag"]
    assert ags == sorted(ags)


def _fleet(n, vram=178, device="cuda:0", cls="b200"):
    from elysium_wan_b200.resources.node import NodeInfo

    return [NodeInfo(node_id=f"n{i}", name=f"g{i}", device=device, device_class=cls,
                     vram_gb=vram, tflops_bf16=1400.0 if device.startswith("cuda") else None)
            for i in range(n)]


def test_plan_mode_prices_every_candidate_and_takes_the_fastest():
    """Plan mode enumerates (depth, moments on device / host, recompute), fits
    the largest microbatch, admits wide stages, prices each candidate's step
    and returns the fastest fitting one with the whole table."""
    from elysium_wan_b200.scheduler import admission as ad
    from elysium_wan_b200.scheduler.fleetplan import plan_job

    spec, rat = plan_job({"preset": "gpt15b"}, _fleet(8))
    priced = [r for r in rat["candidates"] if "tokens_per_s" in r]
    assert priced and len(priced) + sum(1 for r in rat["candidates"] if r.get("refused")) == \
        len(rat["candidates"])
    best = max(r["tokens_per_s"] for r in priced)
    assert rat["price"]["tokens_per_s"] == pytest.approx(best)
    assert spec.stages == rat["depth"]["stages"] and sum(spec.stage_widths) <= 8
    assert rat["width"]["spares"] == 8 - sum(spec.stage_widths)
    assert spec.mb_size >= 1 and spec.microbatches % max(spec.stage_widths) == 0
    # the winner fits: its heaviest stage within the device budget
    if max(spec.stage_widths) > 1:
        ok, reasons, _ = ad.admit(spec, ad.devices_from_nodes(_fleet(sum(spec.stage_widths))))
        assert ok, [r.text() for r in reasons]
    # a depth the plan pins is kept, and so are its microbatches and size
    spec, rat = plan_job({"preset": "gpt15b", "stages": 8, "microbatches": 64, "mb_size": 1},
                         _fleet(8))
    assert spec.stages == 8 and rat["depth"]["given"] and spec.microbatches == 64
    assert rat["mb_size"]["given"] and spec.mb_size == 1
    assert all(r["stages"] == 8 for r in rat["candidates"])
    # a model that fits one device: wide stages win over a pipeline
    spec, _ = plan_job({"preset": "gpt15b", "n_layer": 20, "d_model": 1536, "n_head": 12},
                       _fleet(8))
    assert max(spec.stage_widths) > 1 and spec.shard == "zero1"
    # small devices: host moments or recompute before giving up
    spec, rat = plan_job({"preset": "gpt15b", "n_layer": 8, "d_model": 2048, "n_head": 16},
                         _fleet(1, vram=8))
    assert spec.optimizer == "adamw-host" or spec.recompute
    with pytest.raises(ValueError, match="no candidate"):
        plan_job({"preset": "gpt15b"}, _fleet(2, vram=8))
    with pytest.raises(ValueError, match="mixed"):
        plan_job({"preset": "toy"}, _fleet(1) + _fleet(1, device="cpu", cls="cpu"))


def test_chain_routing_is_exact_and_routes_around_slow_pairs():
    """order_chain equals brute force over every ordering on random matrices
    (bottleneck first, then total RTT); best_chain reports 0 when no order
    connects every node; the heuristic beyond EXACT_MAX returns a valid order
    no worse than the identity; route_gain ignores noise."""
    import itertools
    import random

    from elysium_wan_b200.scheduler import routing as R

    rng = random.Random(7)
    for _ in range(150):
        n = rng.randint(3, 7)
        bw = [[0.0] * n for _ in range(n)]
        rtt = [[0.0] * n for _ in range(n)]
        for i in range(n):
            for j in range(i + 1, n):
                bw[i][j] = bw[j][i] = rng.choice([0, 10, 50, 100, 100, 500, 1000])
                rtt[i][j] = rtt[j][i] = rng.choice([1, 5, 20, 80, 150])
        got = R.order_chain(rtt, bw)
        assert sorted(got) == list(range(n)) and got[0] < got[-1]
        best = max(R.chain_key(list(p), bw, rtt) for p in itertools.permutations(range(n)))
        assert R.chain_key(got, bw, rtt) == best
    # a slow a-b pair: the chain goes a-c-b
    assert R.best_chain(3, [(0, 1, 5), (1, 2, 900), (0, 2, 800)]) == ([0, 2, 1], 800.0)
    assert R.best_chain(4, [(0, 1, 100), (1, 2, 100)])[1] == 0.0
    # one direction unreachable: symmetrize takes the slower direction
    r2, b2 = R.symmetrize([[0, 1], [None, 0]], [[None, 100], [50, None]])
    assert b2[0][1] == b2[1][0] == 50 and r2[0][1] == float("inf")
    n = R.EXACT_MAX + 3
    bw = [[0.0] * n for _ in range(n)]
    for i in range(n):
        for j in range(i + 1, n):
            bw[i][j] = bw[j][i] = rng.choice([10, 100, 1000])
    got = R.order_chain(None, bw)
    assert sorted(got) == list(range(n))
    assert R.chain_key(got, bw) >= R.chain_key(list(range(n)), bw)
    bw3 = [[0, 100, 100], [100, 0, 105], [100, 105, 0]]
    assert not R.route_gain([0, 1, 2], [0, 2, 1], bw3, None)
    assert R.route_gain([0, 1, 2], [0, 2, 1], [[0, 5, 100], [5, 0, 100], [100, 100, 0]], None)


def test_emulation_profile_shapes_probes():
    from elysium_wan_b200.resources import links

    em = links.Emulation.from_profile("a", {"inter": {"mbps": 100, "rtt_ms": 40},
                                            "intra": {"mbps": 0, "rtt_ms": 1},
                                            "pairs": {"a|b": {"mbps": 5, "rtt_ms": 200}}})
    assert em.shape("b", 0.2, 9000.0) == (200.0, 5.0)
    assert em.shape("c", 0.2, 9000.0) == (40.0, 100.0)
    assert em.shape("a", 0.2, 9000.0) == (1.0, 9000.0)  # rate 0: not shaped
    srv, port = links.serve_echo("127.0.0.1", 0)
    try:
        row = links.probe_row([["127.0.0.1", port, "a"], ["127.0.0.1", port, "b"]], 0,
                              secs=0.05, emu=em)
    finally:
        srv.shutdown()
    assert row["rtt_ms"][0] == 0.0 and row["bw_mbps"][0] is None
    assert row["rtt_ms"][1] >= 200.0 and row["bw_mbps"][1] <= 5.0
