"""Control channel framing and admission; coordinator + agents on one box.

Would fail if: frames lost or reordered bytes, a wrong token were admitted,
or the coordinator lifecycle (register -> place -> launch -> monitor ->
complete) lost a loss or disagreed with the oracle.
"""

import socket
import threading

import pytest

from elysium_wan_b200.control.coordinator import Coordinator, CoordinatorConfig, Job
from elysium_wan_b200.launch.cluster import LocalCluster
from elysium_wan_b200.models.config import make_config
from elysium_wan_b200.runtime.spec import JobSpec
from elysium_wan_b200.transport.control import Channel, check_mac, control_dial, token_mac
from elysium_wan_b200.validation.compare import compare
from elysium_wan_b200.validation.reference import run_baseline


def test_channel_roundtrip_with_body():
    a, b = socket.socketpair()
    ca, cb = Channel(a), Channel(b)
    body = bytes(range(256)) * 1000
    t = threading.Thread(target=ca.send, args=("CKPT", body), kwargs=dict(rel="x/y", n=3))
    t.start()
    hdr, got = cb.recv()
    t.join()
    assert hdr == {"kind": "CKPT", "rel": "x/y", "n": 3} and got == body
    ca.close()
    cb.close()


def test_token_mac():
    m = token_mac("tok", "nonce", "cid")
    assert check_mac("tok", "nonce", "cid", m)
    assert not check_mac("other", "nonce", "cid", m)


def test_coordinator_rejects_bad_token(tmp_path):
    c = Coordinator("127.0.0.1", 0, CoordinatorConfig(state_dir=str(tmp_path), token="right")).start()
    try:
        ch = control_dial("127.0.0.1", c.port)
        hdr, _ = ch.recv()
        assert hdr["kind"] == "CHALLENGE"
        ch.send("HELLO", caps={}, mac=token_mac("wrong", hdr["nonce"], hdr["coordinator_id"]))
        hdr, _ = ch.recv()
        assert hdr["kind"] == "REJECT"
    finally:
        c.stop()


@pytest.mark.slow
def test_cluster_run_matches_oracle(tmp_path):
    cfg = make_config("toy", n_layer=2, vocab_size=97, d_model=64, n_head=4, seq_len=16)
    spec = JobSpec(model=cfg, stages=2, microbatches=2, mb_size=2, steps=3, backend="gloo", tag="c")
    cl = LocalCluster(str(tmp_path / "cl"), ["r0", "r0"])
    try:
        res = cl.run(Job(spec=spec))
    finally:
        cl.close()
    assert res.ok, res.why
    # every slot was profiled on its worker and the schedule solved from the measured costs
    import json
    import os

    with open(os.path.join(res.run_dir, "rationale.json")) as f:
        sched = json.load(f)["schedule"]
    assert sched["source"] == "profiled" and len(sched["costs_ms"]) == 2, sched
    # every stage's per-step summary, in the reference's WT_TELEM keys, kept in the run dir
    with open(os.path.join(res.run_dir, "telem_steps.jsonl")) as f:
        tel = [json.loads(line) for line in f]
    assert {tuple(t["slot"]) for t in tel} == {(0, 0), (1, 0)} and len(tel) == 6
    assert {"v", "step", "rank", "peer", "step_ms", "emit_us", "ops", "stall_ms", "hops",
            "recv"} <= set(tel[0]["telem"])
    # both workers were released at the end (idle for the next job)
    with open(os.path.join(res.run_dir, "result.json")) as f:
        assert sorted(json.load(f)["released"]) == ["w0", "w1"]
    # each stage's whole telemetry file, shipped as TELEMETRY when it exits and
    # named by the connection's slot
    for r, q in ((0, 0), (1, 0)):
        with open(os.path.join(res.run_dir, f"telemetry_r{r}p{q}_a0.jsonl")) as f:
            rows = [json.loads(line) for line in f if line.strip()]
        assert [x["step"] for x in rows] == [0, 1, 2] and all(x["events"] for x in rows), rows
    ref = JobSpec.from_dict(spec.to_dict())
    ref.out_dir = str(tmp_path / "oracle")
    ref.finalize()
    r = compare(run_baseline(ref, "reference"), res.losses_path)
    assert r["ok"] and r["compared"] == 6, r


def test_coordinator_probes_pipeline_hops_into_link_memory(tmp_path):
    """Workers with probe servers: the coordinator asks each hop's upstream
    worker to measure the downstream one and remembers the path."""
    import threading
    import time as _t

    from elysium_wan_b200.control.agent import WorkerAgent
    from elysium_wan_b200.control.coordinator import Coordinator, CoordinatorConfig
    from elysium_wan_b200.runtime.spec import JobSpec
    from elysium_wan_b200.models.config import make_config

    co = Coordinator(port=0, cfg=CoordinatorConfig(state_dir=str(tmp_path / "co"), no_probe=False))
    co.start()
    agents = [WorkerAgent(f"127.0.0.1:{co.port}", name=f"w{i}", workdir=str(tmp_path / f"w{i}"),
                          probe_port=0) for i in range(2)]
    for a in agents:
        threading.Thread(target=a.run, daemon=True).start()
    try:
        live = co.wait_for_workers(2, 30)
        spec = JobSpec(model=make_config("toy"), stages=2, microbatches=2, mb_size=1).finalize()
        co.slot_node = {(0, 0): live[0], (1, 0): live[1]}
        co.run_id = "probe-test"
        got = co._probe_links(spec, timeout=30)
        assert "0->1" in got and got["0->1"]["rtt_ms"] > 0
        assert co.link_memory.path("127.0.0.1", "127.0.0.1") is not None
    finally:
        for a in agents:
            a.stop.set()
        co.stop()
        _t.sleep(0.2)


def test_coordinator_routes_the_chain_around_a_slow_pair(tmp_path):
    """Three workers in regions a, b, c whose emulated a-b path is 5 Mbps: the
    probe matrix shows it, the chain is ordered a-c-b (no slow hop), and a
    full measurement far below its probe re-routes with the measured rate."""
    import json as _json
    import threading
    import time as _t

    from elysium_wan_b200.control.agent import WorkerAgent
    from elysium_wan_b200.control.coordinator import Coordinator, CoordinatorConfig

    prof = _json.dumps({"pairs": {"a|b": {"mbps": 5, "rtt_ms": 60}}})
    co = Coordinator(port=0, cfg=CoordinatorConfig(state_dir=str(tmp_path / "co"), no_probe=False,
                                                   probe_secs=0.05))
    co.start()
    agents = [WorkerAgent(f"127.0.0.1:{co.port}", name=f"w{i}", workdir=str(tmp_path / f"w{i}"),
                          region=r, wan_profile=prof, probe_port=0)
              for i, r in enumerate("abc")]
    for a in agents:
        threading.Thread(target=a.run, daemon=True).start()
    try:
        live = sorted(co.wait_for_workers(3, 30), key=lambda n: co.nodes[n].info.name)
        spec = JobSpec(model=make_config("toy", n_layer=3), stages=3, microbatches=3,
                       mb_size=1).finalize()
        got, note = co._route_chain(spec, live)
        assert note["rerouted"] and note["order"] == ["w0", "w2", "w1"], note
        assert note["probe_bw_mbps"][0][1] <= 5.0 and note["bottleneck_mbps"] > 5.0
        assert [co.nodes[n].info.name for n in got] == ["w0", "w2", "w1"]
        # a hop whose full measurement is far below its probe re-routes
        co.slot_node = {(j, 0): got[j] for j in range(3)}
        fake = {"0->1": {"up_mbps": 1.0, "down_mbps": 1.0, "rtt_ms": 300.0},
                "1->2": {"up_mbps": 1e4, "down_mbps": 1e4, "rtt_ms": 0.1}}
        order = co._reroute_on_disagreement(spec, note, fake)
        assert order is not None and order != [0, 2, 1]
        assert co._reroute_on_disagreement(
            spec, note, {"0->1": {"up_mbps": 1e9, "down_mbps": 1e9, "rtt_ms": 0.1}}) is None
    finally:
        for a in agents:
            a.stop.set()
        co.stop()
        _t.sleep(0.2)


def test_routed_job_matches_oracle(tmp_path):
    """A 3-stage job over workers in regions a, b, c with probe servers and an
    emulated 5 Mbps a-b path: the coordinator's probe matrix routes the chain
    a-c-b, measures each chosen hop in full, and the losses still equal the
    single-device oracle bit for bit (placement never changes a bit)."""
    import json
    import os

    prof = json.dumps({"pairs": {"a|b": {"mbps": 5, "rtt_ms": 60}}})
    cfg = make_config("toy", n_layer=3, vocab_size=97, d_model=64, n_head=4, seq_len=16)
    spec = JobSpec(model=cfg, stages=3, microbatches=3, mb_size=2, steps=2, backend="gloo",
                   tag="rt")
    cl = LocalCluster(str(tmp_path / "cl"), ["a", "b", "c"],
                      coord=dict(no_probe=False, probe_secs=0.05, profile=False),
                      worker_args=[["--probe-port", "0", "--wan-profile", prof]] * 3)
    try:
        res = cl.run(Job(spec=spec))
    finally:
        cl.close()
    assert res.ok, res.why
    with open(os.path.join(res.run_dir, "rationale.json")) as f:
        rat = json.load(f)
    route = rat["route"]
    # the a-b pair is never a hop: w2 (region c) sits in the middle
    assert route["order"][1] == "w2" and route["bottleneck_mbps"] > 5.0, route
    assert route["rerouted"] == (route["placed"][1] != "w2"), route
    assert set(rat["measured_links"]) == {"0->1", "1->2"}
    ref = JobSpec.from_dict(spec.to_dict())
    ref.out_dir = str(tmp_path / "oracle")
    ref.finalize()
    r = compare(run_baseline(ref, "reference"), res.losses_path)
    assert r["ok"] and r["compared"] == 6, r


def test_recut_from_telemetry_matches_oracle(tmp_path):
    """Stage 1 runs 6x slower (the timing-only seam moves when, never what):
    at a common wave the coordinator re-cuts the chain toward stage 0 from the
    measured F/B/W, converts the wave to the new cut under a new tag, relaunches
    every slot, and the 20 losses still equal the single-device oracle bit for
    bit."""
    cfg = make_config("toy", n_layer=6, vocab_size=97, d_model=64, n_head=4, seq_len=16)
    spec = JobSpec(model=cfg, stages=2, microbatches=2, mb_size=2, steps=10, backend="gloo",
                   tag="rc", ckpt_every=2, partition=[[0, 4], [4, 8]])
    cl = LocalCluster(str(tmp_path / "cl"), ["r0", "r0"],
                      coord=dict(recut_cost_s=0.0, replan_min_summaries=2, watch_slow=False,
                                 replan=False),
                      worker_env={"WANTRAIN_SIM_SLOW": "1:6"})
    try:
        res = cl.run(Job(spec=spec))
        replans = list(cl.coord.replans)
    finally:
        cl.close()
    assert res.ok, res.why
    assert replans and replans[0]["recut"], replans
    assert replans[0]["to"][0][1] > replans[0]["from"][0][1], replans  # stage 0 took entries
    ref = JobSpec.from_dict(spec.to_dict())
    ref.out_dir = str(tmp_path / "oracle")
    ref.finalize()
    r = compare(run_baseline(ref, "reference"), res.losses_path)
    assert r["ok"] and r["compared"] == 20, r


def test_rebalance_rules():
    from elysium_wan_b200.scheduler import rebalance as rb

    cfg = make_config("toy", n_layer=6, vocab_size=97, d_model=64, n_head=4, seq_len=16)
    spec = JobSpec(model=cfg, stages=2, microbatches=4, mb_size=1).finalize()
    summ = lambda f, b, w: {"ops": {"F": {"n": 4, "med_ms": f}, "B": {"n": 4, "med_ms": b},  # noqa: E731
                                    "W": {"n": 4, "med_ms": w}}}
    even = {(0, 0): [summ(1, 2, 1)] * 3, (1, 0): [summ(1, 2, 1)] * 3}
    prof = rb.profiles_from_telemetry(spec, even)
    assert prof[0][0]["t_f"] == pytest.approx(1e-3)
    # measured equal while the model says stage 1 is lighter: the cut moves toward stage 0
    # only when that shortens the slowest stage by the gain
    slow1 = {(0, 0): [summ(1, 2, 1)] * 3, (1, 0): [summ(6, 12, 6)] * 3}
    new, before, after = rb.refined_partition(spec, rb.profiles_from_telemetry(spec, slow1))
    assert new[0][1] > spec.partition[0][1] and after < before
    assert rb.recut_pays(before, after, 4, 10, 0.0)[0]
    assert not rb.recut_pays(before, after, 4, 0, 0.0)[0]
    assert rb.stage_compute_ms(summ(1, 2, 3)) == 6
    hist = {(0, 0): [10, 10, 14, 14, 14], (1, 0): [10, 14, 10, 14, 14]}
    assert rb.slow_slots(hist, {(0, 0): 10, (1, 0): 10}, 1.3, 3) == [((0, 0), 1.4)]
    with pytest.raises(ValueError):
        rb.profiles_from_telemetry(spec, {(0, 0): [], (1, 0): [summ(1, 2, 1)]})
    tied = make_config("toy", n_layer=2, tie_embeddings=True)
    assert rb.recut_refusal(JobSpec(model=tied, stages=2).finalize()) == "a tied embedding"


def test_slow_slot_moves_to_a_spare(tmp_path):
    """From step 5 on, stage 1 computes 20x slower (timing-only seam). Its
    compute per microbatch stays above 2x its own baseline for three
    summaries, so the coordinator moves the slot to the spare and resumes from
    the common wave; the losses equal the oracle."""
    cfg = make_config("toy", n_layer=2, vocab_size=97, d_model=64, n_head=4, seq_len=16)
    # the cut is pinned: a launch-time refinement would leave stage 1 a sliver
    # whose slowdown the run outlives
    spec = JobSpec(model=cfg, stages=2, microbatches=2, mb_size=2, steps=20, backend="gloo",
                   tag="slow", ckpt_every=2, partition=[[0, 2], [2, 4]])
    cl = LocalCluster(str(tmp_path / "cl"), ["r0", "r0", "r0"],
                      coord=dict(recut=False, replan=False, slow_runs=3, slow_ratio=2.0),
                      worker_env={"WANTRAIN_SIM_SLOW": "1:20@5"})
    try:
        res = cl.run(Job(spec=spec))
        heals = [e for e in cl.coord.events if e[0] == "heal"]
    finally:
        cl.close()
    assert res.ok, res.why
    assert len(heals) == 1 and heals[0][1] == (1, 0) and "baseline" in heals[0][2]["why"], heals
    ref = JobSpec.from_dict(spec.to_dict())
    ref.out_dir = str(tmp_path / "oracle")
    ref.finalize()
    r = compare(run_baseline(ref, "reference"), res.losses_path)
    assert r["ok"] and r["compared"] == 40, r


def test_plan_mode_job_through_the_coordinator(tmp_path):
    """A {plan} job without a stage count: the coordinator plans depth, width
    and layout from the registered fleet (here: one stage, two ZeRO-1
    replicas), records the rationale, and the run equals the oracle."""
    import json
    import os

    plan = {"preset": "toy", "n_layer": 2, "vocab_size": 97, "d_model": 64, "n_head": 4,
            "seq_len": 16, "microbatches": 2, "mb_size": 2, "steps": 2, "backend": "gloo"}
    cl = LocalCluster(str(tmp_path / "cl"), ["r0", "r0"])
    try:
        res = cl.run(Job(plan=plan))
    finally:
        cl.close()
    assert res.ok, res.why
    with open(os.path.join(res.run_dir, "rationale.json")) as f:
        rat = json.load(f)
    assert rat["plan"]["depth"]["stages"] == 1 and rat["plan"]["width"]["layout"] == "zero1"
    with open(os.path.join(res.run_dir, "spec.json")) as f:
        ran = JobSpec.from_dict(json.load(f))
    assert ran.stage_widths == [2]
    ref = JobSpec.from_dict(ran.to_dict())
    ref.out_dir = str(tmp_path / "oracle")
    ref.resume, ref.resume_step = False, None
    ref.finalize()
    r = compare(run_baseline(ref, "reference"), res.losses_path)
    assert r["ok"] and r["compared"] == 4, r


def test_reschedule_from_telemetry_matches_oracle(tmp_path):
    """A job launched with a GPipe-like order (all F, then all B, then all W):
    at a common wave the coordinator re-solves the zero-bubble order from the
    measured F / B / W, relaunches from the wave with it, and the losses stay
    the oracle's (an order never changes a bit)."""
    cfg = make_config("toy", n_layer=4, vocab_size=97, d_model=64, n_head=4, seq_len=16)
    M, S = 6, 3
    naive = [[[["F", m] for m in range(M)] + [["B", m] for m in range(M)]
              + [["W", m] for m in range(M)]] for _ in range(S)]
    spec = JobSpec(model=cfg, stages=S, microbatches=M, mb_size=1, steps=10, backend="gloo",
                   tag="rs", ckpt_every=2, partition=[[0, 2], [2, 4], [4, 6]],
                   schedule_order=naive)
    cl = LocalCluster(str(tmp_path / "cl"), ["r0", "r0", "r0"],
                      coord=dict(profile=False, recut=False, watch_slow=False,
                                 replan_cost_s=0.0, replan_min_gain=0.02,
                                 replan_min_summaries=2))
    try:
        res = cl.run(Job(spec=spec))
        replans = list(cl.coord.replans)
    finally:
        cl.close()
    assert res.ok, res.why
    assert replans and replans[0].get("reschedule"), replans
    ref = JobSpec.from_dict(spec.to_dict())
    ref.out_dir = str(tmp_path / "oracle")
    ref.finalize()
    r = compare(run_baseline(ref, "reference"), res.losses_path)
    assert r["ok"] and r["compared"] == M * 10, r


def test_ownership_replan_from_telemetry_matches_oracle(tmp_path):
    """One replica of a wide stage computes 4x slower from step 2 on (the
    reference's one-slot form of the timing-only seam). At a common wave the
    coordinator re-solves the stage's peer weights from the measured rates,
    re-deals the microbatches (the slow replica keeps at least one), re-solves
    the order and relaunches from the wave; the spec records the table the
    earlier steps ran under, and the losses equal the oracle that follows it."""
    import json
    import os

    cfg = make_config("toy", n_layer=4, vocab_size=97, d_model=64, n_head=4, seq_len=16)
    spec = JobSpec(model=cfg, stages=2, stage_widths=[1, 2], microbatches=8, mb_size=1,
                   steps=10, backend="gloo", tag="ow", ckpt_every=2, partition=[[0, 3], [3, 6]])
    cl = LocalCluster(str(tmp_path / "cl"), ["r0", "r0", "r0"],
                      coord=dict(profile=False, recut=False, watch_slow=False,
                                 replan_cost_s=0.0, replan_min_gain=0.1,
                                 replan_min_summaries=2),
                      worker_env={"WANTRAIN_SIM_SLOW": "1:1:4:2"})
    try:
        res = cl.run(Job(spec=spec))
        replans = list(cl.coord.replans)
    finally:
        cl.close()
    assert res.ok, res.why
    assert replans and replans[0].get("owner_changed"), replans
    with open(os.path.join(res.run_dir, "spec.json")) as f:
        ran = JobSpec.from_dict(json.load(f))
    assert ran.ownership_log and ran.ownership_log[0][1] == spec.finalize().mb_owner
    fast, slow = ran.peer_weights[1]
    assert slow < fast and ran.owned(1, 1) and len(ran.owned(1, 0)) > len(ran.owned(1, 1))
    ref = JobSpec.from_dict(ran.to_dict())
    ref.out_dir = str(tmp_path / "oracle")
    ref.resume, ref.resume_step = False, None
    ref.finalize()
    r = compare(run_baseline(ref, "reference"), res.losses_path)
    assert r["ok"] and r["compared"] == 80, r
    # the oracle of the launch ownership alone differs after the re-plan
    plain = JobSpec.from_dict(spec.to_dict())
    plain.out_dir = str(tmp_path / "oracle_plain")
    plain.finalize()
    assert not compare(run_baseline(plain, "reference"), res.losses_path)["ok"]


def test_ownership_log_and_sim_slow_rules():
    from elysium_wan_b200.runtime.telemetry import parse_sim_slow
    from elysium_wan_b200.scheduler import rebalance as rb

    assert parse_sim_slow("1:3") == {1: (3.0, 0)}
    assert parse_sim_slow("1:2@5,0:1:4:2") == {1: (2.0, 5), (0, 1): (4.0, 2)}
    for bad in ("1", "1:0.5", "a:2", "1:1:2:3:4"):
        with pytest.raises(ValueError):
            parse_sim_slow(bad)
    cfg = make_config("toy", n_layer=4, vocab_size=97, d_model=64, n_head=4, seq_len=16)
    spec = JobSpec(model=cfg, stages=2, stage_widths=[1, 2], microbatches=8, mb_size=1).finalize()
    old = spec.mb_owner
    summ = lambda f, b, w: {"ops": {"F": {"n": 4, "med_ms": f}, "B": {"n": 4, "med_ms": b},  # noqa: E731
                                    "W": {"n": 4, "med_ms": w}}}
    even = {(0, 0): [summ(1, 2, 1)] * 3, (1, 0): [summ(1, 2, 1)] * 3, (1, 1): [summ(1, 2, 1)] * 3}
    r = rb.replan_ownership(spec, rb.profiles_from_telemetry(spec, even))
    assert not r["owner_changed"] and not r["decision"]
    # one replica 8x slower: it keeps one microbatch (IWRR alone would give it none)
    slow = dict(even)
    slow[(1, 1)] = [summ(8, 16, 8)] * 3
    r = rb.replan_ownership(spec, rb.profiles_from_telemetry(spec, slow))
    assert r["decision"] and r["owner_changed"] and r["pred_new_s"] < r["pred_cur_s"]
    assert r["mb_owner"][1].count(1) >= 1 and r["mb_owner"][1].count(0) > r["mb_owner"][1].count(1)
    assert r["mb_owner"][0] == old[0]
    # the log: steps before 4 ran under the launch table
    spec.ownership_log = [[4, old]]
    spec.mb_owner = r["mb_owner"]
    spec.schedule_order = r["schedule_order"]
    spec.finalize()
    assert spec.owner_at(3) == old and spec.owner_at(4) == r["mb_owner"]
    spec.ownership_log = [[4, old], [2, old]]
    with pytest.raises(ValueError):
        spec.finalize()


def test_unrouted_chain_gives_the_hungriest_rank_the_largest_card(tmp_path):
    """Without probing, a chain on cards of different memory is ordered so the
    rank needing the most memory gets the largest card; equal cards keep the
    placement's order."""
    from elysium_wan_b200.control.coordinator import Coordinator, CoordinatorConfig, _Node
    from elysium_wan_b200.resources.node import NodeInfo
    from elysium_wan_b200.scheduler.placement import rank_memory_need

    co = Coordinator(port=0, cfg=CoordinatorConfig(state_dir=str(tmp_path / "co")))
    try:
        spec = JobSpec(model=make_config("toy", n_layer=4), stages=3, microbatches=3,
                       mb_size=1).finalize()
        need = rank_memory_need(spec)
        for k, gb in enumerate([40, 180, 80]):
            co.nodes[f"n{k}"] = _Node(NodeInfo.from_caps(f"n{k}", {"vram_gb": gb}), None)
        live = ["n0", "n1", "n2"]
        got = co._memory_order(spec, live)
        mem = {"n0": 40, "n1": 180, "n2": 80}
        hungriest = max(range(3), key=lambda r: (need[r], -r))
        assert mem[got[hungriest]] == 180, (need, got)
        for k in range(3):
            co.nodes[f"n{k}"] = _Node(NodeInfo.from_caps(f"n{k}", {"vram_gb": 80}), None)
        assert co._memory_order(spec, live) == live
    finally:
        co.nodes.clear()  # never started: no socket, and the fake nodes have no channel


def test_control_channel_streams_large_bodies_to_disk(tmp_path):
    """A file body at least spill_min long is streamed from disk by the sender
    and into a file by the receiver (sha256 computed on the way), then renamed
    into place; small bodies stay in memory."""
    import os
    import socket
    import threading

    from elysium_wan_b200.transport.control import Channel, Spilled, body_sha256, write_body

    a, b = socket.socketpair()
    tx, rx = Channel(a), Channel(b, spill_dir=str(tmp_path / "spill"))
    rx.spill_min = 1 << 16
    src = tmp_path / "state.pt"
    payload = os.urandom(3 << 20)
    src.write_bytes(payload)
    t = threading.Thread(target=lambda: (tx.send_file("CKPT", str(src), name="state.pt"),
                                         tx.send("HEARTBEAT", b"x" * 10)))
    t.start()
    hdr, body = rx.recv()
    assert hdr["kind"] == "CKPT" and isinstance(body, Spilled) and len(body) == len(payload)
    import hashlib

    assert body_sha256(body) == hdr["sha256"] == hashlib.sha256(payload).hexdigest()
    dst = tmp_path / "placed.pt"
    write_body(body, str(dst))
    assert dst.read_bytes() == payload and not os.path.exists(body.path)
    hdr2, small = rx.recv()
    assert hdr2["kind"] == "HEARTBEAT" and small == b"x" * 10
    t.join(10)
    a.close()
    b.close()


def _fit_rig(tmp_path, spec, mem_of_stage, over=1.3):
    """A coordinator (not started) whose slots sit on nodes of the given
    device memory, and a fake FIT whose device uses `over` x what the memory
    model says: resident state, then the order's in-flight microbatches of F
    activations."""
    from elysium_wan_b200.control.coordinator import Coordinator, CoordinatorConfig, _Node
    from elysium_wan_b200.resources.fit import peak_pending
    from elysium_wan_b200.resources.node import NodeInfo
    from elysium_wan_b200.scheduler import admission as ad
    from elysium_wan_b200.scheduler.planner import stage_memory_model

    co = Coordinator("127.0.0.1", 0, CoordinatorConfig(state_dir=str(tmp_path / "st")))
    for r, p in spec.slots():
        nid = f"n{r}{p}"
        info = NodeInfo(node_id=nid, name=nid, device="cuda", device_class="B200",
                        vram_gb=mem_of_stage[r] / 2**30)
        co.nodes[nid] = _Node(info, None)
        co.slot_node[(r, p)] = nid
    calls = []

    def fake(kind, result, sp, slots, timeout):
        assert kind == "FIT"
        calls.append([list(x) for x in sp.partition])
        out = {}
        for r, p in slots:
            mf = stage_memory_model(sp, r)[0]
            base = over * ad.device_bytes(ad.stage_terms(sp, r), sp.stage_widths[r], sp.shard, 0)
            k = peak_pending(sp.schedule_order[r][p])
            out[(r, p)] = {"ok": True, "fits": True, "peak_bytes": base + over * k * mf,
                           "base_bytes": base}
        return out

    co._ask_slots = fake
    return co, calls


def test_fit_loop_recomputes_then_calibrates_the_schedule(tmp_path):
    """A stage whose measured peak is above its node's budget first recomputes;
    when that is not enough, its schedule is solved again under a budget
    calibrated from the measurement (fewer microbatches in flight), and the
    cut stays."""
    from elysium_wan_b200.resources.fit import peak_pending
    from elysium_wan_b200.scheduler import admission as ad
    from elysium_wan_b200.scheduler.planner import stage_memory_model

    cfg = make_config("toy", n_layer=6, vocab_size=97, d_model=256, n_head=4, seq_len=256)
    spec = JobSpec(model=cfg, stages=3, microbatches=12, mb_size=4, backend="gloo",
                   partition=[[0, 3], [3, 5], [5, 8]]).finalize()
    # stage 0's node: room for its state and about 1.4 microbatches of
    # recomputed activations in flight (its order holds 3 or more)
    rec = JobSpec.from_dict(spec.to_dict())
    rec.recompute = True
    rec.schedule_order = None
    rec.finalize()
    state0 = 1.3 * ad.device_bytes(ad.stage_terms(rec, 0), 1, "zero1", 0)
    mf0 = stage_memory_model(rec, 0)[0]
    assert peak_pending(rec.schedule_order[0][0]) >= 3
    budget0 = state0 + 1.3 * 1.4 * mf0
    mem0 = budget0 / 0.88 if 0.12 * budget0 / 0.88 >= 2**30 else budget0 + 2**30
    co, calls = _fit_rig(tmp_path, spec, [mem0, 1e12, 1e12])
    ok, why, notes = co._fit_loop(spec, spec.slots(), cut_given=True)
    assert ok, (why, notes)
    assert "recompute" in notes[0] and "schedule holds at most" in notes[1], notes
    assert spec.recomputes(0) and not spec.recomputes(1) and not spec.recomputes(2)
    assert peak_pending(spec.schedule_order[0][0]) == 1
    assert spec.partition == [[0, 3], [3, 5], [5, 8]] and len(calls) == 3


def test_fit_loop_recuts_when_the_state_itself_overflows(tmp_path):
    """A node too small for its stage's resident state: recompute and a
    smaller schedule cannot help, so the stage plans with less memory and
    the chain is cut again, moving layers off it; a pinned cut is refused
    with the reason instead."""
    from elysium_wan_b200.scheduler import admission as ad

    cfg = make_config("toy", n_layer=6, vocab_size=97, d_model=256, n_head=4, seq_len=64)

    def fresh(part=None):
        return JobSpec(model=cfg, stages=2, microbatches=4, mb_size=1, backend="gloo",
                       partition=part or [[0, 4], [4, 8]]).finalize()

    spec = fresh()
    state0 = 1.3 * ad.device_bytes(ad.stage_terms(spec, 0), 1, "zero1", 0)
    budget0 = 0.8 * state0
    mem0 = budget0 / 0.88 if 0.12 * budget0 / 0.88 >= 2**30 else budget0 + 2**30
    co, calls = _fit_rig(tmp_path, spec, [mem0, 1e12])
    ok, why, notes = co._fit_loop(spec, spec.slots(), cut_given=False)
    assert ok, (why, notes)
    assert "recompute" in notes[0] and "re-cut" in notes[-1], notes
    assert spec.partition[0][1] < 4, spec.partition
    pinned = fresh()
    co, _ = _fit_rig(tmp_path / "b", pinned, [mem0, 1e12])
    ok, why, notes = co._fit_loop(pinned, pinned.slots(), cut_given=True)
    assert not ok and "does not fit" in why and "stage 0 peaks" in why, why


def test_fit_check_runs_on_every_slot_before_launch(tmp_path):
    """With the fit check on, every slot (a pieces replica among them) builds
    its slice, holds its order's in-flight microbatches and steps its
    optimizer before launch; the run's rationale records no remedy and the
    losses equal the oracle."""
    import json
    import os

    cfg = make_config("toy", n_layer=4, vocab_size=97, d_model=64, n_head=4, seq_len=16)
    spec = JobSpec(model=cfg, stages=2, stage_widths=[1, 2], shard="pieces", microbatches=4,
                   mb_size=2, steps=2, backend="gloo", tag="fit")
    cl = LocalCluster(str(tmp_path / "cl"), ["r0", "r0", "r0"], coord=dict(no_fit_check=False))
    try:
        res = cl.run(Job(spec=spec))
    finally:
        cl.close()
    assert res.ok, res.why
    with open(os.path.join(res.run_dir, "rationale.json")) as f:
        assert json.load(f)["fit"] == []
    with open(os.path.join(res.run_dir, "spec.json")) as f:
        ran = JobSpec.from_dict(json.load(f))
    ref = JobSpec.from_dict(ran.to_dict())
    ref.out_dir = str(tmp_path / "oracle")
    ref.finalize()
    r = compare(run_baseline(ref, "reference"), res.losses_path)
    assert r["ok"] and r["compared"] == 8, r


def test_hops_from_telemetry_counts_transfers_and_feed_the_replan():
    """Per-hop transfer time from the TCP plane's per-link statistics: the
    median of busy_ms / frames over the links across the hop (a frame counts
    once whatever its fragments), None where nothing was measured; a slow
    measured hop lengthens the re-plan's predicted step."""
    from elysium_wan_b200.scheduler import rebalance as rb

    cfg = make_config("toy", n_layer=4, vocab_size=97, d_model=64, n_head=4, seq_len=16)
    spec = JobSpec(model=cfg, stages=3, stage_widths=[1, 2, 1], microbatches=4,
                   mb_size=1).finalize()
    ops = {"F": {"n": 2, "med_ms": 1.0}, "B": {"n": 2, "med_ms": 2.0}, "W": {"n": 2, "med_ms": 1.0}}
    win = {(0, 0): [{"ops": ops, "hops": {"frames": 9, "bytes": 1,
                                          "next0": {"frames": 2, "bytes": 8, "busy_ms": 40.0},
                                          "next1": {"frames": 2, "bytes": 8, "busy_ms": 60.0}}}],
           (1, 0): [{"ops": ops, "hops": {"prev0": {"frames": 2, "bytes": 8, "busy_ms": 50.0},
                                          "mesh1": {"frames": 1, "bytes": 8, "busy_ms": 999.0}}}],
           (1, 1): [{"ops": ops, "hops": {"frames": 3, "bytes": 5}}],
           (2, 0): [{"ops": ops, "hops": {}}]}
    hops = rb.hops_from_telemetry(spec, win)
    assert hops[0] == pytest.approx(0.025) and hops[1] is None
    prof = rb.profiles_from_telemetry(spec, win)
    fast = rb.replan_ownership(spec, prof, 0.0, [0.0, 0.0])
    slow = rb.replan_ownership(spec, prof, 0.0, [0.05, 0.0])
    assert slow["pred_cur_s"] > fast["pred_cur_s"]


def test_a_stage_log_that_cannot_be_written_never_stops_the_pump(tmp_path):
    """The agent copies a stage's output to a log file while it forwards the
    marker lines. When that file cannot be written (disk full), every line
    still reaches the handler and the stage never blocks on a full pipe."""
    import sys

    import os

    from elysium_wan_b200.control.agent import StageProcess

    class Full:
        def write(self, _):
            raise OSError(28, "No space left on device")

        def flush(self):
            pass

        def close(self):
            pass

    seen = []
    prog = "import sys\nfor i in range(20000): print(f'WT_STEP {i}')\nprint('WT_DONE 0')\n"
    sp = StageProcess([sys.executable, "-c", prog], dict(os.environ), seen.append,
                      str(tmp_path / "stage.log"))
    sp.log.close()
    sp.log = Full()
    import threading

    rc: list = []
    t = threading.Thread(target=lambda: rc.append(sp.wait()), daemon=True)
    t.start()
    t.join(60)
    if not rc:
        sp.kill()
        pytest.fail("the stage blocked: its output was no longer read")
    assert rc == [0]
    assert len(seen) == 20001 and seen[-1] == "WT_DONE 0" and sp.done_marker


def test_a_send_the_peer_never_drains_fails_instead_of_blocking(monkeypatch):
    """A control channel whose peer stops reading: once the socket buffers are
    full, the send gives up after the stall limit and the no-progress budget
    and fails like a lost peer, instead of blocking its thread (and any lock
    it holds) for good."""
    import socket
    import time

    from elysium_wan_b200.transport import control, sendall

    monkeypatch.setattr(control, "SEND_STALL_S", 1)
    monkeypatch.setattr(sendall, "RETRY_BUDGET_S", 0.5)
    a, b = socket.socketpair()
    ch = control.Channel(a)
    t0 = time.monotonic()
    with pytest.raises(OSError):
        ch.send("BIG", body=b"x" * (64 << 20))  # b never reads
    assert time.monotonic() - t0 < 30
    a.close()
    b.close()
