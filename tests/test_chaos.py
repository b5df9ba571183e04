"""Chaos: a worker machine lost mid-run is convicted, its slot moves to the
spare, the newest common checkpoint wave is restored, every stage relaunches,
and every loss still equals the single-device oracle bit for bit.

The failure is made on the host (SIGKILL of a worker agent process and its
stage); no GPU is involved. Would fail if conviction, spare selection, wave
shipping/restore, resume or loss collection broke any bit.
"""

import pytest

from elysium_wan_b200.control.coordinator import Job
from elysium_wan_b200.launch.cluster import LocalCluster
from elysium_wan_b200.models.config import make_config
from elysium_wan_b200.runtime.spec import JobSpec
from elysium_wan_b200.validation.compare import compare
from elysium_wan_b200.validation.reference import run_baseline


@pytest.mark.slow
def test_worker_killed_heals_bitwise(tmp_path):
    cfg = make_config("toy", n_layer=4, vocab_size=97, d_model=64, n_head=4, seq_len=16)
    spec = JobSpec(model=cfg, stages=3, microbatches=2, mb_size=2, steps=8, backend="gloo",
                   ckpt_every=2, tag="chaos")
    cl = LocalCluster(str(tmp_path / "cl"), ["a", "a", "b", "b"],
                      wan_links={"a|b": {"latency_ms": 5.0, "bw_mbps": 200.0}})
    killed = {}

    def on_progress(slot, step, nid):
        if not killed and step >= 3:
            killed["w"] = cl.worker_of_slot((1, 0))
            cl.kill_worker(killed["w"])

    cl.coord.on_progress = on_progress
    try:
        res = cl.run(Job(spec=spec))
    finally:
        cl.close()
    assert res.ok, res.why
    assert res.heals == 1 and killed
    ref = JobSpec.from_dict(spec.to_dict())
    ref.out_dir = str(tmp_path / "oracle")
    ref.finalize()
    r = compare(run_baseline(ref, "reference"), res.losses_path)
    assert r["ok"] and r["compared"] == 16, r
    # the final training state (masters, moments, step) of the healed run, read
    # from the waves the coordinator collected, is byte-identical to the oracle's
    import json
    import os

    from elysium_wan_b200.validation.state import diff_manifests, distributed_manifest

    with open(os.path.join(res.run_dir, "spec.json")) as f:
        ran = JobSpec.from_dict(json.load(f))
    ran.out_dir = os.path.join(str(tmp_path / "cl"), "coordinator", "store", res.run_id)
    ran.finalize()
    with open(os.path.join(ref.out_dir, "reference_state.json")) as f:
        want = json.load(f)
    assert diff_manifests(want, distributed_manifest(ran, 8)) == []


# ---------------------------------------------------------------- more scenarios
# Same shape as above: a small GPT over gloo on CPU, a checkpoint wave every 2
# steps, the failure injected on the host once the run reaches a step, and the
# healed run's losses diffed against the single-device oracle.

def _recipe(**kw):
    cfg = make_config("toy", n_layer=4, vocab_size=97, d_model=64, n_head=4, seq_len=16)
    base = dict(model=cfg, stages=2, microbatches=2, mb_size=2, steps=10, backend="gloo",
                ckpt_every=2, tag="chaos")
    base.update(kw)
    return JobSpec(**base)


def _oracle_ok(spec, res, tmp_path):
    ref = JobSpec.from_dict(spec.to_dict())
    ref.out_dir = str(tmp_path / "oracle")
    ref.finalize()
    r = compare(run_baseline(ref, "reference"), res.losses_path)
    assert r["ok"] and r["compared"] == spec.steps * spec.microbatches, r


def _at_step(cl, step, action):
    done = {}

    def on_progress(slot, s, nid):
        if not done and s >= step:
            done["x"] = action()

    cl.coord.on_progress = on_progress
    return done


@pytest.mark.slow
def test_killed_stage_process_is_convicted_and_healed(tmp_path):
    """The agent survives, its stage process does not (no done marker): S2
    convicts that slot at once and the spare takes it."""
    spec = _recipe()
    cl = LocalCluster(str(tmp_path / "cl"), ["a"] * 3)
    victim = {}

    def act():
        victim["w"] = cl.worker_of_slot((0, 0))
        cl.kill_stage(victim["w"])
        return True

    fired = _at_step(cl, 3, act)
    try:
        res = cl.run(Job(spec=spec))
    finally:
        cl.close()
    assert fired and res.ok, res.why
    assert res.heals == 1 and res.restarts == 0
    heal = [e for e in cl.coord.events if e[0] == "heal"][0]
    assert heal[1] == (0, 0)
    assert "no done marker" in heal[2]["why"] or "gone" in heal[2]["why"], heal
    _oracle_ok(spec, res, tmp_path)


@pytest.mark.slow
def test_frozen_stage_is_restarted_in_place(tmp_path):
    """Every process alive and heartbeating but no progress (SIGSTOP of one
    stage): S4 declares a stall, every slot restarts from the common wave on
    the same nodes, nobody is replaced."""
    spec = _recipe()
    cl = LocalCluster(str(tmp_path / "cl"), ["a"] * 2,
                      liveness={"stall_floor_s": 6.0, "first_step_timeout_s": 60.0})
    fired = _at_step(cl, 3, lambda: cl.freeze_stage(cl.worker_of_slot((1, 0))) or True)
    try:
        res = cl.run(Job(spec=spec))
    finally:
        cl.close()
    assert fired and res.ok, res.why
    assert res.restarts == 1 and res.heals == 0
    _oracle_ok(spec, res, tmp_path)


@pytest.mark.slow
def test_control_plane_blip_reconnects_without_recovery(tmp_path):
    """The coordinator's connection to a worker drops; the data plane never
    notices, the agent dials back inside the grace, and the run ends with no
    heal and no restart."""
    spec = _recipe()
    cl = LocalCluster(str(tmp_path / "cl"), ["a"] * 2, liveness={"reconnect_grace_s": 20.0})
    fired = _at_step(cl, 2, lambda: cl.sever_control(cl.worker_of_slot((0, 0))) or True)
    try:
        res = cl.run(Job(spec=spec))
    finally:
        cl.close()
    assert fired and res.ok, res.why
    assert res.heals == 0 and res.restarts == 0 and res.attempts == 1
    assert any(e[0] == "reconnected" for e in cl.coord.events)
    _oracle_ok(spec, res, tmp_path)


@pytest.mark.slow
def test_no_spare_fails_with_the_reason(tmp_path):
    spec = _recipe()
    cl = LocalCluster(str(tmp_path / "cl"), ["a"] * 2)
    fired = _at_step(cl, 3, lambda: cl.kill_worker(cl.worker_of_slot((1, 0))) or True)
    try:
        res = cl.run(Job(spec=spec))
    finally:
        cl.close()
    assert fired and not res.ok
    assert "no spare" in res.why


@pytest.mark.slow
def test_wide_stage_peer_death_heals_every_shard(tmp_path):
    """A replica of a ZeRO-1 stage dies holding one optimizer shard: every
    slot, its surviving stage-mate included, resumes from the common wave and
    the run stays exact."""
    spec = _recipe(stage_widths=[2, 1], microbatches=4)
    cl = LocalCluster(str(tmp_path / "cl"), ["a"] * 4)
    fired = _at_step(cl, 3, lambda: cl.kill_worker(cl.worker_of_slot((0, 1))) or True)
    try:
        res = cl.run(Job(spec=spec))
    finally:
        cl.close()
    assert fired and res.ok, res.why
    assert res.heals == 1
    heal = [e for e in cl.coord.events if e[0] == "heal"][0]
    assert heal[1] == (0, 1)
    _oracle_ok(spec, res, tmp_path)


@pytest.mark.slow
@pytest.mark.parametrize("boundary", ["fp8_e4m3_b128", "fp16"])
def test_heal_over_tcp_with_format_boundaries(tmp_path, monkeypatch, boundary):
    """The TCP data plane (sealed multi-flow links, planes codec) in a heal: a
    replica of the wide second stage dies, its slot moves to the spare, every
    stage re-dials its links, and the run stays exact with fp8 (codes + block
    scales travelling as one frame) and fp16 boundaries."""
    monkeypatch.setenv("ELYSIUM_PEER_KEY", str(tmp_path / "peer.key"))
    cfg = make_config("toy", n_layer=4, vocab_size=97, d_model=256, n_head=4, seq_len=32,
                      boundary_dtype=boundary)
    spec = JobSpec(model=cfg, stages=2, stage_widths=[1, 2], microbatches=4, mb_size=2, steps=8,
                   backend="tcp", wire_codec="planes", p2p_streams=2, ckpt_every=2, tag="chaos")
    cl = LocalCluster(str(tmp_path / "cl"), ["a"] * 4)
    fired = _at_step(cl, 3, lambda: cl.kill_worker(cl.worker_of_slot((1, 1))) or True)
    try:
        res = cl.run(Job(spec=spec))
    finally:
        cl.close()
    assert fired and res.ok, res.why
    assert res.heals == 1
    _oracle_ok(spec, res, tmp_path)

