"""Liveness verdicts on crafted slot states, checkpoint waves, replacement.

Would fail if: a killed stage were not convicted at once, a WAN blip inside
the reconnect grace convicted anyone, two simultaneous failures triggered a
heal instead of "failed", heartbeat silence convicted on the first strike, a
deterministic crash were healed, a stall with everyone alive were not a
restart, a wave with a flipped byte validated, or pruning kept more than
WAVE_KEEP waves.
"""

import os

import pytest
import torch

from elysium_wan_b200.fault_tolerance import checkpoint as ckpt
from elysium_wan_b200.fault_tolerance.liveness import PEER_LOST, LivenessJudge, SlotState
from elysium_wan_b200.fault_tolerance.replacement import find_replacement
from elysium_wan_b200.models.config import make_config
from elysium_wan_b200.resources.node import NodeInfo
from elysium_wan_b200.runtime.spec import JobSpec

NOW = 1000.0


def slots(n=3, **kw):
    out = []
    for i in range(n):
        st = SlotState(slot=(i, 0), node_id=f"n{i}", launched=True, last_heartbeat=NOW - 1,
                       started_at=NOW - 50)
        for k, v in kw.items():
            setattr(st, k, v)
        out.append(st)
    return out


def test_all_exit_clean_is_done():
    ss = slots(exit_code=0, done_marker=True)
    assert LivenessJudge().judge(ss, NOW).kind == "done"


def test_killed_stage_is_convicted_at_once():
    ss = slots()
    ss[1].exit_code, ss[1].done_marker = -9, False
    v = LivenessJudge().judge(ss, NOW)
    assert v.kind == "convict" and v.slot == (1, 0)


def test_blip_inside_reconnect_grace_is_only_suspect():
    ss = slots()
    ss[2].connected, ss[2].disconnected_at = False, NOW - 5
    v = LivenessJudge(reconnect_grace_s=30).judge(ss, NOW)
    assert v.kind == "suspect"


def test_disconnect_past_grace_convicts():
    ss = slots()
    ss[2].connected, ss[2].disconnected_at = False, NOW - 40
    v = LivenessJudge(reconnect_grace_s=30).judge(ss, NOW)
    assert v.kind == "convict" and v.slot == (2, 0)


def test_two_failures_at_once_fail_without_heal():
    ss = slots()
    for i in (0, 2):
        ss[i].exit_code, ss[i].done_marker = -9, False
    assert LivenessJudge().judge(ss, NOW).kind == "failed"


def test_deterministic_crash_is_failed_not_healed():
    ss = slots()
    ss[0].exit_code, ss[0].done_marker, ss[0].log_tail = 1, True, "ValueError: bad"
    assert LivenessJudge().judge(ss, NOW).kind == "failed"


def test_heartbeat_silence_needs_two_strikes():
    j = LivenessJudge(heartbeat_timeout_s=10, strike_gap_s=5)
    ss = slots()
    ss[1].last_heartbeat = NOW - 20
    assert j.judge(ss, NOW).kind == "suspect"
    assert j.judge(ss, NOW + 2).kind == "suspect"
    v = j.judge(ss, NOW + 6)
    assert v.kind == "convict" and v.slot == (1, 0)


def test_peer_lost_with_silent_slot_convicts_the_silent_one():
    j = LivenessJudge(heartbeat_timeout_s=10, strike_gap_s=1, exit_report_grace_s=1)
    ss = slots()
    ss[0].exit_code, ss[0].done_marker, ss[0].log_tail = 1, True, f"WT_ERROR {PEER_LOST}: x"
    ss[2].last_heartbeat = NOW - 30
    assert j.judge(ss, NOW).kind == "suspect"
    v = j.judge(ss, NOW + 2)
    assert v.kind == "convict" and v.slot == (2, 0)


def test_everyone_alive_but_no_progress_is_stalled():
    j = LivenessJudge(first_step_timeout_s=100)
    ss = slots(started_at=NOW - 500)
    assert j.judge(ss, NOW).kind == "stalled"


def test_stage_reported_gone_convicts_after_the_exit_report_grace():
    """S2 without an exit report: the agent says its stage process is gone;
    the judge waits the exit-report grace for an explaining EXIT, then
    convicts that slot."""
    j = LivenessJudge(exit_report_grace_s=5)
    ss = slots()
    ss[1].stage_alive = False
    assert j.judge(ss, NOW).kind == "ok"
    assert j.judge(ss, NOW + 4).kind == "ok"
    v = j.judge(ss, NOW + 6)
    assert v.kind == "convict" and v.slot == (1, 0)
    ss[1].stage_alive = True  # it came back: the memory is dropped
    assert j.judge(ss, NOW + 7).kind == "ok"


def test_stall_limit_follows_the_median_step():
    """S4 after the first steps: the limit is max(floor, steps x median step)."""
    j = LivenessJudge(stall_floor_s=10, stall_steps=4, heartbeat_timeout_s=1e9)
    ss = slots()
    for st in ss:
        for k in range(5):
            st.add_progress(k, NOW + 3.0 * k, None)  # 3 s per step
    last = NOW + 12.0
    assert j.judge(ss, last + 11).kind == "ok"  # under 4 x 3 = 12 s
    assert j.judge(ss, last + 13).kind == "stalled"


def test_shutdown_quiet_is_bounded():
    """After every slot reached the final step, quiet is not a stall, but a
    shutdown that takes longer than the limit fails the job."""
    j = LivenessJudge(final_step=3, shutdown_limit_s=50, heartbeat_timeout_s=1e9, stall_floor_s=1)
    ss = slots()
    for st in ss:
        for k in range(4):
            st.add_progress(k, NOW + k, 3)
    ss[0].exit_code, ss[0].done_marker = 0, True
    assert j.judge(ss, NOW + 3 + 40).kind == "ok"
    v = j.judge(ss, NOW + 3 + 60)
    assert v.kind == "failed" and "shutdown" in v.why


def test_several_silent_suspects_wait_instead_of_convicting():
    j = LivenessJudge(heartbeat_timeout_s=10, first_step_timeout_s=100, strike_gap_s=1)
    ss = slots(started_at=NOW - 500)
    ss[0].last_heartbeat = ss[2].last_heartbeat = NOW - 30
    v = j.judge(ss, NOW)
    assert v.kind == "suspect" and v.slot is None and set(v.slots) == {(0, 0), (2, 0)}
    assert j.judge(ss, NOW + 5).kind == "suspect"


def test_rule_table_is_walked_in_order():
    """The decision table names every verdict path; its last rule always holds."""
    from elysium_wan_b200.fault_tolerance.liveness import RULES

    names = [r.name for r in RULES]
    assert names[0] == "nothing launched" and names[-1] == "everyone alive, no progress"
    assert names.index("S1/S2 against one slot") < names.index("connection down inside the grace")
    assert names.index("a stage raised its own error") < names.index("no S3/S4 suspects")


def test_progress_must_increase_within_attempt():
    st = SlotState(slot=(0, 0), node_id="n", start_step=4)
    assert not st.add_progress(3, 1.0, 10)
    assert st.add_progress(4, 1.0, 10)
    assert not st.add_progress(4, 2.0, 10)
    assert not st.add_progress(11, 3.0, 10)


def _spec(tmp_path):
    return JobSpec(model=make_config("toy", n_layer=2), stages=2, out_dir=str(tmp_path), tag="t").finalize()


def test_wave_commit_validate_prune_and_corruption(tmp_path):
    spec = _spec(tmp_path)
    for step in (2, 4, 6, 8):
        ckpt.commit_wave(spec, 1, 0, step, {"step": step, "x": list(range(10))})
    assert ckpt.list_waves(spec.out_dir, "t", 1, 0) == [4, 6, 8]
    d = ckpt.wave_dir(spec.out_dir, "t", 1, 0, 8)
    ckpt.validate_wave(d)
    assert os.path.exists(os.path.join(spec.out_dir, "t_ckpt_rank1p0.pt"))
    p = os.path.join(d, "state.pt")
    b = bytearray(open(p, "rb").read())
    b[-5] ^= 0xFF
    open(p, "wb").write(bytes(b))
    with pytest.raises(ValueError):
        ckpt.validate_wave(d)
    state, step = ckpt.load_latest(spec, 1, 0)
    assert step == 6  # the corrupted newest wave is skipped


def test_resume_refuses_mislabelled_padded_and_foreign_waves(tmp_path):
    """A wave whose manifest names another step, one with a file the manifest
    does not list, and one whose listed state is not a checkpoint are not
    resumed from: the first two are skipped like a corrupted wave, the last
    is refused with the reason."""
    import json

    spec = _spec(tmp_path)
    for step in (2, 4, 6):
        ckpt.commit_wave(spec, 0, 0, step, {"step": step})
    d6 = ckpt.wave_dir(spec.out_dir, "t", 0, 0, 6)
    meta = json.load(open(os.path.join(d6, "wave.json")))
    meta["step"] = 8
    json.dump(meta, open(os.path.join(d6, "wave.json"), "w"))
    with pytest.raises(ValueError, match="names step 8"):
        ckpt.validate_wave(d6, 6)
    open(os.path.join(ckpt.wave_dir(spec.out_dir, "t", 0, 0, 4), "extra.bin"), "wb").write(b"x")
    state, step = ckpt.load_latest(spec, 0, 0)
    assert step == 2  # 6 mislabelled, 4 padded
    with pytest.raises(FileNotFoundError):
        ckpt.load_latest(spec, 0, 0, 6)
    # a manifest that lists garbage as state.pt (its hash is right)
    d2 = ckpt.wave_dir(spec.out_dir, "t", 0, 0, 2)
    open(os.path.join(d2, "state.pt"), "wb").write(b"not a torch file")
    meta = json.load(open(os.path.join(d2, "wave.json")))
    meta["files"]["state.pt"] = {"sha256": ckpt._sha256(os.path.join(d2, "state.pt")),
                                 "size": os.path.getsize(os.path.join(d2, "state.pt"))}
    json.dump(meta, open(os.path.join(d2, "wave.json"), "w"))
    with pytest.raises(ValueError, match="not a checkpoint"):
        ckpt.load_latest(spec, 0, 0, 2)


def test_resume_drops_the_abandoned_timeline_and_sweeps_temps(tmp_path):
    """Resuming at step 4 removes the slot's waves 6 and 8 (they belong to the
    timeline the run abandoned) and a killed writer's temporaries, and the
    alias follows the newest wave left; a fresh launch keeps none. The
    coordinator's store drops every slot's newer waves, except a pinned one."""
    spec = _spec(tmp_path)
    for step in (4, 6, 8):
        ckpt.commit_wave(spec, 0, 0, step, {"step": step})
    d = ckpt.slot_dir(spec.out_dir, "t", 0, 0)
    os.makedirs(os.path.join(d, "step-00000010.staging"))
    os.makedirs(os.path.join(d, "step-00000006.replaced"))
    assert ckpt.drop_after(spec.out_dir, "t", 0, 0, 4) == [6, 8]
    assert sorted(os.listdir(d)) == ["step-00000004"]
    alias = os.path.join(spec.out_dir, "t_ckpt_rank0p0.pt")
    w4 = os.path.join(ckpt.wave_dir(spec.out_dir, "t", 0, 0, 4), "state.pt")
    assert open(alias, "rb").read() == open(w4, "rb").read()
    assert ckpt.drop_after(spec.out_dir, "t", 0, 0, -1) == [4]
    assert ckpt.list_waves(spec.out_dir, "t", 0, 0) == [] and not os.path.exists(alias)
    # the store
    store = ckpt.CheckpointStore(str(tmp_path / "store"))
    src = JobSpec.from_dict(spec.to_dict())
    src.out_dir = str(tmp_path / "src")
    for r in (0, 1):
        for step in (2, 4, 6):
            ckpt.commit_wave(src, r, 0, step, {"step": step})
            wd = ckpt.wave_dir(src.out_dir, "t", r, 0, step)
            for name in ("state.pt", "wave.json"):
                store.stage_part("run1", r, 0, step, name, open(os.path.join(wd, name), "rb").read())
            assert store.commit_staged("run1", "t", r, 0, step)
    store.stage_part("run1", 1, 0, 8, "state.pt", b"half a wave")
    store.pinned.add(6)
    assert store.drop_after("run1", "t", 2) == [("r0p0", 4), ("r1p0", 4)]
    view = JobSpec.from_dict(spec.to_dict())
    view.out_dir = os.path.join(store.root, "run1")
    assert ckpt.list_waves(view.out_dir, "t", 0, 0) == [2, 6]
    assert not os.path.exists(os.path.join(store.root, "run1", ".incoming", "r1p0", "step-00000008"))
    store.pinned.clear()
    store.drop_after("run1", "t", 2)
    assert store.common_step("run1", spec) == 2


def test_resume_refuses_fewer_steps_than_the_wave_holds(tmp_path):
    """A wave of step 6 does not resume a run of 4 steps (it would train
    nothing and report a finished run); as many or more steps resume."""
    spec = _spec(tmp_path)
    ckpt.commit_wave(spec, 0, 0, 6, {"step": 6})
    spec.steps = 4
    with pytest.raises(ValueError, match="past the run"):
        ckpt.load_latest(spec, 0, 0)
    spec.steps = 6
    assert ckpt.load_latest(spec, 0, 0)[1] == 6


def test_resume_refuses_other_recipe(tmp_path):
    spec = _spec(tmp_path)
    ckpt.commit_wave(spec, 0, 0, 2, {"step": 2})
    spec.lr = 0.5
    with pytest.raises(ValueError, match="lr"):
        ckpt.load_latest(spec, 0, 0)


def test_common_step(tmp_path):
    spec = _spec(tmp_path)
    ckpt.commit_wave(spec, 0, 0, 2, {})
    ckpt.commit_wave(spec, 0, 0, 4, {})
    ckpt.commit_wave(spec, 1, 0, 2, {})
    assert ckpt.common_step(spec) == 2


def test_replacement_prefers_same_class_and_region():
    dead = NodeInfo("n0", "w0", region="eu", device_class="b200")
    cands = [NodeInfo("n1", "w1", region="us", device_class="b200"),
             NodeInfo("n2", "w2", region="eu", device_class="b200"),
             NodeInfo("n3", "w3", region="eu", device_class="cpu")]
    assert find_replacement(dead, cands).node_id == "n2"
    assert find_replacement(dead, [cands[2]], match="device") is None


def test_replacement_never_picks_a_dead_spare_even_on_loopback():
    """A spare whose node is not alive is refused whatever its host (the
    loopback exemption only lifts the dead-host memory)."""
    dead = NodeInfo("n0", "w0", host="127.0.0.1", device_class="b200")
    gone = NodeInfo("n1", "w1", host="127.0.0.1", device_class="b200")
    gone.alive = False
    live = NodeInfo("n2", "w2", host="127.0.0.1", device_class="b200")
    assert find_replacement(dead, [gone]) is None
    assert find_replacement(dead, [gone, live], dead_hosts={"127.0.0.1"}).node_id == "n2"
    remote = NodeInfo("n3", "w3", host="10.0.0.7", device_class="b200")
    assert find_replacement(dead, [remote], dead_hosts={"10.0.0.7"}) is None


def _wave_parts(tmp_path, spec, stage, peer, step):
    """The files of a committed worker wave: {name: bytes}."""
    d = ckpt.commit_wave(spec, stage, peer, step, {"step": step})
    return {n: open(os.path.join(d, n), "rb").read() for n in os.listdir(d)}


def test_store_keeps_half_shipped_waves_out_of_the_resume_point(tmp_path):
    """A slot that dies after shipping state.pt but before wave.json leaves
    nothing in the store's wave tree: the common step stays the previous
    whole wave, and only a validated wave is renamed into place."""
    spec = _spec(tmp_path / "w")
    store = ckpt.CheckpointStore(str(tmp_path / "store"))
    run = "run1"
    for step in (2, 4):
        for r in (0, 1):
            parts = _wave_parts(tmp_path, spec, r, 0, step)
            names = sorted(parts, key=lambda n: n == "wave.json")
            for n in names:
                if step == 4 and r == 1 and n == "wave.json":
                    break  # slot 1 dies before its last part of step 4
                store.stage_part(run, r, 0, step, n, parts[n])
                if n == "wave.json":
                    assert store.commit_staged(run, spec.tag, r, 0, step)
    view = _spec(tmp_path / "store" / run)
    assert ckpt.list_waves(view.out_dir, spec.tag, 1, 0) == [2]
    assert ckpt.common_step(view) == 2
    # a wave whose wave.json names another step is refused and dropped
    parts = _wave_parts(tmp_path, spec, 0, 0, 6)
    for n in sorted(parts, key=lambda n: n == "wave.json"):
        store.stage_part(run, 1, 0, 6, n, parts[n])
    assert not store.commit_staged(run, spec.tag, 1, 0, 6)
    assert ckpt.list_waves(view.out_dir, spec.tag, 1, 0) == [2]


@pytest.mark.parametrize("name", ["../../x", "/etc/passwd", "a/b", "..", ".hidden", "", "x\0y"])
def test_store_refuses_part_names_that_leave_the_slot(tmp_path, name):
    store = ckpt.CheckpointStore(str(tmp_path / "store"))
    with pytest.raises(ValueError):
        store.stage_part("run1", 0, 0, 2, name, b"data")
    with pytest.raises(ValueError):
        store.stage_part("../run", 0, 0, 2, "state.pt", b"data")
    with pytest.raises(ValueError):
        store.stage_part("run1", 0, 0, -1, "state.pt", b"data")
    assert not os.path.exists(tmp_path / "x") and not os.path.exists(tmp_path / "run")


def test_store_pins_the_restored_wave_against_pruning(tmp_path):
    spec = _spec(tmp_path / "w")
    store = ckpt.CheckpointStore(str(tmp_path / "store"))
    store.pinned.add(2)
    for step in (2, 4, 6, 8, 10):
        parts = _wave_parts(tmp_path, spec, 0, 0, step)
        for n in sorted(parts, key=lambda n: n == "wave.json"):
            store.stage_part("run1", 0, 0, step, n, parts[n])
        assert store.commit_staged("run1", spec.tag, 0, 0, step)
    view = _spec(tmp_path / "store" / "run1")
    assert ckpt.list_waves(view.out_dir, spec.tag, 0, 0) == [2, 6, 8, 10]


def test_recut_resume_continues_the_run_bitwise(tmp_path):
    """Waves of a 2-stage run at step 2, re-cut to a 3-stage partition, resume
    to step 4: every loss equals the uninterrupted run's."""
    import json as _json
    import os as _os

    from elysium_wan_b200.fault_tolerance.recut import recut
    from elysium_wan_b200.launch.local import run_local
    from elysium_wan_b200.models.config import make_config
    from elysium_wan_b200.runtime.spec import JobSpec

    cfg = make_config("toy", n_layer=4, vocab_size=97, d_model=64, n_head=4, seq_len=16)
    base = 33000 + _os.getpid() % 300 * 11

    def spec(stages, partition, steps, out, tag, resume=False, port=0):
        s = JobSpec(model=cfg, stages=stages, partition=partition, microbatches=2, mb_size=2,
                    steps=steps, out_dir=str(out), tag=tag, ckpt_every=1, resume=resume,
                    port_base=base + port, backend="gloo")
        return s.finalize()

    full = run_local(spec(2, [[0, 3], [3, 6]], 4, tmp_path / "full", "run"), timeout=300)
    part = spec(2, [[0, 3], [3, 6]], 2, tmp_path / "cut", "run", port=3)
    run_local(part, timeout=300)
    new = spec(3, [[0, 2], [2, 4], [4, 6]], 4, tmp_path / "cut", "run", resume=True, port=6)
    assert recut(part, new) == 2
    resumed = run_local(new, timeout=300)
    with open(full) as f:
        want = {(r["step"], r["mb"]): r["loss_hex"] for r in _json.load(f)["losses"]}
    with open(resumed) as f:
        got = {(r["step"], r["mb"]): r["loss_hex"] for r in _json.load(f)["losses"]}
    later = {k: v for k, v in want.items() if k[0] >= 2}
    assert later and all(got.get(k) == v for k, v in later.items()), (later, got)


def test_logical_checkpoint_converts_cut_width_and_shard_mode(tmp_path):
    """Waves of a [1, 2]-wide ZeRO-1 run at step 2 go through the logical form
    (saved to and verified from disk): (a) re-laid as pieces at the same
    widths, the resumed run continues the uninterrupted run bit for bit (the
    fold tree is unchanged); (b) re-laid over another cut, widths and shard
    mode, gathering those waves gives back the same logical state exactly.
    (Changing a stage's width changes its declared gradient fold, hence the
    zero1_widths pin.)"""
    import json as _json
    import os as _os

    from elysium_wan_b200.fault_tolerance import logical
    from elysium_wan_b200.launch.local import run_local
    from elysium_wan_b200.models.config import make_config
    from elysium_wan_b200.runtime.spec import JobSpec

    cfg = make_config("toy", n_layer=4, vocab_size=97, d_model=64, n_head=4, seq_len=16)
    base = 36000 + _os.getpid() % 300 * 11

    def spec(stages, widths, partition, steps, out, shard="zero1", resume=False, port=0):
        return JobSpec(model=cfg, stages=stages, stage_widths=widths, partition=partition,
                       shard=shard, microbatches=4, mb_size=2, steps=steps, out_dir=str(out),
                       tag="run", ckpt_every=1, resume=resume, port_base=base + port,
                       backend="gloo").finalize()

    full = run_local(spec(2, [1, 2], [[0, 3], [3, 6]], 4, tmp_path / "full"), timeout=300)
    old = spec(2, [1, 2], [[0, 3], [3, 6]], 2, tmp_path / "cut", port=3)
    run_local(old, timeout=300)
    state = logical.gather(old, 2)
    logical.save(state, str(tmp_path / "logical"))
    back = logical.load(str(tmp_path / "logical"))
    assert back["t"] == state["t"] and set(back["params"]) == set(state["params"])
    # (a) same widths, pieces layout: bitwise continuation
    new = spec(2, [1, 2], [[0, 3], [3, 6]], 4, tmp_path / "cut", shard="pieces", resume=True,
               port=6)
    logical.scatter(back, new)
    resumed = run_local(new, timeout=300)
    with open(full) as f:
        want = {(r["step"], r["mb"]): r["loss_hex"] for r in _json.load(f)["losses"]}
    with open(resumed) as f:
        got = {(r["step"], r["mb"]): r["loss_hex"] for r in _json.load(f)["losses"]}
    later = {k: v for k, v in want.items() if k[0] >= 2}
    assert later and all(got.get(k) == v for k, v in later.items())
    # (b) another cut, widths and shard mode: the waves hold the same state
    other = spec(3, [2, 1, 1], [[0, 2], [2, 4], [4, 6]], 4, tmp_path / "other", shard="pieces")
    logical.scatter(back, other)
    again = logical.gather(other, 2)
    for key in ("params", "exp_avg", "exp_avg_sq"):
        assert set(again[key]) == set(back[key])
        for n, t in back[key].items():
            assert torch.equal(again[key][n], t), (key, n)
    # a corrupted chunk is refused
    p = tmp_path / "logical" / "params.safetensors"
    b = bytearray(p.read_bytes())
    b[-1] ^= 1
    p.write_bytes(bytes(b))
    with pytest.raises(ValueError):
        logical.load(str(tmp_path / "logical"))


@pytest.mark.parametrize("kind", ["lora", "moe"])
def test_logical_checkpoint_pieces_with_frozen_and_replicated_tensors(tmp_path, kind):
    """A LoRA model (frozen base held whole by every pieces replica, adapters
    replicated) and an MoE model (fp32 router replicated, experts sharded):
    ZeRO-1 waves re-laid as pieces and gathered back give the same logical
    state exactly, and the pieces run resumed from them continues the
    uninterrupted run bit for bit."""
    import json as _json
    import os as _os

    from elysium_wan_b200.fault_tolerance import logical
    from elysium_wan_b200.launch.local import run_local
    from elysium_wan_b200.models.config import make_config
    from elysium_wan_b200.runtime.spec import JobSpec

    llama = dict(norm="rmsnorm", mlp="swiglu", pos="rope", bias=False, n_kv_head=2)
    extra = (dict(lora_rank=8, lora_targets="attn_mlp") if kind == "lora" else
             dict(moe_experts=4, moe_top_k=2, moe_d_ff=64, moe_select="score_bias",
                  moe_bias_rate=0.01))
    cfg = make_config("toy", n_layer=4, vocab_size=97, d_model=64, n_head=4, seq_len=16,
                      **llama, **extra)
    base = 38000 + _os.getpid() % 300 * 11 + (5 if kind == "moe" else 0)

    def spec(widths, steps, out, shard="zero1", resume=False, port=0):
        return JobSpec(model=cfg, stages=2, stage_widths=widths, partition=[[0, 3], [3, 6]],
                       shard=shard, microbatches=4, mb_size=2, steps=steps, out_dir=str(out),
                       tag="run", ckpt_every=1, resume=resume, port_base=base + port,
                       backend="gloo").finalize()

    full = run_local(spec([1, 2], 3, tmp_path / "full"), timeout=300)
    old = spec([1, 2], 2, tmp_path / "cut", port=1)
    run_local(old, timeout=300)
    state = logical.gather(old, 2)
    new = spec([1, 2], 3, tmp_path / "cut", shard="pieces", resume=True, port=2)
    logical.scatter(state, new)
    again = logical.gather(new, 2)
    for key in ("params", "exp_avg", "exp_avg_sq"):
        assert set(again[key]) == set(state[key])
        for n, t in state[key].items():
            assert torch.equal(again[key][n], t), (key, n)
    resumed = run_local(new, timeout=300)
    with open(full) as f:
        want = {(r["step"], r["mb"]): r["loss_hex"] for r in _json.load(f)["losses"]}
    with open(resumed) as f:
        got = {(r["step"], r["mb"]): r["loss_hex"] for r in _json.load(f)["losses"]}
    later = {k: v for k, v in want.items() if k[0] >= 2}
    assert later and all(got.get(k) == v for k, v in later.items()), (later, got)


def test_waves_commit_off_the_step_and_a_failed_commit_fails_the_run(tmp_path, monkeypatch,
                                                                     capsys):
    """The stage's wave writer returns at once while the commit (write, fsync,
    hash, rename) runs on its thread; the wave is announced only once it is
    committed; a commit that fails is raised by the next wait, so the run
    fails with it."""
    import threading

    from elysium_wan_b200.runtime.stage_main import WaveWriter

    spec = _spec(tmp_path)
    release = threading.Event()
    real = ckpt._sha256

    def held(path):
        assert release.wait(30)
        return real(path)

    monkeypatch.setattr(ckpt, "_sha256", held)
    w = WaveWriter(spec, 0, 0)
    state = {"step": 2, "params": torch.arange(4.0)}
    w.submit(2, state)
    assert ckpt.list_waves(spec.out_dir, "t", 0, 0) == []  # still hashing
    assert "WT_WAVE" not in capsys.readouterr().out
    release.set()
    w.wait()
    assert ckpt.list_waves(spec.out_dir, "t", 0, 0) == [2]
    assert "WT_WAVE" in capsys.readouterr().out

    def broken(*a, **k):
        raise OSError(28, "No space left on device")

    monkeypatch.setattr(ckpt, "commit_wave", broken)
    w.submit(4, state)
    with pytest.raises(RuntimeError, match="wave commit failed"):
        w.wait()
    w.wait()  # the error is reported once


def test_engine_state_is_a_copy():
    """A wave is written while the next step runs: every tensor of the
    engine's state (parameters, moments) is a copy, also on the CPU where
    `.cpu()` would alias."""
    from elysium_wan_b200.runtime.engine import StageEngine

    cfg = make_config("toy", n_layer=2, vocab_size=97, d_model=64, n_head=4, seq_len=16)
    spec = JobSpec(model=cfg, stages=1, microbatches=2, mb_size=2).finalize()
    eng = StageEngine(spec, 0, 0, None, "cpu")
    sd = eng.state_dict()
    assert sd["params"].data_ptr() != eng.store.master.data_ptr()
    assert sd["opt"]["m"].data_ptr() != eng.opt.m.data_ptr()
    eng.opt.m.add_(1.0)
    assert float(sd["opt"]["m"].abs().sum()) == 0.0
