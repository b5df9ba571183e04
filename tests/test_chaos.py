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
