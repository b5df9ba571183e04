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
