"""The TCP data plane: native codecs, frames, the identity handshake, the
AEAD record layer, and a pipeline run over sealed TCP that is bitwise equal
to the oracle.

Would fail if: a codec changed a bit, the frame header or fragment
reassembly were wrong, the handshake accepted a forged or untrusted peer, a
tampered, replayed or reordered record were accepted, or the TCP plane
delivered a different tensor than the NCCL/gloo plane.
"""

import os
import socket
import threading

import pytest
import torch

from elysium_wan_b200 import codec
from elysium_wan_b200.transport import framing, identity, secure


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16, torch.int64,
                                   torch.float8_e4m3fn])
def test_planes_roundtrip(dtype):
    torch.manual_seed(0)
    if dtype == torch.int64:
        t = torch.randint(-1000, 1000, (3000, 70))
    else:
        t = (torch.randn(3000, 700) * 5).to(dtype)  # > 1 MiB planes: the threaded stream
    p, shape = codec.planes_encode(t)
    back = codec.planes_decode(p, shape)
    assert back.dtype == dtype and torch.equal(back.view(torch.uint8), t.view(torch.uint8))


def test_planes_streams_are_standard_zlib():
    import struct
    import zlib

    t = torch.randn(4096, 512).to(torch.bfloat16)
    p, _ = codec.planes_encode(t)
    did, nplanes, n = struct.unpack_from("<BBQ", p, 0)
    sizes = struct.unpack_from(f"<{nplanes}I", p, 10)
    off = 10 + 4 * nplanes
    hi = zlib.decompress(p[off:off + sizes[0]])
    assert did == 1 and len(hi) == n
    assert hi == bytes((t.view(torch.int16).numpy().view("uint16") >> 8).astype("uint8"))


def test_fp8_and_f32_planes_and_pair():
    x = torch.randn(777, 33).to(torch.float8_e4m3fn).float()
    p, s = codec.fp8_planes_encode(x)
    assert torch.equal(codec.fp8_planes_decode(p, s), x)
    with pytest.raises(ValueError):
        codec.fp8_planes_encode(torch.tensor([0.1234567]))
    y = torch.randn(1000, 1000)
    p, s = codec.f32_planes_encode(y)
    assert torch.equal(codec.f32_planes_decode(p, s), y)
    q = torch.randn(64, 256).to(torch.float8_e4m3fn)
    sc = torch.rand(64, 2)
    p, s = codec.e4m3_b128_encode(q, sc)
    q2, s2 = codec.e4m3_b128_decode(p, s)
    assert torch.equal(q2.view(torch.uint8), q.view(torch.uint8)) and torch.equal(s2, sc)


def test_frames_and_fragments_over_a_socketpair():
    a, b = socket.socketpair()
    t = torch.randn(300, 500)
    cid, payload, shape = framing.encode_tensor(t, "planes")
    frags = framing.fragments(payload, 3)
    th = threading.Thread(target=lambda: [framing.send_frame(a, framing.FWD, 7, 3, part, chunk=1,
                                                             codec_id=cid, shape=shape,
                                                             frag_idx=i, frag_cnt=len(frags))
                                          for i, part in enumerate(frags)])
    th.start()
    re = framing.Reassembler()
    whole = None
    while whole is None:
        whole = re.push(framing.recv_frame(b))
    th.join()
    assert (whole.type, whole.step, whole.mb, whole.chunk) == (framing.FWD, 7, 3, 1)
    assert torch.equal(whole.tensor(), t)
    a.sendall(b"\x00\x00" + b"\x00" * 30)
    with pytest.raises(framing.FrameError):
        framing.recv_frame(b)
    a.close()
    b.close()


def _pair(tmp_path, trusted=None, expect=None, cipher="chacha20-poly1305", rekey=1 << 24):
    ka = identity.load_or_create_key(str(tmp_path / "a.key"))
    kb = identity.load_or_create_key(str(tmp_path / "b.key"))
    a, b = socket.socketpair()
    out = {}

    def side(name, sock, key, role, **kw):
        try:
            out[name] = identity.authenticate(sock, key, role, **kw)
        except Exception as e:  # noqa: BLE001
            out[name] = e

    ta = threading.Thread(target=side, args=("a", a, ka, "dialer"),
                          kwargs=dict(trusted_peers=trusted))
    tb = threading.Thread(target=side, args=("b", b, kb, "listener"),
                          kwargs=dict(expect_peer=expect))
    ta.start(), tb.start()
    ta.join(10), tb.join(10)
    return a, b, out, ka, kb


def test_handshake_and_sealed_records(tmp_path):
    a, b, out, ka, kb = _pair(tmp_path, rekey=4)
    assert out["a"].peer == identity.peer_id(identity._raw(kb.public_key()))
    assert out["b"].peer == identity.peer_id(identity._raw(ka.public_key()))
    sa = secure.SecureSocket(a, out["a"], rekey_records=4)
    sb = secure.SecureSocket(b, out["b"], rekey_records=4)
    msg = os.urandom(3 * secure.MAX_RECORD + 123)
    th = threading.Thread(target=lambda: [sa.sendall(msg[i:i + 70000])
                                          for i in range(0, len(msg), 70000)])
    th.start()
    got = bytearray()
    while len(got) < len(msg):
        got += sb.recv(1 << 16)
    th.join()
    assert bytes(got) == msg  # crosses several rekeys
    # a flipped byte fails the tag and the stream stays failed
    hdr = secure._LEN.pack(16 + 5)
    a.sendall(hdr + b"\x01" * 21)
    with pytest.raises(ConnectionError):
        sb.recv(10)
    with pytest.raises(ConnectionError):
        sb.recv(10)


def test_handshake_refuses_untrusted_and_wrong_roles(tmp_path):
    _, _, out, _, _ = _pair(tmp_path, trusted=["0" * 32])
    assert isinstance(out["a"], identity.HandshakeError)
    _, _, out, _, _ = _pair(tmp_path, expect="f" * 32)
    assert isinstance(out["b"], identity.HandshakeError)
    ka = identity.load_or_create_key(str(tmp_path / "a.key"))
    a, b = socket.socketpair()
    res = {}
    t = threading.Thread(target=lambda: res.setdefault("x", _try(a, ka, "dialer")))
    t.start()
    r2 = _try(b, ka, "dialer")  # both claim the dialer role
    t.join(10)
    assert isinstance(r2, identity.HandshakeError) or isinstance(res["x"], identity.HandshakeError)


def _try(sock, key, role):
    try:
        return identity.authenticate(sock, key, role)
    except Exception as e:  # noqa: BLE001
        return e


def test_pipeline_over_sealed_tcp_is_bitwise(tmp_path, monkeypatch):
    from elysium_wan_b200.launch.local import run_and_compare
    from elysium_wan_b200.models.config import make_config
    from elysium_wan_b200.runtime.spec import JobSpec

    monkeypatch.setenv("ELYSIUM_PEER_KEY", str(tmp_path / "peer.key"))
    cfg = make_config("toy", n_layer=4, vocab_size=97, d_model=128, n_head=4, seq_len=16,
                      boundary_dtype="bf16")
    port = 31000 + (os.getpid() % 200) * 10
    spec = JobSpec(model=cfg, stages=2, stage_widths=[1, 2], microbatches=4, mb_size=2, steps=2,
                   out_dir=str(tmp_path), port_base=port, backend="tcp", wire_codec="planes",
                   p2p_streams=2)
    r = run_and_compare(spec, timeout=300)
    assert r["ok"], r
    assert r["compared"] == 8


def test_socket_tuning_plan_and_apply():
    from elysium_wan_b200.transport import tuning

    caps = {"wmem_max": 64 << 20, "rmem_max": 8 << 20, "tcp_wmem": 4 << 20, "tcp_rmem": 6 << 20}
    p = tuning.plan(32 << 20, caps)
    assert p == {"sndbuf": 32 << 20, "rcvbuf": None}  # rcvbuf hard cap too low: autotuning kept
    assert tuning.plan(2 << 20, caps) == {"sndbuf": None, "rcvbuf": None}  # below the ceilings
    s = socket.socket()
    rep = tuning.tune(s)  # never raises; reports what holds
    assert set(rep) == {"cc", "sndbuf", "rcvbuf", "pace"}
    s.close()


def test_safe_object_codec_roundtrip_and_no_pickle():
    import math
    import pickle

    import torch

    from elysium_wan_b200.transport import serial

    obj = {"step": 3, "params": torch.randn(10), "names": ["a", "b"],
           "opt": {"t": 2, "m": torch.zeros(3, dtype=torch.bfloat16)},
           "losses": {0: 1.5, 1: float("inf")}, "rng": torch.get_rng_state(),
           "tup": (1, "x", None), "b": b"\x00\x01", "nan": float("nan"), "e": torch.empty(0, 4),
           "f8": torch.randn(8).to(torch.float8_e4m3fn)}
    o = serial.loads(serial.dumps(obj))
    assert torch.equal(o["params"], obj["params"]) and o["names"] == ["a", "b"]
    assert o["opt"]["m"].dtype == torch.bfloat16 and o["losses"] == {0: 1.5, 1: float("inf")}
    assert torch.equal(o["rng"], obj["rng"]) and o["tup"] == (1, "x", None) and o["b"] == b"\x00\x01"
    assert math.isnan(o["nan"]) and o["e"].shape == (0, 4)
    assert torch.equal(o["f8"].view(torch.uint8), obj["f8"].view(torch.uint8))
    # the same bytes for the same object (exact, deterministic)
    assert serial.dumps(obj["opt"]) == serial.dumps(obj["opt"])
    # a pickle is refused, not executed
    with pytest.raises(ValueError):
        serial.loads(pickle.dumps({"x": 1}))
    with pytest.raises(TypeError):
        serial.dumps({"f": object()})


class _TearingProxy:
    """A TCP relay that forwards each direction in random 1..2048-byte pieces
    with random pauses and a few 50 ms stalls: torn reads and stalls on the
    data plane, never a changed or lost byte."""

    def __init__(self, target_port: int, seed: int = 0):
        import random

        self.target = target_port
        self.rng = random.Random(seed)
        self.lsock = socket.socket()
        self.lsock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        self.lsock.bind(("127.0.0.1", 0))
        self.lsock.listen(16)
        self.port = self.lsock.getsockname()[1]
        self.stop = threading.Event()
        self.forwarded = 0
        threading.Thread(target=self._accept, daemon=True).start()

    def _accept(self):
        import time as _t

        while not self.stop.is_set():
            try:
                c, _ = self.lsock.accept()
            except OSError:
                return
            for _ in range(200):  # the target may not listen yet
                try:
                    u = socket.create_connection(("127.0.0.1", self.target))
                    break
                except OSError:
                    _t.sleep(0.05)
            else:
                c.close()
                continue
            for a, b in ((c, u), (u, c)):
                threading.Thread(target=self._pump, args=(a, b), daemon=True).start()

    def _pump(self, src, dst):
        import time as _t

        try:
            while True:
                data = src.recv(65536)
                if not data:
                    break
                i = 0
                while i < len(data):
                    n = self.rng.randint(1, 2048)
                    dst.sendall(data[i:i + n])
                    self.forwarded += len(data[i:i + n])
                    i += n
                    r = self.rng.random()
                    if r < 0.002:
                        _t.sleep(0.05)
                    elif r < 0.05:
                        _t.sleep(0.0005)
            dst.shutdown(socket.SHUT_WR)
        except OSError:
            pass

    def close(self):
        self.stop.set()
        self.lsock.close()


def test_pipeline_through_a_tearing_proxy_is_bitwise(tmp_path, monkeypatch):
    """Stage 0 reaches stage 1 only through a relay that tears every write
    into random pieces and stalls at random: frames, fragments, sealed records
    and the pipeline's losses stay exactly the oracle's."""
    from elysium_wan_b200.launch.local import run_and_compare
    from elysium_wan_b200.models.config import make_config
    from elysium_wan_b200.runtime.spec import JobSpec

    monkeypatch.setenv("ELYSIUM_PEER_KEY", str(tmp_path / "peer.key"))
    cfg = make_config("toy", n_layer=4, vocab_size=97, d_model=128, n_head=4, seq_len=16,
                      boundary_dtype="bf16")
    base = 32000 + (os.getpid() % 200) * 10
    s1_port = base + 1
    proxy = _TearingProxy(s1_port, seed=7)
    try:
        spec = JobSpec(model=cfg, stages=2, microbatches=4, mb_size=2, steps=2,
                       out_dir=str(tmp_path), port_base=base + 5, backend="tcp",
                       wire_codec="planes", p2p_streams=2,
                       endpoints=[[["127.0.0.1", base, base]],
                                  [["127.0.0.1", proxy.port, s1_port]]])
        r = run_and_compare(spec, timeout=300)
    finally:
        proxy.close()
    assert r["ok"], r
    assert r["compared"] == 8
    assert proxy.forwarded > 0


def test_late_receive_fills_with_deferred_w_bitwise(tmp_path, monkeypatch):
    """A slow hop makes receives late; the stage runs deferred W tasks while it
    waits (the order's W sequence kept) and every loss still equals the
    oracle bit for bit."""
    import glob
    import json as _json

    from elysium_wan_b200.launch.local import run_and_compare
    from elysium_wan_b200.models.config import make_config
    from elysium_wan_b200.runtime.spec import JobSpec

    monkeypatch.setenv("ELYSIUM_PEER_KEY", str(tmp_path / "peer.key"))
    cfg = make_config("toy", n_layer=6, vocab_size=97, d_model=128, n_head=4, seq_len=16,
                      boundary_dtype="bf16")
    port = 33000 + (os.getpid() % 200) * 10
    spec = JobSpec(model=cfg, stages=3, microbatches=6, mb_size=2, steps=2,
                   out_dir=str(tmp_path), port_base=port, backend="tcp", wire_codec="planes",
                   links=[{"latency_ms": 40.0, "bw_mbps": 0.0}] * 3)
    r = run_and_compare(spec, timeout=300)
    assert r["ok"], r
    assert r["compared"] == 12
    filled = 0
    for path in glob.glob(os.path.join(str(tmp_path), "*_r*p*.log")):
        for line in open(path):
            if line.startswith("WT_WFILL"):
                filled += _json.loads(line.split(" ", 1)[1])["tasks"]
    assert filled > 0


def _bucket_worker(path, n, nbytes, q):
    import time as _t

    from elysium_wan_b200.transport.pacer import HostBucket

    b = HostBucket(100.0, path, burst_ms=0.0)
    t0 = _t.monotonic()
    end = 0.0
    for _ in range(n):
        end = b.reserve(nbytes)
        d = end - _t.monotonic()
        if d > 0:
            _t.sleep(d)
    q.put((t0, _t.monotonic()))


def test_host_bucket_is_shared_by_processes(tmp_path):
    """Two processes pacing through one 100 Mbit/s bucket take twice as long as
    one: 2 x 10 frames of 125 kB at 10 ms each need >= 0.2 s together."""
    import multiprocessing as mp
    import time as _t

    path = str(tmp_path / "nic.bucket")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_bucket_worker, args=(path, 10, 125_000, q)) for _ in range(2)]
    for p in ps:
        p.start()
    spans = [q.get(timeout=60) for _ in ps]
    for p in ps:
        p.join(30)
    start, end = min(s for s, _ in spans), max(e for _, e in spans)
    assert end - start >= 0.19
    # a bucket at another rate refuses the same file
    from elysium_wan_b200.transport.pacer import HostBucket

    with pytest.raises(ValueError):
        HostBucket(50.0, path)
    _t.sleep(0)


def test_shared_budgets_pace_but_never_change_bits(tmp_path):
    """A wide next stage: stage 0 sends to two replicas through one shared
    egress budget (its NIC) and an uplink budget; losses stay bitwise."""
    from elysium_wan_b200.launch.local import run_and_compare
    from elysium_wan_b200.models.config import make_config
    from elysium_wan_b200.runtime.spec import JobSpec

    cfg = make_config("toy", n_layer=4, vocab_size=97, d_model=128, n_head=4, seq_len=16)
    port = 34000 + (os.getpid() % 200) * 10
    link = {"latency_ms": 2.0, "bw_mbps": 400.0, "egress_key": "node0", "egress_mbps": 200.0,
            "uplink_key": "r0>r1", "uplink_mbps": 300.0}
    spec = JobSpec(model=cfg, stages=2, stage_widths=[1, 2], microbatches=4, mb_size=2, steps=2,
                   out_dir=str(tmp_path), port_base=port, backend="gloo", links=[link, {}])
    r = run_and_compare(spec, timeout=300)
    assert r["ok"], r
    assert os.listdir(os.path.join(str(tmp_path), ".pacers"))


def test_emulated_links_carry_shared_budgets():
    from elysium_wan_b200.resources.links import Emulation
    from elysium_wan_b200.scheduler.placement import emulated_links

    class N:
        def __init__(self, i, region):
            self.node_id, self.region = f"n{i}", region

    prof = {"inter": {"rtt_ms": 40.0, "mbps": 500.0}, "nic_mbps": 1000.0, "shared": True}
    groups = [[N(0, "a")], [N(1, "b")]]
    ems = {"n0": Emulation.from_profile("a", prof), "n1": Emulation.from_profile("b", prof)}
    links = emulated_links(groups, ems)
    assert links[0]["egress_key"] == "n0" and links[0]["egress_mbps"] == 1000.0
    assert links[0]["ingress_key"] == "n1" and links[0]["uplink_key"] == "a>b"
    assert links[0]["uplink_mbps"] == 500.0 and links[0]["latency_ms"] == 20.0
    off = {"n0": Emulation.from_profile("a", {"inter": prof["inter"]}),
           "n1": Emulation.from_profile("b", {"inter": prof["inter"]})}
    assert emulated_links(groups, off)[0]["egress_key"] == ""
    # a wide stage whose replicas sit in two regions: its mesh links are shaped too
    from elysium_wan_b200.scheduler.placement import emulated_mesh_links

    wide = [[N(0, "a")], [N(3, "a"), N(2, "b")]]
    ems["n2"], ems["n3"] = Emulation.from_profile("b", prof), Emulation.from_profile("a", prof)
    mesh = emulated_mesh_links(wide, ems)
    assert mesh[0] == {} and set(mesh[1]) == {"0>1", "1>0"}
    assert mesh[1]["0>1"]["uplink_key"] == "a>b" and mesh[1]["1>0"]["uplink_key"] == "b>a"
    assert mesh[1]["0>1"]["latency_ms"] == 20.0


def test_multi_flow_fragments_reassemble_across_flows(tmp_path, monkeypatch):
    """Boundaries large enough to be cut into one fragment per flow (4 flows,
    256 kB fp32 boundaries): each frame's fragments arrive on different
    sockets and must reassemble into one frame; losses stay bitwise."""
    from elysium_wan_b200.launch.local import run_and_compare
    from elysium_wan_b200.models.config import make_config
    from elysium_wan_b200.runtime.spec import JobSpec

    monkeypatch.setenv("ELYSIUM_PEER_KEY", str(tmp_path / "peer.key"))
    cfg = make_config("toy", n_layer=2, vocab_size=97, d_model=512, n_head=4, seq_len=64)
    port = 35000 + (os.getpid() % 200) * 10
    spec = JobSpec(model=cfg, stages=2, microbatches=2, mb_size=2, steps=2, out_dir=str(tmp_path),
                   port_base=port, backend="tcp", wire_codec="planes", p2p_streams=4)
    r = run_and_compare(spec, timeout=180)
    assert r["ok"], r
    assert r["compared"] == 4


def test_adaptive_fragments_shrink_and_stay_bitwise(tmp_path, monkeypatch):
    """With a tiny send budget every fragment is 'too slow', so the sender
    halves its fragment size down to the floor: a 256 kB boundary then goes
    as many small fragments round-robin over 2 flows, and the losses are
    still bitwise equal to the oracle."""
    from elysium_wan_b200.launch.local import run_and_compare
    from elysium_wan_b200.models.config import make_config
    from elysium_wan_b200.runtime.spec import JobSpec

    monkeypatch.setenv("ELYSIUM_PEER_KEY", str(tmp_path / "peer.key"))
    cfg = make_config("toy", n_layer=2, vocab_size=97, d_model=512, n_head=4, seq_len=64)
    port = 36000 + (os.getpid() % 200) * 10
    spec = JobSpec(model=cfg, stages=2, microbatches=4, mb_size=2, steps=2, out_dir=str(tmp_path),
                   port_base=port, backend="tcp", wire_codec="planes", p2p_streams=2,
                   adapt_budget_ms=1e-6, frag_min_bytes=16384)
    r = run_and_compare(spec, timeout=240)
    assert r["ok"], r
    assert r["compared"] == 8


def test_fragment_size_adaptation_rule():
    from types import SimpleNamespace

    from elysium_wan_b200.transport.tcp import _Link

    link = _Link.__new__(_Link)
    link.comm = SimpleNamespace(spec=SimpleNamespace(adapt_budget_ms=5.0, frag_min_bytes=4096))
    link.frag_size, link.clean = 0, 0
    link._adapt(0.010, 1 << 20, 1 << 20)  # 10 ms > 5 ms: halve
    assert link.frag_size == 1 << 19
    for _ in range(20):
        link._adapt(0.010, link.frag_size, 1 << 20)
    assert link.frag_size == 4096  # the floor
    for _ in range(8):
        link._adapt(0.0001, link.frag_size, 1 << 20)  # well under a quarter: double after 8
    assert link.frag_size == 8192


@pytest.mark.parametrize("boundary", ["fp8_e4m3_b128", "fp8_e5m2_b128"])
def test_fp8_boundaries_over_tcp_wide_shaped_multiflow(tmp_path, monkeypatch, boundary):
    """The fp8 boundary pair (codes + 1x128 scales) as one frame over the
    sealed TCP plane: 3 stages with a wide middle stage, 3 flows per hop,
    adaptive fragments, a shaped link with a shared egress budget; bitwise."""
    from elysium_wan_b200.launch.local import run_and_compare
    from elysium_wan_b200.models.config import make_config
    from elysium_wan_b200.runtime.spec import JobSpec

    monkeypatch.setenv("ELYSIUM_PEER_KEY", str(tmp_path / "peer.key"))
    cfg = make_config("toy", n_layer=4, vocab_size=97, d_model=512, n_head=4, seq_len=64,
                      boundary_dtype=boundary)
    link = {"latency_ms": 3.0, "bw_mbps": 800.0, "egress_key": "n0", "egress_mbps": 600.0}
    port = 38000 + (os.getpid() % 200) * 10 + len(boundary)
    spec = JobSpec(model=cfg, stages=3, stage_widths=[1, 2, 1], microbatches=6, mb_size=2, steps=2,
                   out_dir=str(tmp_path), port_base=port, backend="tcp", wire_codec="planes",
                   p2p_streams=3, adapt_budget_ms=0.5, frag_min_bytes=16384, links=[link, link, {}])
    r = run_and_compare(spec, timeout=300)
    assert r["ok"], r
    assert r["compared"] == 12


# ------------------------------------------------------- transient send refusals
class _FlakyKernel:
    """A fake at the kernel boundary: each send attempt takes the next entry
    of a script (an errno: refused, nothing written; ("cut", n): write at
    most n bytes; None: pass through) and hands what it lets through to a
    real socketpair end, so the receiver reads the bytes really written."""

    def __init__(self, sock, script):
        self.sock, self.script, self.attempts = sock, list(script), 0

    def send(self, data):
        self.attempts += 1
        act = self.script.pop(0) if self.script else None
        if isinstance(act, int):
            raise OSError(act, os.strerror(act))
        if isinstance(act, tuple):
            data = data[:act[1]]
        return self.sock.send(data)


def _drain(sock, n):
    out = bytearray()
    while len(out) < n:
        b = sock.recv(n - len(out))
        if not b:
            break
        out += b
    return bytes(out)


def test_send_all_retries_transient_refusals_from_the_same_offset():
    import errno

    from elysium_wan_b200.transport.sendall import send_all

    a, b = socket.socketpair()
    data = os.urandom(200_000)
    k = _FlakyKernel(a, [errno.ENOBUFS, ("cut", 1000), errno.EAGAIN, errno.ENOBUFS, ("cut", 7),
                         errno.EWOULDBLOCK])
    got = []
    t = threading.Thread(target=lambda: got.append(_drain(b, len(data))))
    t.start()
    send_all(k, data)
    t.join(10)
    assert got and got[0] == data
    assert k.attempts >= 7  # four refusals, two cut sends, then the rest
    a.close()
    b.close()


def test_send_all_raises_other_errors_at_once_and_gives_up_after_the_budget(monkeypatch):
    import errno
    import time

    from elysium_wan_b200.transport import sendall

    a, b = socket.socketpair()
    k = _FlakyKernel(a, [errno.ECONNRESET, None])
    with pytest.raises(ConnectionResetError):
        sendall.send_all(k, b"x" * 10)
    assert k.attempts == 1  # not retried
    monkeypatch.setattr(sendall, "RETRY_BUDGET_S", 0.05)
    k = _FlakyKernel(a, [errno.ENOBUFS] * 10_000)
    t0 = time.monotonic()
    with pytest.raises(OSError) as e:
        sendall.send_all(k, b"x" * 10)
    assert e.value.errno == errno.ENOBUFS and 0.05 <= time.monotonic() - t0 < 2.0
    with pytest.raises(ValueError):
        sendall.enobufs_every("1")
    assert sendall.enobufs_every("") == 0 and sendall.enobufs_every("3") == 3
    a.close()
    b.close()


def test_native_frame_writer_waits_out_a_full_socket_buffer():
    """A non-blocking sender whose buffer fills answers EAGAIN; the native
    frame writer offers the rest again until the reader drains it, and the
    frame arrives whole."""
    import time

    a, b = socket.socketpair()
    a.setsockopt(socket.SOL_SOCKET, socket.SO_SNDBUF, 64 << 10)
    a.setblocking(False)
    payload = os.urandom(8 << 20)
    got = []

    def reader():
        time.sleep(0.3)  # the writer meets a full buffer first
        got.append(framing.recv_frame(b))

    t = threading.Thread(target=reader)
    t.start()
    n = codec.wire().send_frame(a.fileno(), framing.FWD, framing.RAW_F32, 3, 1, 0,
                                [len(payload) // 4], payload, 0, 1)
    t.join(30)
    assert n > len(payload) and got
    assert got[0].step == 3 and got[0].mb == 1 and bytes(got[0].payload) == payload
    a.close()
    b.close()


def test_pipeline_over_sealed_tcp_with_refused_sends_is_bitwise(tmp_path, monkeypatch):
    """WANTRAIN_TEST_ENOBUFS=3: every third send attempt of every sealed
    socket is refused with ENOBUFS; the pipeline still equals the oracle."""
    from elysium_wan_b200.launch.local import run_and_compare
    from elysium_wan_b200.models.config import make_config
    from elysium_wan_b200.runtime.spec import JobSpec

    monkeypatch.setenv("ELYSIUM_PEER_KEY", str(tmp_path / "peer.key"))
    monkeypatch.setenv("WANTRAIN_TEST_ENOBUFS", "3")
    cfg = make_config("toy", n_layer=4, vocab_size=97, d_model=128, n_head=4, seq_len=16,
                      boundary_dtype="bf16")
    port = 31500 + (os.getpid() % 200) * 10
    spec = JobSpec(model=cfg, stages=2, stage_widths=[1, 2], microbatches=4, mb_size=2, steps=2,
                   out_dir=str(tmp_path), port_base=port, backend="tcp", wire_codec="planes",
                   p2p_streams=2)
    r = run_and_compare(spec, timeout=300)
    assert r["ok"], r
    assert r["compared"] == 8


@pytest.mark.parametrize("case", ["tied_zero1_1_2_1", "moe_pieces_1_2"])
def test_wide_stage_exchange_and_tied_relay_cross_the_sealed_plane(tmp_path, monkeypatch, case):
    """On the TCP data plane a wide stage's ZeRO-1 / pieces exchange (the
    partials' scatter, the shards' gather, MoE expert counts) runs over the
    sealed links among its replicas, and a tied table's relay over a sealed
    link between the first and last stages; the losses equal the oracle."""
    import glob

    from elysium_wan_b200.launch.local import run_and_compare
    from elysium_wan_b200.models.config import make_config
    from elysium_wan_b200.runtime.spec import JobSpec

    monkeypatch.setenv("ELYSIUM_PEER_KEY", str(tmp_path / "peer.key"))
    if case == "tied_zero1_1_2_1":
        cfg = make_config("toy", n_layer=4, vocab_size=97, d_model=64, n_head=4, seq_len=16,
                          tie_embeddings=True)
        kw = dict(stages=3, stage_widths=[1, 2, 1])
    else:
        cfg = make_config("toy", n_layer=4, vocab_size=97, d_model=64, n_head=4, seq_len=16,
                          norm="rmsnorm", mlp="swiglu", pos="rope", bias=False, moe_experts=4,
                          moe_top_k=2, moe_d_ff=64, moe_select="score_bias", moe_bias_rate=0.01)
        shaped = {"latency_ms": 2.0, "bw_mbps": 400.0}
        kw = dict(stages=2, stage_widths=[1, 2], shard="pieces",
                  mesh_links=[{}, {"0>1": shaped, "1>0": shaped}])  # the mesh links shaped
    port = 32500 + 40 * (case != "tied_zero1_1_2_1") + (os.getpid() % 200) * 7
    spec = JobSpec(model=cfg, microbatches=4, mb_size=2, steps=3, out_dir=str(tmp_path),
                   port_base=port, backend="tcp", wire_codec="planes", **kw)
    r = run_and_compare(spec, timeout=300)
    assert r["ok"] and r["compared"] == 12, r
    logs = {os.path.basename(p): open(p).read() for p in glob.glob(str(tmp_path / "*_r*p*.log"))}
    wide = [t for n, t in logs.items() if "_r1p" in n]
    assert len(wide) == 2 and all("WT_MESH" in t for t in wide), list(logs)
    # per-link send statistics ride in each step's telemetry
    import json as _json

    telem = [_json.loads(line.split(" ", 1)[1]) for line in wide[0].splitlines()
             if line.startswith("WT_TELEM ")]
    mesh = [h for k, h in telem[-1]["hops"].items() if k.startswith("mesh")]
    assert len(mesh) == 1 and mesh[0]["frames"] > 0 and mesh[0]["busy_ms"] >= 0, telem[-1]
    assert any(k.startswith("prev") for k in telem[-1]["hops"]), telem[-1]
    if case == "tied_zero1_1_2_1":
        ends = [t for n, t in logs.items() if "_r0p0" in n or "_r2p0" in n]
        assert len(ends) == 2 and all("WT_TIED_LINK" in t for t in ends)


def _shared_spec(**kw):
    from elysium_wan_b200.models.config import make_config
    from elysium_wan_b200.runtime.spec import JobSpec

    cfg = make_config("toy", n_layer=4, vocab_size=97, d_model=64, n_head=4, seq_len=16)
    base = dict(model=cfg, stages=2, stage_widths=[1, 2], microbatches=4, mb_size=2, steps=2,
                pacing="shared", peer_egress_mbps=[[400.0], [300.0, 300.0]],
                peer_ingress_mbps=[[500.0], [200.0, 250.0]], sites=[["us"], ["us", "eu"]],
                uplink_mbps={"us->eu": 100.0, "eu->us": 120.0})
    base.update(kw)
    return JobSpec(**base)


def test_shared_pacing_fields_are_checked_and_name_each_connections_budgets():
    """The reference's shared-pacing spec fields: every slot's NIC rates and
    site, and an uplink for both directions of every site pair a connection
    crosses; each connection then draws on its sender's egress, its
    receiver's ingress and, across sites, that direction's uplink."""
    from elysium_wan_b200.transport.pacer import link_buckets, pair_link, reverse_link

    spec = _shared_spec().finalize()
    assert spec.emission_order == ["store", "store"]
    c = pair_link(spec, {"latency_ms": 5.0}, (0, 0), (1, 1))
    assert c["latency_ms"] == 5.0
    assert (c["egress_key"], c["egress_mbps"]) == ("slot0.0", 400.0)
    assert (c["ingress_key"], c["ingress_mbps"]) == ("slot1.1", 250.0)
    assert (c["uplink_key"], c["uplink_mbps"]) == ("us>eu", 100.0)
    same_site = pair_link(spec, {}, (0, 0), (1, 0))
    assert "uplink_key" not in same_site and same_site["ingress_mbps"] == 200.0
    back = pair_link(spec, reverse_link({}), (1, 1), (0, 0))
    assert back["uplink_key"] == "eu>us" and back["uplink_mbps"] == 120.0
    assert len(link_buckets(c, "pacing-test")) == 3
    assert pair_link(_shared_spec(pacing="link").finalize(), {}, (0, 0), (1, 1)) == {}
    for bad in (dict(uplink_mbps={"us->eu": 100.0}),            # eu->us missing
                dict(peer_egress_mbps=[[400.0], [300.0]]),       # not every slot
                dict(peer_ingress_mbps=[[0.0], [1.0, 1.0]]),      # not > 0
                dict(sites=[["us"], ["us", ""]]),
                dict(pacing="fair"),
                dict(emission_order=["store"]),
                dict(piece_bounds=[None, None])):
        with pytest.raises((ValueError, NotImplementedError)):
            _shared_spec(**bad).finalize()


@pytest.mark.parametrize("backend", ["tcp", "gloo"])
def test_pipeline_under_shared_pacing_across_sites_is_bitwise(tmp_path, monkeypatch, backend):
    """A run paced by the spec's shared budgets (two sites, a wide stage whose
    replicas sit on both): the connections open their budgets (on the gloo
    plane one pacer per direction serves a whole neighbour stage, so the
    receiver's budgets apply only toward a one-peer stage), and the losses
    equal the oracle."""
    import glob

    from elysium_wan_b200.launch.local import run_and_compare

    monkeypatch.setenv("ELYSIUM_PEER_KEY", str(tmp_path / "peer.key"))
    port = 33500 + 30 * (backend == "gloo") + (os.getpid() % 200) * 7
    spec = _shared_spec(out_dir=str(tmp_path), port_base=port, backend=backend,
                        wire_codec="planes")
    r = run_and_compare(spec, timeout=300)
    assert r["ok"] and r["compared"] == 8, r
    names = {os.path.basename(p).split("-")[0]
             for p in glob.glob(str(tmp_path / ".pacers" / "*.bucket"))}
    want = {"egress_slot0.0", "egress_slot1.0", "egress_slot1.1", "ingress_slot0.0",
            "uplink_eu>us"}
    if backend == "tcp":
        want |= {"ingress_slot1.0", "ingress_slot1.1", "uplink_us>eu"}
    assert want <= names, names
