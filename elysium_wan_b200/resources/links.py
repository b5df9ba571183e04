"""Link probes: round-trip time and TCP bandwidth between two machines, and
the device-to-device copy rate between two GPUs of one box.

Reference behaviour: src/wantrain/resources/links.py (`serve_echo` :78,
`measure_pair` :351, `classify_duplex` :326, `Emulation` :44). A worker runs
an echo server; the prober measures the median round trip of small
messages, then the rate of upload, download and both at once over `flows`
parallel connections (each tuned like the data plane). Comparing the three
rates classifies the path: full duplex (both directions at once add up),
half duplex (they share one rate), or in between. Over NVLink the transfer
that matters is a peer copy, measured with the CUDA copy engine.

`Emulation` describes experiment regions (round trip and rate between named
regions) for runs that emulate a WAN on one box; placement turns it into the
per-hop shim settings of a spec.
"""

from __future__ import annotations

import socket
import socketserver
import statistics
import struct
import threading
import time
from dataclasses import dataclass, field

from elysium_wan_b200.transport import tuning

_PING, _UP, _DOWN = b"P", b"U", b"D"
_CHUNK = 1 << 20


class _Handler(socketserver.BaseRequestHandler):
    def handle(self):
        s = self.request
        try:
            while True:
                op = s.recv(1)
                if not op:
                    return
                if op == _PING:
                    s.sendall(_PING)
                elif op == _UP:  # the client streams until it closes its side; count and ack
                    (secs,) = struct.unpack("<d", _exact(s, 8))
                    got = 0
                    s.settimeout(secs + 10)
                    while True:
                        b = s.recv(_CHUNK)
                        if not b:
                            break
                        got += len(b)
                    s.sendall(struct.pack("<Q", got))
                    return
                elif op == _DOWN:  # stream to the client for n seconds
                    (secs,) = struct.unpack("<d", _exact(s, 8))
                    buf = bytes(_CHUNK)
                    end = time.monotonic() + secs
                    while time.monotonic() < end:
                        s.sendall(buf)
                    return
                else:
                    return
        except OSError:
            return


class _Server(socketserver.ThreadingTCPServer):
    allow_reuse_address = True
    daemon_threads = True


def _exact(s, n):
    b = b""
    while len(b) < n:
        c = s.recv(n - len(b))
        if not c:
            raise ConnectionError("peer closed")
        b += c
    return b


def serve_echo(host: str = "0.0.0.0", port: int = 0):
    """Start the echo / bandwidth server in a thread; -> (server, port)."""
    srv = _Server((host, port), _Handler)
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    return srv, srv.server_address[1]


def rtt_ms(host: str, port: int, n: int = 20, timeout: float = 5.0) -> float:
    s, _ = tuning.connect(host, port, timeout)
    try:
        ts = []
        for _ in range(n):
            t = time.perf_counter()
            s.sendall(_PING)
            _exact(s, 1)
            ts.append((time.perf_counter() - t) * 1e3)
        return statistics.median(ts)
    finally:
        s.close()


def _up(host, port, secs, out, i, timeout):
    s, _ = tuning.connect(host, port, timeout)
    try:
        s.sendall(_UP + struct.pack("<d", secs))
        buf = bytes(_CHUNK)
        end = time.monotonic() + secs
        while time.monotonic() < end:
            s.sendall(buf)
        s.shutdown(socket.SHUT_WR)
        (got,) = struct.unpack("<Q", _exact(s, 8))
        out[i] = got
    except OSError:
        out[i] = 0
    finally:
        s.close()


def _down(host, port, secs, out, i, timeout):
    s, _ = tuning.connect(host, port, timeout)
    try:
        s.sendall(_DOWN + struct.pack("<d", secs))
        got = 0
        s.settimeout(secs + timeout)
        while True:
            b = s.recv(_CHUNK)
            if not b:
                break
            got += len(b)
        out[i] = got
    except OSError:
        out[i] = 0
    finally:
        s.close()


def _rate(fns, secs) -> float:
    out = [0] * len(fns)
    th = [threading.Thread(target=f, args=(out, i)) for i, f in enumerate(fns)]
    t = time.perf_counter()
    for x in th:
        x.start()
    for x in th:
        x.join()
    dt = max(secs, time.perf_counter() - t)
    return sum(out) * 8 / dt / 1e6


def classify_duplex(up: float, down: float, both: float) -> str:
    """full: both at once carry about up + down; half: about max(up, down)."""
    if up <= 0 or down <= 0 or both <= 0:
        return "unknown"
    if both >= 0.8 * (up + down):
        return "full"
    if both <= 1.2 * max(up, down):
        return "half"
    return "shared"


def measure_pair(host: str, port: int, flows: int = 4, secs: float = 1.0,
                 timeout: float = 5.0, emu: Emulation | None = None,
                 region: str | None = None) -> dict:
    """{rtt_ms, up_mbps, down_mbps, both_mbps, duplex} to an echo server
    (shaped by `emu` toward `region` when an emulation is given)."""
    r = rtt_ms(host, port, timeout=timeout)
    up = _rate([lambda o, i: _up(host, port, secs, o, i, timeout)] * flows, secs)
    down = _rate([lambda o, i: _down(host, port, secs, o, i, timeout)] * flows, secs)
    both = _rate([lambda o, i: _up(host, port, secs, o, i, timeout)] * flows
                 + [lambda o, i: _down(host, port, secs, o, i, timeout)] * flows, secs)
    if emu is not None and emu.enabled:
        r, up = emu.shape(region, r, up)
        _, down = emu.shape(region, r, down)
        _, both = emu.shape(region, r, both)
    return {"rtt_ms": round(r, 3), "up_mbps": round(up, 1), "down_mbps": round(down, 1),
            "both_mbps": round(both, 1), "duplex": classify_duplex(up, down, both),
            "flows": flows}


def peer_copy_gbs(src: int = 0, dst: int = 1, nbytes: int = 1 << 30, iters: int = 5) -> float:
    """GPU src -> GPU dst copy rate (GB/s, CUDA events on the source stream)."""
    import torch

    a = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{src}")
    b = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{dst}")
    b.copy_(a)
    torch.cuda.synchronize(src)
    torch.cuda.synchronize(dst)
    with torch.cuda.device(src):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            b.copy_(a, non_blocking=True)
        e1.record()
        e1.synchronize()
        return nbytes * iters / (e0.elapsed_time(e1) * 1e-3) / 1e9


@dataclass
class Link:
    rtt_ms: float
    mbps: float


@dataclass
class Emulation:
    """Experiment regions: this node's region and the (rtt, rate) to others.

    `links` maps another region to {"rtt_ms", "mbps"}. A worker's
    `--wan-profile` file uses the reference's region-pair form instead
    ({"intra": {...}, "inter": {...}, "pairs": {"A|B": {...}}}, reference:
    src/wantrain/resources/links.py:44-66); `from_profile` reads it. A rate of
    0 means not shaped."""

    region: str
    links: dict = field(default_factory=dict)  # region -> {"rtt_ms", "mbps"}
    enabled: bool = True
    default: Link = field(default_factory=lambda: Link(0.0, 0.0))
    pairs: dict = field(default_factory=dict)  # "A|B" (sorted) -> {"rtt_ms", "mbps"}
    intra: Link | None = None
    # Shared-pacer mode (this engine's profile keys "nic_mbps" and "shared"):
    # the node's NIC rate shared by all its connections, and whether flows
    # between two regions share one uplink per direction.
    nic_mbps: float = 0.0
    shared: bool = False

    @staticmethod
    def from_profile(region: str, prof: dict | None) -> "Emulation":
        prof = prof or {}

        def link(d):
            return Link(float(d.get("rtt_ms", 0.0)), float(d.get("mbps", 0.0)))

        return Emulation(region, enabled=bool(prof),
                         default=link(prof.get("inter") or {}),
                         pairs=dict(prof.get("pairs") or {}),
                         intra=link(prof["intra"]) if prof.get("intra") else None,
                         nic_mbps=float(prof.get("nic_mbps") or 0.0),
                         shared=bool(prof.get("shared", False)))

    def link_to(self, region: str) -> Link:
        ent = self.pairs.get("|".join(sorted((self.region or "", region or ""))))
        if ent is not None:
            return Link(float(ent.get("rtt_ms", 0.0)), float(ent.get("mbps", 0.0)))
        if region == self.region:
            return self.intra or Link(0.0, 0.0)
        ent = self.links.get(region)
        return Link(float(ent["rtt_ms"]), float(ent["mbps"])) if ent else self.default

    def shape(self, region: str, rtt: float, mbps: float) -> tuple[float, float]:
        """A measured (rtt, rate) as the emulated path would show it: the
        round trip at least the emulated one, the rate at most the emulated one."""
        lk = self.link_to(region)
        return max(rtt, lk.rtt_ms), (min(mbps, lk.mbps) if lk.mbps > 0 else mbps)


def load_emulation(region: str, wan_profile: str | None) -> Emulation | None:
    """A worker's `--wan-profile`: a path to the JSON region-pair model, or the
    JSON itself. None when there is none."""
    import json
    import os

    if not wan_profile:
        return None
    s = wan_profile.strip()
    if not s.startswith("{"):
        if not os.path.exists(s):
            return None
        with open(s) as f:
            s = f.read()
    return Emulation.from_profile(region, json.loads(s))


def probe_row(targets: list, self_index: int, secs: float = 0.25, flows: int = 1,
              emu: Emulation | None = None, timeout: float = 5.0) -> dict:
    """One row of the probe matrix: this node's round trip and upload rate to
    every target [host, port, region]. Unreachable targets give None; the own
    index gives rtt 0 and rate None (reference: the PROBE request,
    src/wantrain/worker/agent.py:649-658)."""
    rtts, rates = [], []
    for j, t in enumerate(targets):
        host, port = t[0], int(t[1])
        region = t[2] if len(t) > 2 else None
        if j == self_index:
            rtts.append(0.0)
            rates.append(None)
            continue
        try:
            r = rtt_ms(host, port, n=5, timeout=timeout)
            b = _rate([lambda o, i: _up(host, port, secs, o, i, timeout)] * flows, secs)
        except OSError:
            rtts.append(None)
            rates.append(None)
            continue
        if emu is not None and emu.enabled:
            r, b = emu.shape(region, r, b)
        rtts.append(round(r, 3))
        rates.append(round(b, 1))
    return {"rtt_ms": rtts, "bw_mbps": rates}
