"""Shared pacing for WAN emulation: bandwidth that several connections share.

A link's own `bw_mbps` paces that connection alone. A real machine has one
NIC for all its connections, and two sites one uplink per direction for all
the flows between them, so concurrent flows split those rates instead of
each getting its own (reference behaviour: the shared-pacer mode of
src/wantrain/transport/shim.py, TRANSPORT-I10; semantics only).

`HostBucket` is a token bucket that every thread and process of one host
opening the same file shares. The file holds two doubles: the CLOCK_MONOTONIC
time at which the bucket's last reserved byte will have left, and the rate
(checked on open, so two runs never share a bucket at different rates). A
reservation takes an exclusive `lockf` on the file (processes) under a thread
lock (threads), reads the clock, advances it by bytes / rate starting no
earlier than now minus the burst allowance, and writes it back; the caller
then sleeps until that time. Pacing delays bytes and never touches them.

Budgets are named by a key (a node id for a NIC, "regionA>regionB" for an
uplink) inside a directory shared by the run's processes: `EWB_PACER_DIR`
when set (the local launcher and the agents set it per run), else a
per-user directory under the system temporary directory.
"""

from __future__ import annotations

import hashlib
import math
import os
import re
import struct
import tempfile
import threading
import time

_REC = struct.Struct("<dd")  # next free time (monotonic s), rate (Mbit/s)
_STALE_S = 3600.0


class HostBucket:
    def __init__(self, mbps: float, path: str, burst_ms: float = 10.0):
        if not (isinstance(mbps, (int, float)) and math.isfinite(mbps) and mbps > 0):
            raise ValueError(f"bucket rate must be a finite positive Mbit/s, got {mbps!r}")
        if burst_ms < 0:
            raise ValueError("burst_ms must be >= 0")
        self.mbps, self.path, self.burst_s = float(mbps), path, burst_ms / 1e3
        self._lock = threading.Lock()
        self._fd, self._pid = -1, -1
        self._open()

    def _open(self):
        import fcntl

        fd = os.open(self.path, os.O_RDWR | os.O_CREAT | getattr(os, "O_NOFOLLOW", 0), 0o600)
        st = os.fstat(fd)
        if not (st.st_mode & 0o170000 == 0o100000) or st.st_uid != os.getuid():
            os.close(fd)
            raise ValueError(f"{self.path}: not a regular file of this user")
        fcntl.lockf(fd, fcntl.LOCK_EX)
        try:
            raw = os.pread(fd, _REC.size, 0)
            if len(raw) == 0:
                os.pwrite(fd, _REC.pack(0.0, self.mbps), 0)
            elif len(raw) != _REC.size:
                raise ValueError(f"{self.path}: not a bucket file")
            else:
                _, rate = _REC.unpack(raw)
                if rate != self.mbps:
                    raise ValueError(f"{self.path}: a {rate} Mbit/s bucket, not {self.mbps}")
        except BaseException:
            fcntl.lockf(fd, fcntl.LOCK_UN)
            os.close(fd)
            raise
        fcntl.lockf(fd, fcntl.LOCK_UN)
        self._fd, self._pid = fd, os.getpid()

    def reserve(self, nbytes: int) -> float:
        """Book nbytes on the bucket; returns the monotonic time they have left by."""
        import fcntl

        if nbytes < 0:
            raise ValueError("negative reservation")
        cost = nbytes * 8.0 / (self.mbps * 1e6)
        with self._lock:
            if self._pid != os.getpid():  # a forked child opens its own descriptor
                os.close(self._fd)
                self._open()
            fcntl.lockf(self._fd, fcntl.LOCK_EX)
            try:
                now = time.monotonic()
                clock, _ = _REC.unpack(os.pread(self._fd, _REC.size, 0))
                if not math.isfinite(clock) or clock - now > _STALE_S:
                    clock = now  # a file from another boot: start over
                end = max(clock, now - self.burst_s) + cost
                os.pwrite(self._fd, _REC.pack(end, self.mbps), 0)
            finally:
                fcntl.lockf(self._fd, fcntl.LOCK_UN)
        return end

    def close(self):
        with self._lock:
            if self._fd >= 0 and self._pid == os.getpid():
                os.close(self._fd)
            self._fd = -1


def pacer_dir(tag: str = "run") -> str:
    d = os.environ.get("EWB_PACER_DIR")
    if not d:
        d = os.path.join(tempfile.gettempdir(), f"ewb-pacers-{os.getuid()}", tag)
    os.makedirs(d, mode=0o700, exist_ok=True)
    return d


_open: dict = {}
_open_lock = threading.Lock()


def bucket(key: str, mbps: float, tag: str = "run") -> HostBucket:
    """The process's handle on the shared bucket `key` (one per key and rate)."""
    safe = re.sub(r"[^A-Za-z0-9_.>-]", "_", key)[:80]
    name = f"{safe}-{hashlib.sha256(key.encode()).hexdigest()[:12]}.bucket"
    path = os.path.join(pacer_dir(tag), name)
    with _open_lock:
        b = _open.get((path, mbps))
        if b is None:
            b = _open[(path, mbps)] = HostBucket(mbps, path)
        return b


def reverse_link(link: dict) -> dict:
    """The same hop seen from its other end (the backward direction): the
    receiver's NIC becomes the sender's, and the uplink runs the other way."""
    out = dict(link or {})
    out["egress_key"], out["ingress_key"] = out.get("ingress_key", ""), out.get("egress_key", "")
    out["egress_mbps"], out["ingress_mbps"] = out.get("ingress_mbps", 0.0), out.get("egress_mbps", 0.0)
    up = out.get("uplink_key") or ""
    if ">" in up:
        a, b = up.split(">", 1)
        out["uplink_key"] = f"{b}>{a}"
    return out


def link_buckets(link: dict, tag: str = "run") -> list:
    """The shared budgets a link configuration names: egress (the sender's
    NIC), uplink (the site pair's uplink in this direction) and ingress (the
    receiver's NIC), each as {kind}_key and {kind}_mbps."""
    out = []
    for kind in ("egress", "uplink", "ingress"):
        key, mbps = link.get(f"{kind}_key") or "", float(link.get(f"{kind}_mbps") or 0.0)
        if key and mbps > 0:
            out.append(bucket(f"{kind}:{key}", mbps, tag))
    return out


def pair_link(spec, base: dict, src: tuple, dst: tuple | None) -> dict:
    """The configuration of the connection from slot `src` to slot `dst`:
    the hop's own shaping, plus, under the spec's pacing "shared", the
    sender's NIC egress budget, the receiver's NIC ingress budget and, between
    two sites, that direction's uplink (the reference's peer_egress_mbps,
    peer_ingress_mbps, sites and uplink_mbps fields). `dst` None (a plane
    whose one pacer serves several receivers): the sender's NIC only."""
    out = dict(base or {})
    if getattr(spec, "pacing", "link") != "shared":
        return out
    r, p = src
    out["egress_key"], out["egress_mbps"] = f"slot{r}.{p}", float(spec.peer_egress_mbps[r][p])
    if dst is not None:
        r2, q = dst
        out["ingress_key"] = f"slot{r2}.{q}"
        out["ingress_mbps"] = float(spec.peer_ingress_mbps[r2][q])
        a, b = spec.sites[r][p], spec.sites[r2][q]
        if a != b:
            out["uplink_key"], out["uplink_mbps"] = f"{a}>{b}", float(spec.uplink_mbps[f"{a}->{b}"])
    return out
