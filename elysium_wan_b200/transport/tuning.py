"""Socket tuning for long, fat WAN hops of the TCP data plane.

Reference behaviour: src/wantrain/transport/tuning.py (TRANSPORT-I10 / I13).
Three per-socket knobs, none of which changes a payload byte, all applied
before connect() / listen() (accepted sockets inherit the listener's):

- congestion control: BBR when the kernel offers it (it paces at the
  measured bottleneck rate instead of halving its window on every loss);
- buffers: SO_SNDBUF / SO_RCVBUF sized for the bandwidth-delay product, set
  only when the kernel's hard cap admits the size and the size beats the
  autotuning ceiling (setting a buffer turns autotuning off for it);
- pacing: SO_MAX_PACING_RATE turns on the kernel's own TCP pacing, so many
  flows do not burst one boundary into a shallow bottleneck queue at once.

Environment: ELYSIUM_TCP_CC (default "bbr", "off" keeps the system's),
ELYSIUM_TCP_BUF (bytes, default 32 MiB), ELYSIUM_TCP_PACE_MBPS (per flow,
default 10000, "off"); the reference's WANTRAIN_TCP_* names are accepted too.
Nothing here raises: a knob the kernel refuses keeps its default, and the
report says what holds.
"""

from __future__ import annotations

import os
import socket
import struct

DEFAULT_CC = "bbr"
DEFAULT_BUF = 32 << 20
DEFAULT_PACE_MBPS = 10000.0
SO_MAX_PACING_RATE = getattr(socket, "SO_MAX_PACING_RATE",
                             47 if os.uname().sysname == "Linux" else None)
_PROC = "/proc/sys/net"


def _env(name: str, default: str) -> str:
    return os.environ.get(f"ELYSIUM_{name}", os.environ.get(f"WANTRAIN_{name}", default))


def _read_int(path: str) -> int | None:
    try:
        with open(path) as fh:
            return int(fh.read().split()[-1])
    except (OSError, ValueError, IndexError):
        return None


def available_cc() -> set:
    try:
        with open(f"{_PROC}/ipv4/tcp_available_congestion_control") as fh:
            return set(fh.read().split())
    except OSError:
        return set()


def kernel_caps() -> dict:
    return {"wmem_max": _read_int(f"{_PROC}/core/wmem_max"),
            "rmem_max": _read_int(f"{_PROC}/core/rmem_max"),
            "tcp_wmem": _read_int(f"{_PROC}/ipv4/tcp_wmem"),
            "tcp_rmem": _read_int(f"{_PROC}/ipv4/tcp_rmem")}


def plan(want_buf: int, caps: dict) -> dict:
    """{"sndbuf", "rcvbuf"}: bytes to set, or None to keep autotuning (pure)."""
    out = {}
    for key, hard, auto in (("sndbuf", "wmem_max", "tcp_wmem"), ("rcvbuf", "rmem_max", "tcp_rmem")):
        cap, ceiling = caps.get(hard), caps.get(auto)
        out[key] = want_buf if cap and cap >= want_buf and (ceiling is None or want_buf > ceiling) \
            else None
    return out


def pace(sock) -> int | str:
    want = _env("TCP_PACE_MBPS", str(DEFAULT_PACE_MBPS))
    if want == "off":
        return "off"
    if SO_MAX_PACING_RATE is None:
        return "unsupported"
    try:
        rate = int(float(want) * 1e6 / 8)
        sock.setsockopt(socket.SOL_SOCKET, SO_MAX_PACING_RATE, struct.pack("Q", rate))
        return struct.unpack("Q", sock.getsockopt(socket.SOL_SOCKET, SO_MAX_PACING_RATE, 8))[0]
    except (OSError, ValueError, struct.error):
        return "unsupported"


def tune(sock) -> dict:
    """Apply congestion control, buffers and pacing; -> what holds after."""
    out: dict = {}
    want_cc = _env("TCP_CC", DEFAULT_CC)
    if not hasattr(socket, "TCP_CONGESTION"):
        out["cc"] = "unsupported"
    else:
        if want_cc and want_cc != "off" and want_cc in available_cc():
            try:
                sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_CONGESTION, want_cc.encode())
            except OSError:
                pass
        try:
            out["cc"] = sock.getsockopt(socket.IPPROTO_TCP, socket.TCP_CONGESTION, 16) \
                .split(b"\0", 1)[0].decode()
        except OSError:
            out["cc"] = "unsupported"
    want_buf = int(_env("TCP_BUF", str(DEFAULT_BUF)))
    sizes = plan(want_buf, kernel_caps())
    for key, opt in (("sndbuf", socket.SO_SNDBUF), ("rcvbuf", socket.SO_RCVBUF)):
        if sizes[key] is None:
            out[key] = "auto"
            continue
        try:
            sock.setsockopt(socket.SOL_SOCKET, opt, sizes[key])
            out[key] = sock.getsockopt(socket.SOL_SOCKET, opt)
        except OSError:
            out[key] = "auto"
    out["pace"] = pace(sock)
    try:
        sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
    except OSError:
        pass
    return out


def connect(host: str, port: int, timeout: float):
    """A connected, tuned socket and the tuning report."""
    err: OSError | None = None
    for af, kind, proto, _n, addr in socket.getaddrinfo(host, port, type=socket.SOCK_STREAM):
        s = socket.socket(af, kind, proto)
        try:
            applied = tune(s)
            s.settimeout(timeout)
            s.connect(addr)
            s.settimeout(None)
            return s, applied
        except OSError as e:
            err = e
            s.close()
    raise err or OSError(f"no address for {host}:{port}")
