"""Control channel between the coordinator and worker agents.

Wire format (reference: src/wantrain/transport/control.py:54-277): a frame is a
u32 big-endian header length, a JSON header, a u64 big-endian body length and
the body bytes (files travel as bodies, streamed to disk by the receiver).
Admission: the coordinator sends CHALLENGE {nonce, coordinator_id}; the agent
answers HELLO with mac = HMAC-SHA256(token, nonce || coordinator_id); a wrong
mac gets REJECT and the connection is closed. The token comes from --token or
WANTRAIN_COORD_TOKEN.

Message kinds (public surface):
  agent -> coordinator: HELLO, HEARTBEAT, PROGRESS, TELEM_STEP, TELEMETRY, EXIT, CKPT,
                        RESULT, *_ACK, *_RESULT
  coordinator -> agent: CHALLENGE, WELCOME, REJECT, ASSIGN, PROFILE, FIT,
                        MEASURE, PROBE, ABORT, RESTORE, RELEASE, SHUTDOWN
"""

from __future__ import annotations

import hashlib
import hmac
import json
import os
import socket
import struct
import threading

MAX_HEADER = 16 << 20
MAX_BODY = 1 << 40


def token_mac(token: str, nonce: str, coordinator_id: str) -> str:
    return hmac.new(token.encode(), (nonce + coordinator_id).encode(), hashlib.sha256).hexdigest()


def check_mac(token: str, nonce: str, coordinator_id: str, mac: str) -> bool:
    return hmac.compare_digest(token_mac(token, nonce, coordinator_id), str(mac))


def _recv_exact(sock: socket.socket, n: int) -> bytes:
    buf = bytearray()
    while len(buf) < n:
        chunk = sock.recv(min(n - len(buf), 1 << 20))
        if not chunk:
            raise ConnectionError("control connection closed")
        buf += chunk
    return bytes(buf)


class Channel:
    """A framed, thread-safe (for sends) message channel over one socket."""

    def __init__(self, sock: socket.socket):
        self.sock = sock
        self.lock = threading.Lock()
        self.closed = False
        try:
            sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        except OSError:
            pass

    def send(self, kind: str, body: bytes = b"", **fields):
        hdr = json.dumps(dict(fields, kind=kind)).encode()
        with self.lock:
            self.sock.sendall(struct.pack(">I", len(hdr)) + hdr + struct.pack(">Q", len(body)))
            if body:
                self.sock.sendall(body)

    def send_file(self, kind: str, path: str, **fields):
        with open(path, "rb") as f:
            data = f.read()
        fields.setdefault("sha256", hashlib.sha256(data).hexdigest())
        self.send(kind, data, **fields)

    def recv(self) -> tuple[dict, bytes]:
        (n,) = struct.unpack(">I", _recv_exact(self.sock, 4))
        if n > MAX_HEADER:
            raise ValueError(f"control header of {n} bytes refused")
        hdr = json.loads(_recv_exact(self.sock, n))
        (m,) = struct.unpack(">Q", _recv_exact(self.sock, 8))
        if m > MAX_BODY:
            raise ValueError("control body too large")
        body = _recv_exact(self.sock, m) if m else b""
        return hdr, body

    def close(self):
        self.closed = True
        try:
            self.sock.shutdown(socket.SHUT_RDWR)
        except OSError:
            pass
        self.sock.close()


def control_dial(host: str, port: int, timeout: float = 10.0) -> Channel:
    s = socket.create_connection((host, port), timeout=timeout)
    s.settimeout(None)
    return Channel(s)


def control_listen(host: str, port: int) -> socket.socket:
    s = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
    s.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
    s.bind((host, port))
    s.listen(64)
    return s


def new_nonce() -> str:
    return os.urandom(16).hex()
