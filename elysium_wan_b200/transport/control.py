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

from elysium_wan_b200.transport.sendall import send_all

MAX_HEADER = 16 << 20
MAX_BODY = 1 << 40
SPILL_MIN = 64 << 20  # bodies this large go to a file as they arrive (when the channel has a spill dir)
_CHUNK = 4 << 20


class Spilled:
    """A message body the receiver streamed into a file as it arrived, with
    its sha256 computed on the way (a checkpoint part of gigabytes never sits
    in memory). `move_to` renames it into place (same filesystem)."""

    def __init__(self, path: str, size: int, sha256: str):
        self.path, self.size, self.sha256 = path, size, sha256

    def __len__(self):
        return self.size

    def read(self) -> bytes:
        with open(self.path, "rb") as f:
            return f.read()

    def move_to(self, dst: str):
        os.replace(self.path, dst)

    def discard(self):
        try:
            os.unlink(self.path)
        except FileNotFoundError:
            pass


def body_sha256(body) -> str:
    return body.sha256 if isinstance(body, Spilled) else hashlib.sha256(body).hexdigest()


def write_body(body, dst: str):
    """Put a received body at dst (through dst + '.part', renamed when whole)."""
    if isinstance(body, Spilled):
        body.move_to(dst)
        return
    with open(dst + ".part", "wb") as f:
        f.write(body)
    os.replace(dst + ".part", dst)


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


SEND_STALL_S = 10


class Channel:
    """A framed, thread-safe (for sends) message channel over one socket."""

    def __init__(self, sock: socket.socket, spill_dir: str | None = None):
        self.sock = sock
        self.lock = threading.Lock()
        self.closed = False
        self.spill_dir = spill_dir  # where large bodies are streamed (None: in memory)
        self.spill_min = int(os.environ.get("EWB_CONTROL_SPILL_MIN", SPILL_MIN))
        try:
            sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        except OSError:
            pass
        # A send that the peer does not drain must not block forever (two
        # sides sending at once with full buffers, one of them holding a lock
        # its own reader needs, would never end): the kernel gives up on a
        # blocked send after SEND_STALL_S (EAGAIN), send_all retries until it
        # has made no progress for its budget, and the send then fails like a
        # lost peer.
        raw = getattr(sock, "sock", sock)
        try:
            raw.setsockopt(socket.SOL_SOCKET, socket.SO_SNDTIMEO,
                           struct.pack("ll", int(SEND_STALL_S), 0))
        except (OSError, AttributeError):
            pass

    def _send(self, data) -> None:
        """Every byte out; a plain socket retries the kernel's transient
        refusals (transport/sendall.py), a sealed one does so per record."""
        if getattr(self.sock, "sealed", False):
            self.sock.sendall(data)
        else:
            send_all(self.sock, data)

    def send(self, kind: str, body: bytes = b"", **fields):
        hdr = json.dumps(dict(fields, kind=kind)).encode()
        with self.lock:
            self._send(struct.pack(">I", len(hdr)) + hdr + struct.pack(">Q", len(body)))
            if body:
                self._send(body)

    def send_file(self, kind: str, path: str, **fields):
        """Send a file as the body, streamed from disk in 4 MiB pieces (its
        sha256 from a first pass over the file unless given)."""
        size = os.path.getsize(path)
        if "sha256" not in fields:
            h = hashlib.sha256()
            with open(path, "rb") as f:
                for piece in iter(lambda: f.read(_CHUNK), b""):
                    h.update(piece)
            fields["sha256"] = h.hexdigest()
        hdr = json.dumps(dict(fields, kind=kind)).encode()
        with self.lock, open(path, "rb") as f:
            self._send(struct.pack(">I", len(hdr)) + hdr + struct.pack(">Q", size))
            sent = 0
            for piece in iter(lambda: f.read(_CHUNK), b""):
                self._send(piece)
                sent += len(piece)
            if sent != size:
                raise ConnectionError(f"{path} changed size while being sent")

    def recv(self) -> tuple:
        """(header, body): body is bytes, or a Spilled file for bodies of at
        least SPILL_MIN bytes when the channel has a spill directory."""
        (n,) = struct.unpack(">I", _recv_exact(self.sock, 4))
        if n > MAX_HEADER:
            raise ValueError(f"control header of {n} bytes refused")
        hdr = json.loads(_recv_exact(self.sock, n))
        (m,) = struct.unpack(">Q", _recv_exact(self.sock, 8))
        if m > MAX_BODY:
            raise ValueError("control body too large")
        if m and m >= self.spill_min and self.spill_dir:
            return hdr, self._spill(m)
        body = _recv_exact(self.sock, m) if m else b""
        return hdr, body

    def _spill(self, m: int) -> Spilled:
        import tempfile

        os.makedirs(self.spill_dir, exist_ok=True)
        fd, path = tempfile.mkstemp(prefix="body-", dir=self.spill_dir)
        h = hashlib.sha256()
        left = m
        try:
            with os.fdopen(fd, "wb") as f:
                while left:
                    piece = self.sock.recv(min(left, _CHUNK))
                    if not piece:
                        raise ConnectionError("control connection closed")
                    h.update(piece)
                    f.write(piece)
                    left -= len(piece)
        except BaseException:
            try:
                os.unlink(path)
            except FileNotFoundError:
                pass
            raise
        return Spilled(path, m, h.hexdigest())

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
