"""Peer identity and the transcript-bound handshake of the data plane.

Reference behaviour: src/wantrain/transport/identity.py. Each agent holds an
ed25519 key; its peer id is sha256(public key)[:32 hex]. On connect both sides
send their public key, a fresh 16-byte challenge and an X25519 ephemeral key;
each then signs, under its own role, SHA-256 over the plane's domain, its role
and the hash of the whole transcript (both hellos in role order). Refused: a
reflected challenge, non-complementary roles, a bad signature, a peer outside
`trusted_peers` or other than `expect_peer`. The session keys of the two
directions come from HKDF-SHA256 over the X25519 secret, salted with the
transcript hash; `secure.SecureSocket` seals every later byte with them.
"""

from __future__ import annotations

import hashlib
import json
import os
import struct

from cryptography.exceptions import InvalidSignature
from cryptography.hazmat.primitives import hashes, serialization
from cryptography.hazmat.primitives.asymmetric.ed25519 import Ed25519PrivateKey, Ed25519PublicKey
from cryptography.hazmat.primitives.asymmetric.x25519 import X25519PrivateKey, X25519PublicKey
from cryptography.hazmat.primitives.kdf.hkdf import HKDF

from elysium_wan_b200.transport.sendall import send_all

P2P_DOMAIN = "elysium-p2p|v1|"
CTL_DOMAIN = "elysium-ctl|v1|"
COMPLEMENT = {"dialer": "listener", "listener": "dialer", "coordinator": "worker",
              "worker": "coordinator"}
FIRST = ("dialer", "coordinator")  # the role whose hello comes first in the transcript
KEY_LEN, PREFIX_LEN, CHAL_LEN = 32, 4, 16
_MAX_MSG = 64 * 1024


class HandshakeError(ConnectionError):
    pass


def _raw(pub) -> bytes:
    return pub.public_bytes(serialization.Encoding.Raw, serialization.PublicFormat.Raw)


def peer_id(pub_bytes: bytes) -> str:
    return hashlib.sha256(pub_bytes).hexdigest()[:32]


def default_key_path() -> str:
    """ELYSIUM_PEER_KEY, or the reference's WANTRAIN_PEER_KEY, else ~/.elysium/peer_key."""
    return os.environ.get("ELYSIUM_PEER_KEY") or os.environ.get(
        "WANTRAIN_PEER_KEY", os.path.join(os.path.expanduser("~"), ".elysium", "peer_key"))


def load_or_create_key(path: str | None = None) -> Ed25519PrivateKey:
    """The agent's ed25519 key (32 raw bytes, hex, mode 0600), created once."""
    path = path or default_key_path()
    if os.path.exists(path):
        with open(path) as f:
            return Ed25519PrivateKey.from_private_bytes(bytes.fromhex(f.read().strip()))
    key = Ed25519PrivateKey.generate()
    os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
    # Written whole to a private temp file, then linked into place: processes
    # of one agent starting together all end up with the one key that won.
    tmp = f"{path}.{os.getpid()}.tmp"
    fd = os.open(tmp, os.O_WRONLY | os.O_CREAT | os.O_EXCL, 0o600)
    with os.fdopen(fd, "w") as f:
        f.write(key.private_bytes(serialization.Encoding.Raw, serialization.PrivateFormat.Raw,
                                  serialization.NoEncryption()).hex())
    try:
        os.link(tmp, path)
    except FileExistsError:
        pass
    finally:
        os.unlink(tmp)
    with open(path) as f:
        return Ed25519PrivateKey.from_private_bytes(bytes.fromhex(f.read().strip()))


def _send(sock, obj: dict) -> bytes:
    b = json.dumps(obj, sort_keys=True, separators=(",", ":")).encode()
    send_all(sock, struct.pack("<I", len(b)) + b)
    return b


def _recv(sock) -> tuple[dict, bytes]:
    def exact(n):
        buf = b""
        while len(buf) < n:
            c = sock.recv(n - len(buf))
            if not c:
                raise HandshakeError("peer closed during the handshake")
            buf += c
        return buf

    (n,) = struct.unpack("<I", exact(4))
    if n > _MAX_MSG:
        raise HandshakeError("handshake message too large")
    b = exact(n)
    try:
        return json.loads(b.decode()), b
    except ValueError as e:
        raise HandshakeError("handshake message is not JSON") from e


def _hexfield(msg: dict, name: str, n: int) -> bytes:
    v = msg.get(name)
    if not isinstance(v, str) or len(v) != 2 * n or v != v.lower():
        raise HandshakeError(f"handshake field {name!r} is not {n} bytes of lowercase hex")
    try:
        return bytes.fromhex(v)
    except ValueError as e:
        raise HandshakeError(f"handshake field {name!r} is not hex") from e


def _digest(domain: str, role: str, th: bytes) -> bytes:
    return hashlib.sha256(domain.encode() + role.encode() + b"|" + th).digest()


class Session:
    """Result of a handshake: the peer's id and the two directions' keys."""

    def __init__(self, peer: str, send_key, send_prefix, recv_key, recv_prefix):
        self.peer = peer
        self.send_key, self.send_prefix = send_key, send_prefix
        self.recv_key, self.recv_prefix = recv_key, recv_prefix


def authenticate(sock, key: Ed25519PrivateKey, role: str, domain: str = P2P_DOMAIN,
                 trusted_peers=None, expect_peer: str | None = None) -> Session:
    if role not in COMPLEMENT:
        raise ValueError(f"unknown role {role!r}")
    eph = X25519PrivateKey.generate()
    chal = os.urandom(CHAL_LEN)
    mine = {"pub": _raw(key.public_key()).hex(), "chal": chal.hex(),
            "eph": _raw(eph.public_key()).hex(), "role": role}
    mine_b = _send(sock, mine)
    theirs, theirs_b = _recv(sock)
    pub = _hexfield(theirs, "pub", 32)
    their_chal = _hexfield(theirs, "chal", CHAL_LEN)
    their_eph = _hexfield(theirs, "eph", 32)
    if theirs.get("role") != COMPLEMENT[role]:
        raise HandshakeError(f"peer declared role {theirs.get('role')!r}, expected "
                             f"{COMPLEMENT[role]!r}")
    if their_chal == chal:
        raise HandshakeError("reflected challenge")
    first, second = (mine_b, theirs_b) if role in FIRST else (theirs_b, mine_b)
    th = hashlib.sha256(struct.pack("<I", len(first)) + first + struct.pack("<I", len(second))
                        + second).digest()
    _send(sock, {"sig": key.sign(_digest(domain, role, th)).hex()})
    msg, _ = _recv(sock)
    sig = _hexfield(msg, "sig", 64)
    try:
        Ed25519PublicKey.from_public_bytes(pub).verify(sig, _digest(domain, theirs["role"], th))
    except InvalidSignature as e:
        raise HandshakeError("peer signature does not verify") from e
    pid = peer_id(pub)
    if trusted_peers is not None and pid not in set(trusted_peers):
        raise HandshakeError(f"peer {pid} is not in trusted_peers")
    if expect_peer is not None and pid != expect_peer:
        raise HandshakeError(f"peer {pid} is not the expected {expect_peer}")
    secret = eph.exchange(X25519PublicKey.from_public_bytes(their_eph))
    okm = HKDF(algorithm=hashes.SHA256(), length=2 * (KEY_LEN + PREFIX_LEN), salt=th,
               info=domain.encode()).derive(secret)
    a = (okm[:KEY_LEN], okm[KEY_LEN:KEY_LEN + PREFIX_LEN])
    b = (okm[KEY_LEN + PREFIX_LEN:2 * KEY_LEN + PREFIX_LEN], okm[2 * KEY_LEN + PREFIX_LEN:])
    send, recv = (a, b) if role in FIRST else (b, a)
    return Session(pid, send[0], send[1], recv[0], recv[1])
