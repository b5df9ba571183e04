"""AEAD record layer of the data plane.

Reference behaviour: src/wantrain/transport/secure.py. Every byte written
through a SecureSocket travels in a record

    u32 big-endian L | ciphertext || 16-byte tag        (L = ciphertext + 16)

of at most MAX_RECORD plaintext bytes; the length header is the associated
data. The nonce is the direction's 4-byte prefix and its 64-bit big-endian
record counter, implicit (never on the wire), from 0 upward, so a replayed,
reordered or dropped record fails its tag. Each direction rekeys
deterministically every `rekey_records` records: key[e+1] =
HKDF-Expand-SHA256(key[e], "elysium rekey" || u64be(e+1)); the counter is never
reset. Any failure on receive (bad tag, oversized length, truncated record)
leaves the socket failed: it never resynchronises, and there is no plaintext
mode. The AEAD calls release the interpreter lock on large records.
"""

from __future__ import annotations

import errno
import struct

from cryptography.exceptions import InvalidTag
from cryptography.hazmat.primitives import hashes
from cryptography.hazmat.primitives.ciphers.aead import AESGCM, ChaCha20Poly1305
from cryptography.hazmat.primitives.kdf.hkdf import HKDFExpand

from elysium_wan_b200.transport.sendall import enobufs_every, send_all

CIPHERS = {"chacha20-poly1305": ChaCha20Poly1305, "aes-256-gcm": AESGCM}
MAX_RECORD = 1 << 20
TAG = 16
REKEY_RECORDS = 1 << 24
_LEN = struct.Struct(">I")


def _next_key(key: bytes, epoch: int) -> bytes:
    return HKDFExpand(hashes.SHA256(), 32, b"elysium rekey" + struct.pack(">Q", epoch)).derive(key)


class _Direction:
    def __init__(self, cipher: str, key: bytes, prefix: bytes, rekey_records: int):
        if cipher not in CIPHERS:
            raise ValueError(f"cipher {cipher!r} is not one of {sorted(CIPHERS)}")
        if len(key) != 32 or len(prefix) != 4:
            raise ValueError("a direction needs a 32-byte key and a 4-byte nonce prefix")
        self.cls, self.key, self.prefix = CIPHERS[cipher], key, prefix
        self.aead = self.cls(key)
        self.counter = 0
        self.epoch = 0
        self.rekey_records = rekey_records

    def nonce(self) -> bytes:
        if self.counter and self.counter % self.rekey_records == 0 and \
                self.counter // self.rekey_records > self.epoch:
            self.epoch += 1
            self.key = _next_key(self.key, self.epoch)
            self.aead = self.cls(self.key)
        n = self.prefix + struct.pack(">Q", self.counter)
        self.counter += 1
        return n


class SecureSocket:
    """A socket whose every byte is sealed (see the module docstring)."""

    sealed = True

    def __init__(self, sock, session, cipher: str = "chacha20-poly1305",
                 rekey_records: int = REKEY_RECORDS):
        self.sock = sock
        self.peer = session.peer
        self.tx = _Direction(cipher, session.send_key, session.send_prefix, rekey_records)
        self.rx = _Direction(cipher, session.recv_key, session.recv_prefix, rekey_records)
        self._buf = b""
        self._off = 0
        self._failed = False
        self._every = enobufs_every()
        self._attempts = 0
        self._seam = self._refuse if self._every else None

    def _refuse(self):
        """The ENOBUFS test seam: every N-th send attempt is refused before
        it reaches the kernel (nothing written)."""
        self._attempts += 1
        if self._attempts % self._every == 0:
            raise OSError(errno.ENOBUFS, "No buffer space available (test seam)")

    def fileno(self):
        return self.sock.fileno()

    def settimeout(self, t):
        self.sock.settimeout(t)

    def close(self):
        self.sock.close()

    def shutdown(self, how):
        self.sock.shutdown(how)

    def sendall(self, data) -> None:
        view = memoryview(data)
        if len(view) == 0:
            return
        for i in range(0, len(view), MAX_RECORD):
            chunk = view[i:i + MAX_RECORD]
            hdr = _LEN.pack(len(chunk) + TAG)
            send_all(self.sock, hdr + self.tx.aead.encrypt(self.tx.nonce(), bytes(chunk), hdr),
                     self._seam)

    def _fail(self, why: str):
        self._failed = True
        self._buf, self._off = b"", 0
        return ConnectionError(f"sealed stream failed: {why}")

    def _exact(self, n: int) -> bytes:
        buf = bytearray(n)
        view = memoryview(buf)
        got = 0
        while got < n:
            r = self.sock.recv_into(view[got:], n - got)
            if r == 0:
                if got == 0 and n == _LEN.size:
                    raise ConnectionError("peer closed")
                raise self._fail("truncated record")
            got += r
        return bytes(buf)

    def _next_record(self):
        hdr = self._exact(_LEN.size)
        (L,) = _LEN.unpack(hdr)
        if L < TAG or L > MAX_RECORD + TAG:
            raise self._fail(f"record length {L} out of range")
        body = self._exact(L)
        try:
            self._buf = self.rx.aead.decrypt(self.rx.nonce(), body, hdr)
        except InvalidTag:
            raise self._fail("record does not authenticate") from None
        self._off = 0

    def recv_into(self, buffer, nbytes: int = 0) -> int:
        if self._failed:
            raise ConnectionError("sealed stream failed earlier")
        view = memoryview(buffer)
        n = nbytes or len(view)
        if self._off >= len(self._buf):
            try:
                self._next_record()
            except ConnectionError as e:
                if str(e) == "peer closed":
                    return 0
                raise
        k = min(n, len(self._buf) - self._off)
        view[:k] = self._buf[self._off:self._off + k]
        self._off += k
        return k

    def recv(self, n: int) -> bytes:
        buf = bytearray(n)
        k = self.recv_into(buf, n)
        return bytes(buf[:k])
