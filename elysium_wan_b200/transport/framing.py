"""Frames of the TCP data plane.

Reference: src/wantrain/transport/framing.py. The header is kept
byte-compatible (an interface two ends must share):

    magic u16 0xE17A | type u8 | codec u8 | step u32 | mb u32 | chunk u16 |
    ndim u8 | frag_idx u16 | frag_cnt u16 | dims u32 x ndim | paylen u64 |
    payload                                                   (little-endian)

Types FWD, BWD, END, GRADS, PARAMS, LOSS, HELLO, TIED; codecs RAW_F32,
RAW_I64, FP8_PLANES, OBJ, F32_PLANES, PLANES. `chunk` is the sending peer of
a wide stage. Fragments are byte ranges of one payload, reassembled by
concatenation in frag_idx order, so re-fragmenting never changes a value. OBJ
payloads are JSON (control objects only; decoding never executes code). A
type outside the known set is refused before its payload is read; a payload
above MAX_PAYLOAD is refused before it is allocated.

Plain sockets go through the native `_wire` sendmsg / recv loop with the
interpreter lock released; a sealed socket (transport/secure.py) takes the
same bytes through its record layer.
"""

from __future__ import annotations

import json
import os
import struct
import time
from dataclasses import dataclass

import torch

from elysium_wan_b200 import codec

MAGIC = 0xE17A
FWD, BWD, END, GRADS, PARAMS, LOSS, HELLO, TIED = range(8)
FRAME_TYPES = frozenset({FWD, BWD, END, GRADS, PARAMS, LOSS, HELLO, TIED})
RAW_F32, RAW_I64, FP8_PLANES, OBJ, F32_PLANES, PLANES = range(6)
_HDR = struct.Struct("<HBBIIHBHH")
MAX_PAYLOAD = int(os.environ.get("WANTRAIN_MAX_FRAME_BYTES", str(4 << 30)))


class FrameError(ConnectionError):
    """The byte stream is not a valid frame sequence."""


@dataclass
class Frame:
    type: int
    codec: int
    step: int
    mb: int
    chunk: int
    payload: bytes
    shape: tuple
    frag_idx: int = 0
    frag_cnt: int = 1

    def tensor(self):
        """The payload as a tensor (an fp8 b128 PLANES payload gives the
        (codes, scales) pair)."""
        if self.codec == OBJ:
            raise ValueError("control frame has no tensor")
        if self.codec == PLANES:
            if self.payload and self.payload[0] in codec.Q8_B128:
                return codec.q8_b128_decode(self.payload, self.shape)
            return codec.planes_decode(self.payload, self.shape)
        if self.codec == FP8_PLANES:
            return codec.fp8_planes_decode(self.payload, self.shape)
        if self.codec == F32_PLANES:
            return codec.f32_planes_decode(self.payload, self.shape)
        dt = {RAW_F32: torch.float32, RAW_I64: torch.int64}.get(self.codec)
        if dt is None:
            raise FrameError(f"unknown tensor codec {self.codec}")
        return codec._tensor_of(self.payload, dt, self.shape)

    def obj(self):
        if self.codec != OBJ:
            raise FrameError(f"frame codec {self.codec} carries no object")
        return json.loads(self.payload.decode()) if self.payload else None


def encode_tensor(t, wire_codec: str = "raw", level: int = 1):
    """(codec id, payload, shape) of a tensor under a spec's wire_codec.
    raw: exact bytes (fp32 / int64 as RAW, other dtypes as uncompressed
    PLANES); planes: byte planes + zlib; f32_planes / fp8_planes as named.
    A (codes, scales) pair is this engine's fp8 b128 boundary."""
    if isinstance(t, tuple):
        payload, shape = codec.q8_b128_encode(t[0], t[1], 0 if wire_codec == "raw" else level)
        return PLANES, payload, shape
    if wire_codec == "raw":
        if t.dtype == torch.float32:
            return RAW_F32, bytes(codec._bytes_of(t)), tuple(t.shape)
        if t.dtype == torch.int64:
            return RAW_I64, bytes(codec._bytes_of(t)), tuple(t.shape)
        p, s = codec.planes_encode(t, level=0)
        return PLANES, p, s
    if wire_codec == "planes":
        p, s = codec.planes_encode(t, level)
        return PLANES, p, s
    if wire_codec == "f32_planes":
        p, s = codec.f32_planes_encode(t, level)
        return F32_PLANES, p, s
    if wire_codec == "fp8_planes":
        p, s = codec.fp8_planes_encode(t, level)
        return FP8_PLANES, p, s
    raise ValueError(f"unknown wire_codec {wire_codec!r}")


def header(ftype, codec_id, step, mb, chunk, shape, frag_idx, frag_cnt, paylen) -> bytes:
    if ftype not in FRAME_TYPES:
        raise ValueError(f"unknown frame type {ftype}")
    return (_HDR.pack(MAGIC, ftype, codec_id, step, mb, chunk, len(shape), frag_idx, frag_cnt)
            + (struct.pack(f"<{len(shape)}I", *shape) if shape else b"")
            + struct.pack("<Q", paylen))


def send_frame(sock, ftype, step, mb, payload, chunk=0, codec_id=None, shape=(), frag_idx=0,
               frag_cnt=1) -> int:
    """Send one frame; payload is bytes (with codec_id) or a JSON-able object
    (OBJ). Returns the bytes written."""
    if codec_id is None:
        payload, codec_id = json.dumps(payload).encode(), OBJ
    if hasattr(sock, "sealed"):
        data = header(ftype, codec_id, step, mb, chunk, shape, frag_idx, frag_cnt,
                      len(payload)) + bytes(payload)
        sock.sendall(data)
        return len(data)
    return codec.wire().send_frame(sock.fileno(), ftype, codec_id, step, mb, chunk,
                                   [int(x) for x in shape], payload, frag_idx, frag_cnt)


def send_end(sock):
    send_frame(sock, END, 0, 0, None)


def _recv_exact(sock, n: int) -> bytes:
    buf = bytearray(n)
    view = memoryview(buf)
    got = 0
    while got < n:
        r = sock.recv_into(view[got:], n - got)
        if r == 0:
            raise ConnectionError("peer closed")
        got += r
    return bytes(buf)


def recv_frame(sock) -> Frame:
    if not hasattr(sock, "sealed"):
        try:
            t, c, st, mb, ch, shape, fi, fc, payload = codec.wire().recv_frame(sock.fileno(),
                                                                                MAX_PAYLOAD)
        except RuntimeError as e:
            raise FrameError(str(e)) if "magic" in str(e) or "type" in str(e) or \
                "limit" in str(e) else ConnectionError(str(e)) from e
        return Frame(t, c, st, mb, ch, payload, tuple(shape), fi, fc)
    magic, t, c, st, mb, ch, ndim, fi, fc = _HDR.unpack(_recv_exact(sock, _HDR.size))
    if magic != MAGIC:
        raise FrameError("bad frame magic")
    if t not in FRAME_TYPES:
        raise FrameError(f"unknown frame type {t}")
    shape = struct.unpack(f"<{ndim}I", _recv_exact(sock, 4 * ndim)) if ndim else ()
    (n,) = struct.unpack("<Q", _recv_exact(sock, 8))
    if n > MAX_PAYLOAD:
        raise FrameError(f"frame payload {n} exceeds limit {MAX_PAYLOAD}")
    return Frame(t, c, st, mb, ch, _recv_exact(sock, n), tuple(shape), fi, fc)


class Reassembler:
    """Collects fragments; returns the whole Frame when its last one lands."""

    def __init__(self):
        self._parts: dict = {}
        self._first: dict = {}
        self.spread_s = 0.0

    def push(self, f: Frame):
        if f.frag_cnt <= 1:
            self.spread_s = 0.0
            return f
        if f.frag_idx >= f.frag_cnt:
            raise FrameError(f"fragment {f.frag_idx} of {f.frag_cnt}")
        key = (f.type, f.step, f.mb, f.chunk)
        parts = self._parts.setdefault(key, {})
        if not parts:
            self._first[key] = time.monotonic()
        parts[f.frag_idx] = f
        if len(parts) < f.frag_cnt:
            return None
        del self._parts[key]
        self.spread_s = time.monotonic() - self._first.pop(key)
        first = parts[0]
        return Frame(first.type, first.codec, first.step, first.mb, first.chunk,
                     b"".join(parts[i].payload for i in range(f.frag_cnt)), first.shape)


def fragments(payload: bytes, n: int) -> list:
    """n contiguous byte ranges of the payload (fewer when it is short)."""
    n = max(1, min(n, len(payload) // 65536 or 1))
    step = (len(payload) + n - 1) // n
    return [payload[i * step:(i + 1) * step] for i in range(n)]
