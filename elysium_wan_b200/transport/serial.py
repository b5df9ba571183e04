"""Safe object codec: a JSON tree plus raw tensor blobs, exact bytes, no pickle.

Reference behaviour: src/wantrain/transport/serial.py:135-170 (`dumps` /
`loads`). Loading never executes code from the bytes: the header is JSON and
every tensor is rebuilt from (dtype, shape, offset, nbytes) over the blob, so
a state file shipped between machines (a checkpoint wave, a logical
checkpoint's extras) cannot carry a payload that runs on load, which an
unpickler could.

Layout:  b"EWBS" | u32 version | u64 header length | header JSON | blobs
The header is the object with every tensor replaced by
{"__t__": index, "dtype", "shape"} and every bytes value by {"__b__": index};
the blob table lists (offset, nbytes) per index, offsets 64-byte aligned.
Supported: dict (str keys), list, tuple, str, int, float (incl. inf / nan),
bool, None, bytes, torch.Tensor (any dense dtype, stored contiguous on CPU).
"""

from __future__ import annotations

import json
import math
import struct

import torch

MAGIC = b"EWBS"
VERSION = 1
_ALIGN = 64

_DTYPES = {str(d).replace("torch.", ""): d for d in (
    torch.float32, torch.float64, torch.float16, torch.bfloat16, torch.int8, torch.uint8,
    torch.int16, torch.int32, torch.int64, torch.bool, torch.float8_e4m3fn, torch.float8_e5m2)}


_RESERVED = {"__t__", "__b__", "__tuple__", "__f__", "__d__"}


def _enc(obj, blobs: list):
    if isinstance(obj, torch.Tensor):
        t = obj.detach().to("cpu").contiguous()
        blobs.append(t.reshape(-1).view(torch.uint8).numpy().tobytes() if t.numel() else b"")
        return {"__t__": len(blobs) - 1, "dtype": str(t.dtype).replace("torch.", ""),
                "shape": list(t.shape)}
    if isinstance(obj, (bytes, bytearray)):
        blobs.append(bytes(obj))
        return {"__b__": len(blobs) - 1}
    if isinstance(obj, dict):
        if not all(isinstance(k, str) for k in obj) or _RESERVED & set(obj):
            # non-string keys (stage indices, ...) and keys that would read as a
            # marker travel as {"__d__": [[key, value], ...]}
            return {"__d__": [[_enc(k, blobs), _enc(v, blobs)] for k, v in obj.items()]}
        return {k: _enc(v, blobs) for k, v in obj.items()}
    if isinstance(obj, tuple):
        return {"__tuple__": [_enc(v, blobs) for v in obj]}
    if isinstance(obj, list):
        return [_enc(v, blobs) for v in obj]
    if isinstance(obj, float) and not math.isfinite(obj):
        return {"__f__": repr(obj)}
    if obj is None or isinstance(obj, (str, int, float, bool)):
        return obj
    raise TypeError(f"serial: cannot encode {type(obj).__name__}")


def dumps(obj) -> bytes:
    blobs: list = []
    tree = _enc(obj, blobs)
    table, off = [], 0
    for b in blobs:
        table.append([off, len(b)])
        off += len(b) + (-len(b)) % _ALIGN
    head = json.dumps({"tree": tree, "blobs": table}, separators=(",", ":")).encode()
    pre = MAGIC + struct.pack("<IQ", VERSION, len(head)) + head
    pad = (-len(pre)) % _ALIGN
    out = bytearray(pre + b"\0" * pad)
    for b in blobs:
        out += b + b"\0" * ((-len(b)) % _ALIGN)
    return bytes(out)


def _dec(node, data: memoryview, base: int, table: list):
    if isinstance(node, list):
        return [_dec(v, data, base, table) for v in node]
    if isinstance(node, dict):
        if "__t__" in node:
            off, n = table[node["__t__"]]
            dt = _DTYPES.get(node["dtype"])
            if dt is None:
                raise ValueError(f"serial: unknown dtype {node['dtype']!r}")
            raw = bytearray(data[base + off: base + off + n])
            flat = torch.frombuffer(raw, dtype=torch.uint8) if n else torch.empty(0, dtype=torch.uint8)
            return flat.view(dt).reshape(node["shape"]).clone()
        if "__b__" in node:
            off, n = table[node["__b__"]]
            return bytes(data[base + off: base + off + n])
        if "__tuple__" in node:
            return tuple(_dec(v, data, base, table) for v in node["__tuple__"])
        if "__f__" in node:
            return float(node["__f__"])
        if "__d__" in node:
            return {_dec(k, data, base, table): _dec(v, data, base, table) for k, v in node["__d__"]}
        return {k: _dec(v, data, base, table) for k, v in node.items()}
    return node


def loads(data: bytes):
    if data[:4] != MAGIC:
        raise ValueError("serial: not an EWBS object")
    ver, hlen = struct.unpack("<IQ", data[4:16])
    if ver != VERSION:
        raise ValueError(f"serial: version {ver} (this build reads {VERSION})")
    head = json.loads(bytes(data[16:16 + hlen]))
    base = 16 + hlen
    base += (-base) % _ALIGN
    return _dec(head["tree"], memoryview(data), base, head["blobs"])


def save(obj, path: str):
    with open(path, "wb") as f:
        f.write(dumps(obj))


def load(path: str):
    with open(path, "rb") as f:
        return loads(f.read())
