"""Lossless wire codecs of the TCP data plane (host side, native C++).

Reference: src/wantrain/codec/planes.py, fp8_planes.py, f32_planes.py. The
payload layouts are the reference's (so either side decodes the other's
frames; the entropy coder is zlib, which the reference's decoder also
accepts); the byte shuffling and compression run in the `_wire` extension,
planes compressed on parallel threads with the interpreter lock released.

- planes: any dtype, exact bytes split into byte planes (most significant
  first) and compressed; one-byte dtypes go as one interleaved blob.
- e4m3_b128 / e5m2_b128 (this engine's fp8 boundaries): the fp8 codes and
  their fp32 1x128 block scales in one payload (wire dtype ids 34 / 35).
- fp8_planes: e4m3 codes split into sign+exponent / mantissa nibble planes.
- f32_planes: fp32 bytes in plane-major order, one compressed blob.

No codec quantizes: decode returns the exact bytes that were encoded.
"""

from __future__ import annotations

import importlib

import torch

# wire dtype ids (append only; the reference's ids 0-5, scaled fp8 32-33)
DT = {0: torch.float32, 1: torch.bfloat16, 2: torch.float16, 3: torch.float8_e4m3fn,
      4: torch.float8_e5m2, 5: torch.int64}
ID = {v: k for k, v in DT.items()}
E4M3_B128_ID = 34
E5M2_B128_ID = 35
Q8_B128 = {E4M3_B128_ID: torch.float8_e4m3fn, E5M2_B128_ID: torch.float8_e5m2}
_Q8_B128_ID = {v: k for k, v in Q8_B128.items()}

_IVIEW = {1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}


def wire():
    """The native module; raises ImportError with the build command if absent."""
    try:
        return importlib.import_module("elysium_wan_b200._wire")
    except ImportError as e:
        raise ImportError("elysium_wan_b200._wire is not built: run "
                          "`python setup.py build_ext --inplace`") from e


def _bytes_of(t: torch.Tensor) -> memoryview:
    t = t.detach().cpu().contiguous()
    return memoryview(t.view(torch.uint8).reshape(-1).numpy())


def _tensor_of(raw: bytes, dtype, shape) -> torch.Tensor:
    if not raw:
        return torch.empty(shape, dtype=dtype)
    return torch.frombuffer(bytearray(raw), dtype=torch.uint8).view(dtype).reshape(shape).clone()


def planes_encode(t: torch.Tensor, level: int = 1) -> tuple[bytes, tuple]:
    if t.dtype not in ID:
        raise ValueError(f"no wire encoding for dtype {t.dtype}")
    return wire().planes_encode(_bytes_of(t), t.element_size(), ID[t.dtype], level), tuple(t.shape)


def planes_decode(payload: bytes, shape) -> torch.Tensor:
    did = payload[0]
    if did in Q8_B128:
        raise ValueError("an fp8 b128 payload decodes with q8_b128_decode")
    dtype = DT[did]
    esz = torch.empty(0, dtype=dtype).element_size()
    _, _, raw = wire().planes_decode(payload, esz)
    return _tensor_of(raw, dtype, shape)


def q8_b128_encode(codes: torch.Tensor, scales: torch.Tensor, level: int = 1):
    """(fp8 codes [T, d] (e4m3 or e5m2), fp32 scales [T, d / 128]) ->
    (payload, shape of codes); the payload's dtype id names the format."""
    return (wire().pair_encode(_bytes_of(codes), _bytes_of(scales.float()), 4,
                               _Q8_B128_ID[codes.dtype], level), tuple(codes.shape))


def q8_b128_decode(payload: bytes, shape):
    did, a, b = wire().pair_decode(payload, 4)
    codes = _tensor_of(a, Q8_B128[did], shape)
    scales = _tensor_of(b, torch.float32, (shape[0], shape[1] // 128))
    return codes, scales


e4m3_b128_encode = q8_b128_encode
e4m3_b128_decode = q8_b128_decode


def fp8_planes_encode(t: torch.Tensor, level: int = 1) -> tuple[bytes, tuple]:
    """Exactly e4m3-representable values -> nibble-plane payload (refuses
    anything an e4m3 round trip would change: the wire never quantizes)."""
    t = t.detach().cpu().contiguous()
    f8 = t if t.dtype == torch.float8_e4m3fn else t.to(torch.float8_e4m3fn)
    if t.dtype != torch.float8_e4m3fn and not torch.equal(f8.to(t.dtype), t):
        raise ValueError("boundary is not e4m3-representable: recipe mismatch")
    return wire().fp8_planes_encode(_bytes_of(f8), level), tuple(t.shape)


def fp8_planes_decode(payload: bytes, shape) -> torch.Tensor:
    raw = wire().fp8_planes_decode(payload)
    return _tensor_of(raw, torch.float8_e4m3fn, shape).to(torch.float32)


def f32_planes_encode(t: torch.Tensor, level: int = 1) -> tuple[bytes, tuple]:
    if t.dtype != torch.float32:
        raise ValueError("f32_planes carries fp32 only")
    return wire().f32_planes_encode(_bytes_of(t), level), tuple(t.shape)


def f32_planes_decode(payload: bytes, shape) -> torch.Tensor:
    return _tensor_of(wire().f32_planes_decode(payload), torch.float32, shape)
