"""A GGUF v3 writer for the tests: the byte layout of the reference's fixture
builder (tests/gguf_builder.py in the reference), restated so that GGUF inputs
can be made without the reference present.

Layout: "GGUF", u32 version 3, u64 tensor count, u64 metadata count; metadata
entries (u64-length key, u32 value type, value), general.architecture and
general.alignment first; the tensor directory (name, u32 n_dims, u64 dims,
u32 GGML type, u64 offset relative to the data start, each payload starting on
the alignment); zero padding to the alignment; the payloads, each padded to
the alignment.  Value types follow the builder's inference: bool -> BOOL,
non-negative int -> UINT32 (UINT64 above 2^32 - 1), negative int -> INT32
(INT64 below -2^31), float -> FLOAT32, str -> STRING.
tests/golden/make_gguf_digests.py records the SHA-256 of the reference
builder's output for the tiny goldens; tests/test_gguf.py checks that this
writer produces the same bytes.
"""
from __future__ import annotations

import struct

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_PACK = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", U64: "<Q", I64: "<q",
         F64: "<d"}


def _string(s: str) -> bytes:
    raw = s.encode("utf-8")
    return struct.pack("<Q", len(raw)) + raw


def _kind(v) -> int:
    if isinstance(v, bool):
        return BOOL
    if isinstance(v, int):
        if v < 0:
            return I32 if v >= -(2 ** 31) else I64
        return U32 if v <= 0xFFFFFFFF else U64
    if isinstance(v, float):
        return F32
    if isinstance(v, str):
        return STRING
    raise TypeError(f"unsupported metadata value {v!r}")


def encode_value(v, kind: int | None = None) -> tuple[int, bytes]:
    if isinstance(v, (list, tuple)):
        et = kind if kind is not None else _kind(v[0])
        return ARRAY, struct.pack("<IQ", et, len(v)) + b"".join(encode_value(x, et)[1] for x in v)
    k = kind if kind is not None else _kind(v)
    if k == STRING:
        return k, _string(str(v))
    if k == BOOL:
        return k, struct.pack("<B", 1 if v else 0)
    return k, struct.pack(_PACK[k], v)


def gguf_bytes(architecture: str, metadata: dict, tensors: list[tuple[str, tuple[int, ...], int, bytes]],
               alignment: int = 32, version: int = 3) -> bytes:
    """The whole file: metadata after general.architecture / general.alignment,
    tensors in the given order."""
    entries = [("general.architecture", architecture), ("general.alignment", alignment), *metadata.items()]
    meta = b""
    for key, value in entries:
        k, raw = encode_value(value)
        meta += _string(key) + struct.pack("<I", k) + raw
    header = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(entries))
    directory, offset, offsets = b"", 0, []
    for name, dims, ggml_type, payload in tensors:
        offsets.append(offset)
        directory += _string(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        directory += struct.pack("<IQ", ggml_type, offset)
        offset += len(payload)
        offset += (-offset) % alignment
    prefix = bytearray(header + meta + directory)
    prefix += b"\0" * ((-len(prefix)) % alignment)
    body = bytearray()
    for (_, _, _, payload), off in zip(tensors, offsets):
        body += b"\0" * (off - len(body))
        body += payload
    body += b"\0" * ((-len(body)) % alignment)
    return bytes(prefix + body)
