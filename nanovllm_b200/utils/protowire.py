"""Minimal protobuf wire-format reader (varint, fixed32/64, length-delimited) for ONNX and SentencePiece files.

Only what the loaders need: iterate the (field number, wire type, value) triples of a message.  Length-delimited
values are returned as memoryviews so large tensors are not copied.
"""
from __future__ import annotations

import struct
from typing import Iterator, Tuple, Union

VARINT, FIXED64, LEN, FIXED32 = 0, 1, 2, 5


def read_varint(buf, pos: int) -> Tuple[int, int]:
    result = 0
    shift = 0
    while True:
        if pos >= len(buf):
            raise ValueError("truncated varint")
        b = buf[pos]
        pos += 1
        result |= (b & 0x7F) << shift
        if not b & 0x80:
            return result, pos
        shift += 7
        if shift > 70:
            raise ValueError("varint too long")


def iter_fields(buf) -> Iterator[Tuple[int, int, Union[int, memoryview]]]:
    mv = memoryview(buf)
    pos = 0
    n = len(mv)
    while pos < n:
        key, pos = read_varint(mv, pos)
        field, wt = key >> 3, key & 7
        if wt == VARINT:
            v, pos = read_varint(mv, pos)
        elif wt == FIXED64:
            v = mv[pos:pos + 8]
            pos += 8
        elif wt == LEN:
            ln, pos = read_varint(mv, pos)
            v = mv[pos:pos + ln]
            pos += ln
        elif wt == FIXED32:
            v = mv[pos:pos + 4]
            pos += 4
        else:
            raise ValueError(f"unsupported wire type {wt}")
        yield field, wt, v


def as_float(v) -> float:
    return struct.unpack("<f", bytes(v))[0]


def as_str(v) -> str:
    return bytes(v).decode("utf-8", errors="replace")


def signed64(v: int) -> int:
    return v - (1 << 64) if v >= (1 << 63) else v


def packed_varints(v) -> list:
    out = []
    pos = 0
    while pos < len(v):
        x, pos = read_varint(v, pos)
        out.append(signed64(x))
    return out
