"""GGUF v2/v3 container: reader (memory-mapped, packed tensors stay packed) and writer.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/llmcontainer/GgufReader.java:28-440 --
magic / version (2, 3) / counts, typed key-value metadata, tensor infos, ``general.alignment`` (default 32),
dims reversed to the HF ``[out, in]`` order, ``getTensor`` dequantises and ``getPackedWeight`` keeps the blocks.
String lengths and dimension counts are capped by ResourceLimits.  The writer produces GGUF checkpoints for tests
and random-init benchmark models (it packs already-quantised blocks; ``quantize_q8_0`` / ``pack_random_blocks``
help produce them).
"""
from __future__ import annotations

import mmap
import os
import math
import struct
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Tuple

import numpy as np
import warnings

import torch

from ..exceptions import ModelLoadException
from ..utils.limits import ResourceLimits
from .dequant import GGML_TYPES, block_info, dequantize, packed_nbytes, type_name

GGUF_MAGIC = b"GGUF"
# value types
T_UINT8, T_INT8, T_UINT16, T_INT16, T_UINT32, T_INT32, T_FLOAT32, T_BOOL, T_STRING, T_ARRAY, T_UINT64, T_INT64, \
    T_FLOAT64 = range(13)
_SCALAR = {T_UINT8: "<B", T_INT8: "<b", T_UINT16: "<H", T_INT16: "<h", T_UINT32: "<I", T_INT32: "<i",
           T_FLOAT32: "<f", T_BOOL: "<?", T_UINT64: "<Q", T_INT64: "<q", T_FLOAT64: "<d"}


@dataclass
class GgufTensorInfo:
    name: str
    shape: Tuple[int, ...]   # HF order ([out, in] for matrices)
    ggml_type: int
    offset: int              # absolute file offset
    nbytes: int

    @property
    def numel(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n

    @property
    def type_name(self) -> str:
        return type_name(self.ggml_type)


class GgufFile:
    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        size = os.fstat(self._f.fileno()).st_size
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self._pos = 0
        if self._read(4) != GGUF_MAGIC:
            raise ModelLoadException(f"{path}: not a GGUF file")
        (self.version,) = self._unpack("<I")
        if self.version not in (2, 3):
            raise ModelLoadException(f"{path}: unsupported GGUF version {self.version}")
        (n_tensors,) = self._unpack("<Q")
        (n_kv,) = self._unpack("<Q")
        self.metadata: Dict[str, Any] = {}
        for _ in range(n_kv):
            key = self._string()
            (vt,) = self._unpack("<I")
            self.metadata[key] = self._value(vt)
        infos = []
        for _ in range(n_tensors):
            name = self._string()
            (nd,) = self._unpack("<I")
            if nd > ResourceLimits.MAX_DIMS:
                raise ModelLoadException(f"{path}: tensor {name} has {nd} dims")
            dims = [self._unpack("<Q")[0] for _ in range(nd)]
            (tt,) = self._unpack("<I")
            (off,) = self._unpack("<Q")
            infos.append((name, tuple(reversed(dims)), tt, off))
        align = int(self.metadata.get("general.alignment", 32))
        self.data_start = (self._pos + align - 1) // align * align
        self.tensors: Dict[str, GgufTensorInfo] = {}
        for name, shape, tt, off in infos:
            if tt not in GGML_TYPES:
                raise ModelLoadException(f"{path}: tensor {name} has unsupported type {tt}")
            numel = int(np.prod(shape)) if shape else 1
            nb = packed_nbytes(tt, numel)
            abs_off = self.data_start + off
            if abs_off + nb > size:
                raise ModelLoadException(f"{path}: tensor {name} extends past the end of the file")
            self.tensors[name] = GgufTensorInfo(name, shape, tt, abs_off, nb)

    # ------------------------------------------------------------------ primitives
    def _read(self, n: int) -> bytes:
        b = self._mm[self._pos:self._pos + n]
        if len(b) != n:
            raise ModelLoadException(f"{self.path}: truncated header")
        self._pos += n
        return b

    def _unpack(self, fmt: str):
        return struct.unpack(fmt, self._read(struct.calcsize(fmt)))

    def _string(self) -> str:
        (n,) = self._unpack("<Q")
        if n > ResourceLimits.GGUF_MAX_STRING:
            raise ModelLoadException(f"{self.path}: string of {n} bytes exceeds the limit")
        return self._read(n).decode("utf-8", errors="replace")

    def _value(self, vt: int):
        if vt in _SCALAR:
            return self._unpack(_SCALAR[vt])[0]
        if vt == T_STRING:
            return self._string()
        if vt == T_ARRAY:
            (et,) = self._unpack("<I")
            (n,) = self._unpack("<Q")
            if et in _SCALAR and et != T_BOOL:
                fmt = _SCALAR[et]
                sz = struct.calcsize(fmt)
                arr = np.frombuffer(self._read(sz * n), dtype=np.dtype(fmt))
                return arr.tolist()
            return [self._value(et) for _ in range(n)]
        raise ModelLoadException(f"{self.path}: unknown metadata value type {vt}")

    # ------------------------------------------------------------------ access
    @property
    def architecture(self) -> Optional[str]:
        return self.metadata.get("general.architecture")

    def keys(self) -> List[str]:
        return list(self.tensors.keys())

    def raw(self, name: str) -> memoryview:
        t = self.tensors[name]
        return memoryview(self._mm)[t.offset:t.offset + t.nbytes]

    def packed(self, name: str) -> torch.Tensor:
        """Packed bytes as a uint8 tensor (zero-copy view of the mapping)."""
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")  # read-only mapping: tensors are never written
            return torch.frombuffer(self.raw(name), dtype=torch.uint8)

    def get(self, name: str, dtype=torch.float32, device="cpu") -> torch.Tensor:
        t = self.tensors[name]
        return dequantize(self.packed(name), t.ggml_type, t.numel, device=device, dtype=dtype).reshape(t.shape)

    def close(self):
        try:
            self._mm.close()
        except BufferError:
            pass
        self._f.close()


# ----------------------------------------------------------------------------------------------- writer
def _pack_value(v) -> Tuple[int, bytes]:
    if isinstance(v, bool):
        return T_BOOL, struct.pack("<?", v)
    if isinstance(v, int):
        if -2 ** 31 <= v < 2 ** 31:
            return T_INT32, struct.pack("<i", v)
        return T_INT64, struct.pack("<q", v)
    if isinstance(v, float):
        return T_FLOAT32, struct.pack("<f", v)
    if isinstance(v, str):
        b = v.encode("utf-8")
        return T_STRING, struct.pack("<Q", len(b)) + b
    if isinstance(v, (list, tuple)):
        if not v:
            return T_ARRAY, struct.pack("<IQ", T_INT32, 0)
        et, _ = _pack_value(v[0])
        body = b"".join(_pack_value(x)[1] for x in v)
        return T_ARRAY, struct.pack("<IQ", et, len(v)) + body
    raise TypeError(f"cannot store {type(v)} in GGUF metadata")


def write_gguf(path: str, metadata: Dict[str, Any], tensors: Dict[str, Tuple[int, Tuple[int, ...], bytes]],
               alignment: int = 32) -> None:
    """tensors: name -> (ggml type, HF-order shape, packed bytes)."""
    meta = dict(metadata)
    meta.setdefault("general.alignment", alignment)
    out = bytearray()
    out += GGUF_MAGIC + struct.pack("<IQQ", 3, len(tensors), len(meta))
    for k, v in meta.items():
        kb = k.encode()
        vt, vb = _pack_value(v)
        out += struct.pack("<Q", len(kb)) + kb + struct.pack("<I", vt) + vb
    offset = 0
    order = list(tensors.keys())
    offsets = {}
    for name in order:
        tt, shape, data = tensors[name]
        offsets[name] = offset
        offset += (len(data) + alignment - 1) // alignment * alignment
    for name in order:
        tt, shape, data = tensors[name]
        nb = name.encode()
        dims = list(reversed(shape))
        out += struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(dims))
        out += b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", tt, offsets[name])
    pad = (-len(out)) % alignment
    out += b"\0" * pad
    with open(path, "wb") as f:
        f.write(out)
        for name in order:
            data = tensors[name][2]
            f.write(data)
            f.write(b"\0" * ((-len(data)) % alignment))


def quantize_q8_0(x: torch.Tensor) -> bytes:
    """fp -> Q8_0 blocks (d = max|x| / 127 per 32 values, round-to-nearest)."""
    v = x.float().reshape(-1, 32)
    amax = v.abs().amax(1, keepdim=True)
    d = amax / 127.0
    q = torch.where(d > 0, torch.round(v / d.clamp_min(1e-30)), torch.zeros_like(v)).clamp(-127, 127).to(torch.int8)
    d16 = d.to(torch.float16)
    blocks = torch.cat([d16.view(torch.uint8).reshape(-1, 2), q.view(torch.uint8)], 1)
    return blocks.contiguous().numpy().tobytes()


def f16_bytes(x: torch.Tensor) -> bytes:
    return x.to(torch.float16).contiguous().view(torch.uint8).numpy().tobytes()


def f32_bytes(x: torch.Tensor) -> bytes:
    return x.to(torch.float32).contiguous().numpy().tobytes()


def pack_random_blocks(ggml_type: int, shape: Tuple[int, ...], seed: int, std: float = 0.02) -> bytes:
    """Random packed blocks whose dequantised values have roughly N(0, std) magnitude: random codes with the
    block scales chosen for that spread (random-init stand-in for a quantised checkpoint)."""
    be, bb = block_info(ggml_type)
    numel = int(np.prod(shape))
    nblocks = numel // be
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
    name = type_name(ggml_type)
    f16 = lambda v: np.frombuffer(np.full(nblocks, v, dtype=np.float16).tobytes(), dtype=np.uint8).reshape(nblocks, 2)
    # 6-bit scale / min of 32 for all 8 sub-blocks of a K-quant block: bytes 0-7 = 0xA0, bytes 8-11 = 0
    k_scales = np.array([0xA0] * 8 + [0] * 4, dtype=np.uint8)
    if name == "Q4_K":  # d, dmin, 12 scale bytes, 128 qs; codes 0..15 (std 4.6) centred by the min
        d = std / (32 * 4.6)
        raw[:, 0:2] = f16(d)
        raw[:, 2:4] = f16(d * 7.5)
        raw[:, 4:16] = k_scales
    elif name == "Q5_K":  # codes 0..31 (std 9.2)
        d = std / (32 * 9.2)
        raw[:, 0:2] = f16(d)
        raw[:, 2:4] = f16(d * 15.5)
        raw[:, 4:16] = k_scales
    elif name == "Q6_K":  # 128 ql, 64 qh, 16 int8 scales, d; codes -32..31 (std 18.5)
        raw[:, 192:208] = 16
        raw[:, 208:210] = f16(std / (16 * 18.5))
    elif name == "Q8_0":  # int8 codes (std 74)
        raw[:, 0:2] = f16(std / 74.0)
    elif name == "Q4_0":  # codes -8..7 (std 4.6)
        raw[:, 0:2] = f16(std / 4.6)
    elif name == "Q4_1":  # d * code + m, codes 0..15 centred by m
        raw[:, 0:2] = f16(std / 4.6)
        raw[:, 2:4] = f16(-7.5 * std / 4.6)
    elif name == "IQ4_NL":  # non-linear grid, spread ~66
        raw[:, 0:2] = f16(std / 66.0)
    elif name == "IQ4_XS":  # every 6-bit sub-block scale = 1 (stored +32): low nibbles 1, high bits 2
        raw[:, 0:2] = f16(std / 66.0)
        raw[:, 2:4] = 0xAA
        raw[:, 4:8] = 0x11
    elif name == "MXFP4":  # doubled e2m1 grid (spread ~5.7) times 2^(e - 128)
        raw[:, 0] = 128 + int(round(math.log2(std / 5.7)))
    elif name == "NVFP4":  # four ue4m3 sub-scales of 4 * 2^-10
        raw[:, 0:4] = 0x04
    elif name == "Q5_0":  # codes -16..15 (std 9.2)
        raw[:, 0:2] = f16(std / 9.2)
    elif name == "Q5_1":  # d * code + m, codes 0..31 centred by m
        raw[:, 0:2] = f16(std / 9.2)
        raw[:, 2:4] = f16(-15.5 * std / 9.2)
    elif name == "Q2_K":  # 16 scale bytes (scale 1, min 1), 64 qs, d, dmin; codes 0..3 (std 1.1) centred by dmin
        raw[:, 0:16] = 0x11
        raw[:, 80:82] = f16(std / 1.1)
        raw[:, 82:84] = f16(1.5 * std / 1.1)
    elif name == "Q3_K":  # 32 hmask, 64 qs, 6-bit scales all 1 (+32 bias: low nibbles 1, high pairs 2), d
        raw[:, 96:104] = 0x11
        raw[:, 104:108] = 0xAA
        raw[:, 108:110] = f16(std / 2.3)
    elif name == "TQ1_0":  # trits -1..1 (std 0.82)
        raw[:, 52:54] = f16(std / 0.82)
    elif name == "TQ2_0":  # codes -1..2 (std 1.1)
        raw[:, 64:66] = f16(std / 1.1)
    else:
        raise ValueError(f"random packing not provided for {name}")
    return raw.tobytes()
