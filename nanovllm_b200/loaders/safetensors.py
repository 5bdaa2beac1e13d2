"""Safetensors reader / writer (format: 8-byte little-endian header length, JSON header, raw payload).

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/llmcontainer/SafetensorsReader.java:27-317
and SafetensorsTransport.java:26-210 (header cap, F32/F16/BF16/F64 payloads, sorted shards, positioned reads).
Here the payload is memory-mapped and exposed as torch tensors without copying; a multi-file checkpoint is
opened through ``model.safetensors.index.json`` or by globbing ``*.safetensors`` (sorted).  The writer is used
to produce random-init checkpoints for tests and benchmarks.
"""
from __future__ import annotations

import glob
import json
import mmap
import os
import struct
from typing import Dict, Iterator, List, Optional, Tuple

import numpy as np
import warnings

import torch

from ..exceptions import ModelLoadException
from ..utils.limits import ResourceLimits

_DTYPES = {
    "F64": torch.float64, "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16,
    "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8,
    "BOOL": torch.bool, "F8_E4M3": torch.float8_e4m3fn, "F8_E5M2": torch.float8_e5m2,
}
_NAMES = {v: k for k, v in _DTYPES.items()}


class SafetensorsFile:
    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        size = os.fstat(self._f.fileno()).st_size
        if size < 8:
            raise ModelLoadException(f"{path}: too small for a safetensors file")
        (hlen,) = struct.unpack("<Q", self._f.read(8))
        if hlen > ResourceLimits.SAFETENSORS_HEADER_BYTES or 8 + hlen > size:
            raise ModelLoadException(f"{path}: header length {hlen} exceeds limits")
        try:
            header = json.loads(self._f.read(hlen).decode("utf-8"))
        except Exception as e:
            raise ModelLoadException(f"{path}: bad safetensors header: {e}") from e
        self.metadata = header.pop("__metadata__", {}) or {}
        self.entries: Dict[str, dict] = header
        self.data_start = 8 + hlen
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ) if size > 0 else None
        for name, e in self.entries.items():
            b, en = e["data_offsets"]
            if en < b or self.data_start + en > size:
                raise ModelLoadException(f"{path}: tensor {name} outside the payload")

    def keys(self) -> List[str]:
        return list(self.entries.keys())

    def dtype_name(self, name: str) -> str:
        return self.entries[name]["dtype"]

    def shape(self, name: str) -> Tuple[int, ...]:
        return tuple(self.entries[name]["shape"])

    def raw(self, name: str) -> memoryview:
        e = self.entries[name]
        b, en = e["data_offsets"]
        return memoryview(self._mm)[self.data_start + b:self.data_start + en]

    def get(self, name: str) -> torch.Tensor:
        e = self.entries[name]
        dt = e["dtype"]
        if dt not in _DTYPES:
            raise ModelLoadException(f"{self.path}: unsupported dtype {dt} for {name}")
        buf = self.raw(name)
        shape = tuple(e["shape"])
        if len(buf) == 0:
            return torch.empty(shape, dtype=_DTYPES[dt])
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")  # read-only mapping: tensors are never written
            t = torch.frombuffer(buf, dtype=_DTYPES[dt])
        return t.reshape(shape)

    def close(self):
        try:
            if self._mm is not None:
                self._mm.close()
        except BufferError:
            pass  # tensors still reference the mapping; it closes when they are freed
        self._f.close()


class SafetensorsCheckpoint:
    """All shards of a checkpoint folder (or a single file) behind one name -> tensor interface."""

    def __init__(self, path: str):
        if os.path.isdir(path):
            idx = os.path.join(path, "model.safetensors.index.json")
            if os.path.exists(idx):
                with open(idx) as f:
                    wm = json.load(f).get("weight_map", {})
                files = sorted(set(os.path.join(path, v) for v in wm.values()))
            else:
                files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
        else:
            files = [path]
        if not files:
            raise ModelLoadException(f"no .safetensors files under {path}")
        self.files = [SafetensorsFile(p) for p in files]
        self.where: Dict[str, SafetensorsFile] = {}
        for f in self.files:
            for k in f.keys():
                self.where[k] = f

    def keys(self) -> List[str]:
        return list(self.where.keys())

    def __contains__(self, k):
        return k in self.where

    def get(self, name: str) -> torch.Tensor:
        return self.where[name].get(name)

    def dtype_name(self, name: str) -> str:
        return self.where[name].dtype_name(name)

    def shape(self, name: str):
        return self.where[name].shape(name)

    def raw(self, name: str) -> memoryview:
        return self.where[name].raw(name)

    def tensors(self) -> Dict[str, torch.Tensor]:
        return {k: self.get(k) for k in self.keys()}

    def close(self):
        for f in self.files:
            f.close()


def save_file(tensors: Dict[str, torch.Tensor], path: str, metadata: Optional[dict] = None) -> None:
    header = {}
    offset = 0
    blobs = []
    for name in sorted(tensors):
        t = tensors[name].detach().contiguous().cpu()
        if t.dtype not in _NAMES:
            raise ValueError(f"cannot store dtype {t.dtype}")
        if t.dtype == torch.bfloat16:
            data = t.view(torch.int16).numpy().tobytes()
        elif t.dtype in (torch.float8_e4m3fn, torch.float8_e5m2):
            data = t.view(torch.uint8).numpy().tobytes()
        else:
            data = t.numpy().tobytes()
        header[name] = {"dtype": _NAMES[t.dtype], "shape": list(t.shape), "data_offsets": [offset, offset + len(data)]}
        offset += len(data)
        blobs.append(data)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode("utf-8")
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
