"""ONNX "Tier A" loader: weights from graph initializers only (no graph execution).

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/llmcontainer/OnnxProtoReader.java:26-438,
OnnxTransport.java:34-269, OnnxWeightReader.java, OnnxDataTypes.java:15-168 and llmarch/OnnxWeightNames.java:20-114:
* file choice: ``model.onnx`` / ``model_fp16.onnx`` / ``decoder_model_merged.onnx`` in the folder or its ``onnx/``
  sub-folder, else the first sorted ``*.onnx``; quantised exports (``_q4``, ``_int8``, ``_uint8``, ``_bnb4``,
  ``_quantized``) and ``with_past`` files are never picked;
* raw data in field 9 or typed arrays, external data (field 13) read from side-car files next to the model;
* FLOAT / FLOAT16 / BFLOAT16 / DOUBLE initializers of rank >= 1 are weights; int / bool / string / complex
  constants are skipped; float8 / int4 / fp4 weights fail loudly;
* MatMul right-hand operands are stored [in, out] and are transposed to [out, in]; anonymous ``onnx::MatMul_*``
  initializers take their name from the consuming node's path (``/model/layers.0/self_attn/q_proj/MatMul`` ->
  ``model.layers.0.self_attn.q_proj.weight``);
* BERT names are mapped onto the GGUF tensor names the BERT encoder consumes.
"""
from __future__ import annotations

import os
import re
import struct
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from ..exceptions import ModelLoadException
from ..utils import protowire as pw

PREFERRED = ("model.onnx", "model_fp16.onnx", "decoder_model_merged.onnx")
_BAD = ("_q4", "_int8", "_uint8", "_bnb4", "_quantized", "with_past")

FLOAT, UINT8, INT8, UINT16, INT16, INT32, INT64, STRING, BOOL, FLOAT16, DOUBLE, UINT32, UINT64, COMPLEX64, \
    COMPLEX128, BFLOAT16 = range(1, 17)
_LOADABLE = {FLOAT: np.float32, FLOAT16: np.float16, DOUBLE: np.float64, BFLOAT16: None}
_SKIP = {0, UINT8, INT8, UINT16, INT16, INT32, INT64, STRING, BOOL, UINT32, UINT64, COMPLEX64, COMPLEX128}


def is_allowed_name(name: str) -> bool:
    low = name.lower()
    return low.endswith(".onnx") and not any(b in low for b in _BAD)


def select_file(model_dir: str) -> Optional[str]:
    for d in (model_dir, os.path.join(model_dir, "onnx")):
        if not os.path.isdir(d):
            continue
        for n in PREFERRED:
            p = os.path.join(d, n)
            if os.path.isfile(p) and is_allowed_name(n):
                return p
        others = sorted(f for f in os.listdir(d) if os.path.isfile(os.path.join(d, f)) and is_allowed_name(f))
        if others:
            return os.path.join(d, others[0])
    return None


class _Tensor:
    __slots__ = ("name", "dims", "dtype", "raw", "typed", "external")

    def __init__(self):
        self.name = ""
        self.dims: List[int] = []
        self.dtype = 0
        self.raw = None
        self.typed = None
        self.external: Dict[str, str] = {}


def _parse_tensor(buf) -> _Tensor:
    t = _Tensor()
    floats, doubles = [], []
    for f, wt, v in pw.iter_fields(buf):
        if f == 1:
            if wt == pw.LEN:
                t.dims.extend(pw.packed_varints(v))
            else:
                t.dims.append(pw.signed64(v))
        elif f == 2:
            t.dtype = v
        elif f == 4:  # float_data
            if wt == pw.LEN:
                floats.append(np.frombuffer(bytes(v), dtype="<f4"))
            else:
                floats.append(np.array([pw.as_float(v)], dtype=np.float32))
        elif f == 10:  # double_data
            if wt == pw.LEN:
                doubles.append(np.frombuffer(bytes(v), dtype="<f8"))
        elif f == 5 and t.typed is None:  # int32_data (also carries fp16 / bf16 bit patterns)
            t.typed = np.array(pw.packed_varints(v) if wt == pw.LEN else [v], dtype=np.int64)
        elif f == 8:
            t.name = pw.as_str(v)
        elif f == 9:
            t.raw = v
        elif f == 13:
            k = val = None
            for f2, _, v2 in pw.iter_fields(v):
                if f2 == 1:
                    k = pw.as_str(v2)
                elif f2 == 2:
                    val = pw.as_str(v2)
            if k is not None:
                t.external[k] = val
    if floats:
        t.typed = np.concatenate(floats)
    elif doubles:
        t.typed = np.concatenate(doubles)
    return t


def _tensor_to_torch(t: _Tensor, base_dir: str) -> torch.Tensor:
    shape = tuple(int(d) for d in t.dims)
    n = int(np.prod(shape)) if shape else 1
    if t.external:
        loc = t.external.get("location")
        off = int(t.external.get("offset", "0"))
        length = int(t.external.get("length", "0")) or None
        path = os.path.join(base_dir, loc)
        with open(path, "rb") as f:
            f.seek(off)
            raw = f.read(length) if length else f.read()
    elif t.raw is not None:
        raw = bytes(t.raw)
    else:
        raw = None
    if t.dtype == BFLOAT16:
        if raw is not None:
            arr = torch.frombuffer(bytearray(raw), dtype=torch.bfloat16)
        else:
            arr = torch.tensor(t.typed.astype(np.int16), dtype=torch.int16).view(torch.bfloat16)
        return arr[:n].reshape(shape).float()
    np_dt = _LOADABLE[t.dtype]
    if raw is not None:
        arr = np.frombuffer(raw, dtype=np.dtype(np_dt).newbyteorder("<"))
    elif t.dtype == FLOAT16 and t.typed is not None:
        arr = t.typed.astype(np.uint16).view(np.float16)
    elif t.typed is not None:
        arr = t.typed.astype(np_dt)
    else:
        raise ModelLoadException(f"ONNX initializer {t.name!r} has no data")
    return torch.from_numpy(np.array(arr[:n], dtype=np.float32)).reshape(shape)


def _node_weight_name(node_name: str) -> Optional[str]:
    """'/model/layers.0/self_attn/q_proj/MatMul' -> 'model.layers.0.self_attn.q_proj.weight'"""
    parts = [p for p in node_name.strip("/").split("/") if p]
    if len(parts) < 2:
        return None
    return ".".join(parts[:-1]) + ".weight"


def _scan(path: str):
    """(initializer records by name, MatMul B-operand name -> node name): the graph structure only; no tensor
    payload is decoded."""
    with open(path, "rb") as f:
        data = f.read()
    graph = None
    for fnum, wt, v in pw.iter_fields(data):
        if fnum == 7 and wt == pw.LEN:
            graph = v
    if graph is None:
        raise ModelLoadException(f"{path}: no graph in ONNX model")
    inits: Dict[str, _Tensor] = {}
    matmul_b: Dict[str, str] = {}
    for fnum, wt, v in pw.iter_fields(graph):
        if fnum == 5:
            t = _parse_tensor(v)
            if t.name:
                inits[t.name] = t
        elif fnum == 1:
            ins, name, op = [], "", ""
            for f2, _, v2 in pw.iter_fields(v):
                if f2 == 1:
                    ins.append(pw.as_str(v2))
                elif f2 == 3:
                    name = pw.as_str(v2)
                elif f2 == 4:
                    op = pw.as_str(v2)
            if op == "MatMul" and len(ins) >= 2:
                matmul_b[ins[1]] = name
    return inits, matmul_b


def _graph_name(name: str, matmul_b: Dict[str, str]) -> str:
    if name in matmul_b and "onnx::" in name:
        alias = _node_weight_name(matmul_b[name])
        if alias is not None:
            return alias
    return name


def initializer_infos(path: str) -> Dict[str, tuple]:
    """name -> (shape as loaded, ONNX data_type) of every loadable weight, from the graph records alone (MatMul
    operands reported transposed to [out, in]); used to bind a model before reading any payload."""
    inits, matmul_b = _scan(path)
    out: Dict[str, tuple] = {}
    for name, t in inits.items():
        if t.dtype in _LOADABLE and len(t.dims) >= 1:
            dims = tuple(int(d) for d in t.dims)
            if name in matmul_b and len(dims) == 2:
                dims = (dims[1], dims[0])
            out[_graph_name(name, matmul_b)] = (dims, int(t.dtype))
    return out


def read_initializers(path: str) -> Dict[str, torch.Tensor]:
    """All loadable float weights of an ONNX file, MatMul operands transposed to [out, in]."""
    inits, matmul_b = _scan(path)
    base = os.path.dirname(os.path.abspath(path))
    out: Dict[str, torch.Tensor] = {}
    for name, t in inits.items():
        rank = len(t.dims)
        if t.dtype in _LOADABLE and rank >= 1:
            w = _tensor_to_torch(t, base)
            if name in matmul_b:
                w = w.t().contiguous() if w.dim() == 2 else w
            out[_graph_name(name, matmul_b)] = w
        elif t.dtype in _SKIP or rank == 0:
            continue
        else:
            raise ModelLoadException(f"ONNX initializer {name!r} has unsupported data_type {t.dtype}; only "
                                     f"FLOAT / FLOAT16 / BFLOAT16 / DOUBLE weights load")
    return out


# ----------------------------------------------------------------------------------------------- names
_BERT_LAYER = re.compile(r"^encoder\.layer\.(\d+)\.(.+)$")
_BERT_MAP = {
    "attention.self.query.weight": "attn_q.weight", "attention.self.query.bias": "attn_q.bias",
    "attention.self.key.weight": "attn_k.weight", "attention.self.key.bias": "attn_k.bias",
    "attention.self.value.weight": "attn_v.weight", "attention.self.value.bias": "attn_v.bias",
    "attention.output.dense.weight": "attn_output.weight", "attention.output.dense.bias": "attn_output.bias",
    "attention.output.LayerNorm.weight": "attn_output_norm.weight",
    "attention.output.LayerNorm.bias": "attn_output_norm.bias",
    "intermediate.dense.weight": "ffn_up.weight", "intermediate.dense.bias": "ffn_up.bias",
    "output.dense.weight": "ffn_down.weight", "output.dense.bias": "ffn_down.bias",
    "output.LayerNorm.weight": "layer_output_norm.weight", "output.LayerNorm.bias": "layer_output_norm.bias",
}


def _strip(name: str) -> str:
    name = name.strip().lstrip("/")
    if "onnx::" not in name.lower() and (name.startswith("model/") or name.startswith("bert/")):
        name = name.replace("/", ".")
    return name


def normalize_chat_name(name: str) -> str:
    name = _strip(name)
    if name.startswith("model.model."):
        name = name[len("model."):]
    return name


def normalize_bert_name(name: str) -> str:
    name = _strip(name)
    if name.startswith("bert."):
        name = name[5:]
    name = name.replace("LayerNorm.gamma", "LayerNorm.weight").replace("LayerNorm.beta", "LayerNorm.bias")
    fixed = {"embeddings.word_embeddings.weight": "token_embd.weight",
             "embeddings.position_embeddings.weight": "position_embd.weight",
             "embeddings.token_type_embeddings.weight": "token_types.weight",
             "embeddings.LayerNorm.weight": "token_embd_norm.weight",
             "embeddings.LayerNorm.bias": "token_embd_norm.bias"}
    if name in fixed:
        return fixed[name]
    m = _BERT_LAYER.match(name)
    if m and m.group(2) in _BERT_MAP:
        return f"blk.{int(m.group(1))}.{_BERT_MAP[m.group(2)]}"
    return name


# ----------------------------------------------------------------------------------------------- writer (tests)
def _key(field: int, wt: int) -> bytes:
    return _varint(field << 3 | wt)


def _varint(v: int) -> bytes:
    out = bytearray()
    v &= (1 << 64) - 1
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _len_field(field: int, payload: bytes) -> bytes:
    return _key(field, pw.LEN) + _varint(len(payload)) + payload


def write_onnx(path: str, weights: Dict[str, torch.Tensor], matmul: Dict[str, str] = None, fp16: bool = False) -> None:
    """Minimal ONNX file: initializers (+ MatMul nodes that consume ``matmul`` {initializer: node name})."""
    graph = bytearray()
    for node_in, node_name in (matmul or {}).items():
        node = _len_field(1, b"x") + _len_field(1, node_in.encode()) + _len_field(3, node_name.encode()) + \
            _len_field(4, b"MatMul")
        graph += _len_field(1, node)
    for name, w in weights.items():
        arr = w.detach().cpu().numpy().astype(np.float16 if fp16 else np.float32)
        t = _len_field(1, b"".join(_varint(d) for d in arr.shape)) + _key(2, pw.VARINT) + \
            _varint(FLOAT16 if fp16 else FLOAT) + _len_field(8, name.encode()) + _len_field(9, arr.tobytes())
        graph += _len_field(5, t)
    model = _key(1, pw.VARINT) + _varint(8) + _len_field(7, bytes(graph))
    with open(path, "wb") as f:
        f.write(model)
