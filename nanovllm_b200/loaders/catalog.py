"""Metadata-only view of a checkpoint container, for binding a model before any tensor payload is read.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/llmcontainer/ContainerCatalog.java:25-124
(metadata + tensor names + source, consumed by the architecture processors' ``bind``) and the binding tests
(T/models/llmarch/ModelBindingTest.java:60-129: synthetic GGUF / HF / ONNX catalogs bind without payloads).

``ContainerCatalog.bind(path)`` parses only headers: the GGUF key/value metadata and tensor infos, every
safetensors shard's JSON header, or the ONNX graph's initializer records (names, dims, types; the raw data is
never decoded).  It resolves the architecture with the same rules as the loader (``model_support``), builds the
``HfConfig``, and can check the tensor inventory against the architecture's parameter schema (``missing``), so
a wrong or incomplete checkpoint is rejected before gigabytes are read.
"""
from __future__ import annotations

import os
import re
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

from ..config import HfConfig
from ..exceptions import ModelLoadException
from . import model_support as MS


@dataclass(frozen=True)
class TensorEntry:
    name: str          # as the model graph consumes it (GGUF qwen3 names mapped to Hugging Face names)
    shape: Tuple[int, ...]
    dtype: str         # e.g. "BF16", "F32", a GGML type name ("Q4_K"), or "onnx:<data_type>"


@dataclass
class ContainerCatalog:
    container: str                      # "gguf" | "safetensors" | "onnx"
    source: str                         # file or folder
    architecture: str                   # model_support architecture id
    hf: HfConfig
    metadata: Dict[str, object] = field(default_factory=dict)
    tensors: Dict[str, TensorEntry] = field(default_factory=dict)

    # ------------------------------------------------------------------ queries
    def names(self) -> List[str]:
        return sorted(self.tensors)

    def has(self, name: str) -> bool:
        return name in self.tensors

    def shape(self, name: str) -> Tuple[int, ...]:
        return self.tensors[name].shape

    def expected(self) -> List[Tuple[str, tuple]]:
        """(name, shape) the architecture's graph consumes, for the schemas this package declares."""
        hf = self.hf
        a = self.architecture
        if a in (MS.QWEN3, MS.LLAMA):
            from ..models.qwen3 import param_shapes
            return param_shapes(hf, qk_norm=(a == MS.QWEN3))
        if a == MS.GEMMA3:
            from ..models.gemma3 import param_shapes
            return param_shapes(hf)
        if a == MS.LFM2:
            from ..models.lfm2 import param_shapes
            return param_shapes(hf)
        if a == MS.BERT:
            from ..models.bert import param_shapes
            return param_shapes(hf)
        return []

    def missing(self) -> List[str]:
        """Expected tensors the container lacks (a tied LM head, absent q/k norms of a biased attention and
        optional BERT token types are not required)."""
        have = set(self.tensors)
        out = []
        for name, _ in self.expected():
            if name in have:
                continue
            if name == "lm_head.weight" or name.endswith("token_types.weight"):
                continue
            if name in ("output.weight",):
                continue
            out.append(name)
        return out

    def mismatched(self) -> List[Tuple[str, tuple, tuple]]:
        """(name, expected shape, catalog shape) of tensors present with another shape."""
        out = []
        for name, shape in self.expected():
            e = self.tensors.get(name)
            if e is not None and tuple(e.shape) != tuple(shape):
                out.append((name, tuple(shape), tuple(e.shape)))
        return out

    def require_complete(self) -> "ContainerCatalog":
        miss, bad = self.missing(), self.mismatched()
        if miss or bad:
            raise ModelLoadException(f"{self.source}: checkpoint does not match the {self.architecture} schema: "
                                     f"missing {miss[:5]}{'...' if len(miss) > 5 else ''}, "
                                     f"shape mismatches {bad[:3]}")
        return self

    # ------------------------------------------------------------------ bind
    @staticmethod
    def bind(path) -> "ContainerCatalog":
        path = os.fspath(path)
        if os.path.isfile(path):
            with open(path, "rb") as f:
                magic = f.read(4)
            if magic == b"GGUF":
                return _bind_gguf(path)
            raise ModelLoadException(f"{path}: not a GGUF file (single-file containers are GGUF)")
        if os.path.isdir(path):
            return _bind_folder(path)
        raise ModelLoadException(f"{path}: no such model file or folder")


def _bind_gguf(path: str) -> ContainerCatalog:
    from .gguf import GgufFile
    from .gguf_configs import hf_config_from_gguf, hf_name_for_qwen3
    g = GgufFile(path)
    try:
        sel = MS.resolve_gguf(g.architecture)
        MS.check_source(sel, MS.SRC_GGUF, g.architecture, [])
        hf = hf_config_from_gguf(g.metadata, sel.architecture)
        tensors: Dict[str, TensorEntry] = {}
        for name, info in g.tensors.items():
            target = hf_name_for_qwen3(name) if sel.architecture == MS.QWEN3 else name
            if target is None:
                continue
            tensors[target] = TensorEntry(target, tuple(info.shape), info.type_name)
        if sel.architecture == MS.QWEN3 and "lm_head.weight" not in tensors:
            hf.tie_word_embeddings = True
        return ContainerCatalog("gguf", path, sel.architecture, hf, dict(g.metadata), tensors)
    finally:
        g.close()


def _bind_folder(d: str) -> ContainerCatalog:
    cfg = os.path.join(d, "config.json")
    if not os.path.isfile(cfg):
        raise ModelLoadException(f"{d}: no config.json")
    hf = HfConfig.load(cfg)
    files = sorted(os.listdir(d))
    shards = [os.path.join(d, f) for f in files if f.endswith(".safetensors")]
    tensors: Dict[str, TensorEntry] = {}
    if shards:
        from .safetensors import SafetensorsFile
        sel = MS.require(hf, MS.SRC_HF_SAFETENSORS)
        for p in shards:
            sf = SafetensorsFile(p)
            try:
                for k in sf.keys():
                    tensors[k] = TensorEntry(k, tuple(sf.shape(k)), sf.dtype_name(k))
            finally:
                sf.close()
        container = "safetensors"
    else:
        from .onnx import initializer_infos, normalize_bert_name, normalize_chat_name, select_file
        onnx_file = select_file(d)
        if onnx_file is None:
            raise ModelLoadException(f"{d}: no *.safetensors or loadable *.onnx weights")
        sel = MS.require(hf, MS.SRC_ONNX)
        norm = normalize_bert_name if sel.architecture == MS.BERT else normalize_chat_name
        for k, (shape, dt) in initializer_infos(onnx_file).items():
            n = norm(k)
            tensors[n] = TensorEntry(n, tuple(shape), f"onnx:{dt}")
        container = "onnx"
    if hf.tie_word_embeddings is False and "lm_head.weight" not in tensors and sel.architecture != MS.BERT:
        hf.tie_word_embeddings = True
    import json
    with open(cfg, "r", encoding="utf-8") as f:
        meta = json.load(f)
    return ContainerCatalog(container, d, sel.architecture, hf, meta, tensors)
