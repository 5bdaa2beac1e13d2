"""Model file sources: where the factory reads checkpoint files from.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/{ModelFileSource.java:43,
ModelFileSources.java:30-198, ModelFileId.java:16-54} and internal/ModelFileBundle.java (role ids for config,
tokenizer files, generation config, ONNX, weight index / shards and GGUF; sources over a folder, a single
.gguf file, classpath resources and in-memory streams).

Here a source is anything with ``open(role_or_name) -> Optional[bytes]``, ``names()`` and ``display_name()``:
``PathSource`` (a folder or a single .gguf), ``PackageSource`` (files shipped inside an importable package,
the analogue of classpath resources) and ``BytesSource`` (an in-memory name -> bytes map).  Loaders in this
package memory-map files, so a non-path source is spooled once into a private temporary folder that is
removed when the source is closed (the mapped tensors keep their pages alive until they are freed).
"""
from __future__ import annotations

import enum
import importlib.resources
import os
import shutil
import tempfile
from typing import Dict, Iterable, List, Optional


class ModelFileId(enum.Enum):
    CONFIG = "config.json"
    TOKENIZER = "tokenizer.json"
    TOKENIZER_CONFIG = "tokenizer_config.json"
    TOKENIZER_MODEL = "tokenizer.model"
    GENERATION_CONFIG = "generation_config.json"
    ADDED_TOKENS = "added_tokens.json"
    SPECIAL_TOKENS_MAP = "special_tokens_map.json"
    SAFE_TENSORS_INDEX = "model.safetensors.index.json"
    MODEL_SAFE_TENSORS = "model.safetensors"
    MODEL_ONNX = "model.onnx"
    MODEL_ONNX_FP16 = "model_fp16.onnx"
    GGUF = "model.gguf"

    @property
    def file_name(self) -> str:
        return self.value


def _name(key) -> str:
    return key.file_name if isinstance(key, ModelFileId) else str(key)


class ModelFileSource:
    def open(self, key) -> Optional[bytes]:
        raise NotImplementedError

    def names(self) -> List[str]:
        raise NotImplementedError

    def display_name(self) -> str:
        return type(self).__name__

    def local_path(self) -> str:
        """A filesystem path the loaders can map (a folder, or a .gguf file)."""
        raise NotImplementedError

    def close(self) -> None:
        pass


class PathSource(ModelFileSource):
    def __init__(self, path: str):
        self.path = os.path.abspath(path)
        if not os.path.exists(self.path):
            raise FileNotFoundError(self.path)

    def is_gguf(self) -> bool:
        return os.path.isfile(self.path) and self.path.lower().endswith(".gguf")

    def names(self) -> List[str]:
        if os.path.isfile(self.path):
            return [os.path.basename(self.path)]
        out = []
        for root, _, files in os.walk(self.path):
            for f in files:
                out.append(os.path.relpath(os.path.join(root, f), self.path))
        return sorted(out)

    def open(self, key) -> Optional[bytes]:
        name = _name(key)
        if os.path.isfile(self.path):
            return open(self.path, "rb").read() if (key == ModelFileId.GGUF or name == os.path.basename(self.path)) else None
        p = os.path.join(self.path, name)
        if not os.path.isfile(p) and isinstance(key, ModelFileId) and key in (ModelFileId.MODEL_ONNX, ModelFileId.MODEL_ONNX_FP16):
            p = os.path.join(self.path, "onnx", name)
        return open(p, "rb").read() if os.path.isfile(p) else None

    def display_name(self) -> str:
        return self.path

    def local_path(self) -> str:
        return self.path


class _Spooled(ModelFileSource):
    """Shared spooling of a byte-level source into a private folder for the memory-mapping loaders."""

    _dir: Optional[str] = None

    def local_path(self) -> str:
        if self._dir is None:
            self._dir = tempfile.mkdtemp(prefix="nvb-model-")
            for n in self.names():
                data = self.open(n)
                if data is None:
                    continue
                dst = os.path.join(self._dir, n)
                os.makedirs(os.path.dirname(dst), exist_ok=True)
                with open(dst, "wb") as f:
                    f.write(data)
        ggufs = [n for n in self.names() if n.lower().endswith(".gguf")]
        if len(ggufs) == 1 and not any(n == "config.json" for n in self.names()):
            return os.path.join(self._dir, ggufs[0])
        return self._dir

    def close(self) -> None:
        if self._dir is not None:
            shutil.rmtree(self._dir, ignore_errors=True)
            self._dir = None


class BytesSource(_Spooled):
    def __init__(self, files: Dict[str, bytes], label: str = "memory"):
        self.files = {str(k): bytes(v) for k, v in files.items()}
        self.label = label

    def names(self) -> List[str]:
        return sorted(self.files)

    def open(self, key) -> Optional[bytes]:
        return self.files.get(_name(key))

    def display_name(self) -> str:
        return f"{self.label} ({len(self.files)} files)"


class PackageSource(_Spooled):
    """Files under ``folder`` inside an importable package (``importlib.resources``)."""

    def __init__(self, package: str, folder: str = ""):
        self.package, self.folder = package, folder.strip("/")
        root = importlib.resources.files(package)
        self.root = root.joinpath(self.folder) if self.folder else root
        if not self.root.is_dir():
            raise FileNotFoundError(f"package resource folder not found: {package}/{folder}")

    def names(self) -> List[str]:
        out = []

        def walk(node, prefix):
            for child in node.iterdir():
                if child.is_dir():
                    walk(child, prefix + child.name + "/")
                else:
                    out.append(prefix + child.name)
        walk(self.root, "")
        return sorted(out)

    def open(self, key) -> Optional[bytes]:
        node = self.root
        for part in _name(key).split("/"):
            node = node.joinpath(part)
        return node.read_bytes() if node.is_file() else None

    def display_name(self) -> str:
        return f"package:{self.package}/{self.folder}"


class ModelFileSources:
    @staticmethod
    def from_path(path: str) -> PathSource:
        return PathSource(path)

    @staticmethod
    def from_bytes(files: Dict[str, bytes], label: str = "memory") -> BytesSource:
        return BytesSource(files, label)

    @staticmethod
    def package(package: str, folder: str = "") -> PackageSource:
        return PackageSource(package, folder)
