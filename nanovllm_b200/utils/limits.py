"""Process-wide resource caps and ``NANOVLLM_*`` properties.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/utils/ResourceLimits.java:39-106 (file 32 MiB,
corpus 256 MiB / 10k files, safetensors header 100 MiB, JSON depth 64 / 64 MiB, GGUF string 16 MiB, dims 8,
history 200) and NanoLlvmProps.java:44-95 (model / models dir / rag dir / arch / kernels / cpu threads / color,
as system properties or NANOLLVM_* env).  Here the environment prefix is NANOVLLM_ and every cap can be
overridden through it (e.g. NANOVLLM_MAX_FILE_BYTES).
"""
from __future__ import annotations

import os


def _env_int(name: str, default: int) -> int:
    v = os.environ.get("NANOVLLM_" + name)
    try:
        return int(v) if v is not None else default
    except ValueError:
        return default


class ResourceLimits:
    MAX_FILE_BYTES = _env_int("MAX_FILE_BYTES", 32 << 20)
    MAX_CORPUS_BYTES = _env_int("MAX_CORPUS_BYTES", 256 << 20)
    MAX_CORPUS_FILES = _env_int("MAX_CORPUS_FILES", 10_000)
    SAFETENSORS_HEADER_BYTES = _env_int("SAFETENSORS_HEADER_BYTES", 100 << 20)
    JSON_MAX_DEPTH = _env_int("JSON_MAX_DEPTH", 64)
    JSON_MAX_BYTES = _env_int("JSON_MAX_BYTES", 64 << 20)
    GGUF_MAX_STRING = _env_int("GGUF_MAX_STRING", 16 << 20)
    MAX_DIMS = _env_int("MAX_DIMS", 8)
    MAX_HISTORY_MESSAGES = _env_int("MAX_HISTORY_MESSAGES", 200)

    def __init__(self, max_file_bytes: int = None, max_total_corpus_bytes: int = None, max_corpus_files: int = None):
        """An instance carries the corpus budgets of one loader (class attributes are the process defaults)."""
        self.max_file_bytes = self.MAX_FILE_BYTES if max_file_bytes is None else int(max_file_bytes)
        self.max_total_corpus_bytes = self.MAX_CORPUS_BYTES if max_total_corpus_bytes is None \
            else int(max_total_corpus_bytes)
        self.max_corpus_files = self.MAX_CORPUS_FILES if max_corpus_files is None else int(max_corpus_files)
        if min(self.max_file_bytes, self.max_total_corpus_bytes, self.max_corpus_files) <= 0:
            raise ValueError("resource limits must be positive")

    @classmethod
    def current(cls) -> "ResourceLimits":
        return cls()

    def __repr__(self) -> str:
        return (f"ResourceLimits(file={self.max_file_bytes}, corpus={self.max_total_corpus_bytes}, "
                f"files={self.max_corpus_files})")


class Props:
    """NANOVLLM_* properties (model path, models dir, rag dir, arch confirmation, threads, color)."""

    @staticmethod
    def get(name: str, default=None):
        return os.environ.get("NANOVLLM_" + name.upper().replace(".", "_"), default)

    @staticmethod
    def model():
        return Props.get("model")

    @staticmethod
    def models_dir():
        return Props.get("models_dir", "models")

    @staticmethod
    def rag_dir():
        return Props.get("rag_dir", "rag")

    @staticmethod
    def arch():
        return Props.get("arch")

    @staticmethod
    def cpu_threads() -> int:
        v = Props.get("cpu_threads")
        return int(v) if v and v.isdigit() else (os.cpu_count() or 1)

    @staticmethod
    def color() -> bool:
        return Props.get("color", "1") not in ("0", "false", "no")
