"""Entry points that build retrieval indexes from folders, files, package resources or inline texts.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/rag/RagFactory.java:40-669 (make / try_make from
a folder or file, of(texts...), resource corpora, builder with options / tuners / listeners, and
``with_embeddings`` / ``build(encoder)`` producing a BM25 + dense hybrid).
"""
from __future__ import annotations

import os
from typing import Iterable, Optional

from ..chat.listeners import LlmListener
from .corpus import CorpusLoader, RagLoadOptions, RagTuner
from .dense import DenseRagIndex, HybridRagIndex
from .lexical import PreparedRag


class RagFactory:
    @staticmethod
    def make(folder_or_file: str, options: Optional[RagLoadOptions] = None,
             listener: Optional[LlmListener] = None, encoder=None):
        b = RagFactory.builder().options(options or RagLoadOptions.defaults()).listen(listener)
        b.add_path(folder_or_file)
        return b.build(encoder)

    @staticmethod
    def try_make(folder_or_file: Optional[str], options: Optional[RagLoadOptions] = None,
                 listener: Optional[LlmListener] = None, encoder=None):
        """None when the path is missing or holds no indexable text (instead of raising)."""
        if not folder_or_file or not os.path.exists(folder_or_file):
            return None
        try:
            return RagFactory.make(folder_or_file, options, listener, encoder)
        except ValueError:
            return None

    @staticmethod
    def of(*texts: str, options: Optional[RagLoadOptions] = None) -> PreparedRag:
        if len(texts) == 1 and not isinstance(texts[0], str):
            texts = tuple(texts[0])
        return RagFactory.builder().options(options or RagLoadOptions.defaults()).add_all(texts).build()

    @staticmethod
    def make_resource(package: str, name: str, options: Optional[RagLoadOptions] = None) -> PreparedRag:
        return RagFactory.builder().options(options or RagLoadOptions.defaults()).add_resource(package, name).build()

    @staticmethod
    def with_embeddings(lexical: PreparedRag, encoder, on_passage_embedded=None) -> HybridRagIndex:
        return HybridRagIndex.of(lexical, DenseRagIndex.of(lexical, encoder, on_passage_embedded))

    @staticmethod
    def builder() -> "RagBuilder":
        return RagBuilder()


class RagBuilder:
    def __init__(self):
        self._opts = RagLoadOptions.defaults()
        self._listener = None
        self._tuners = []
        self._exts = None
        self._root = None
        self._ops = []

    def options(self, opts: RagLoadOptions) -> "RagBuilder":
        self._opts = opts
        return self

    def for_tiny_models(self) -> "RagBuilder":
        return self.options(RagLoadOptions.for_tiny_models())

    def listen(self, listener) -> "RagBuilder":
        self._listener = listener
        return self

    def add_processor(self, *tuners: RagTuner) -> "RagBuilder":
        self._tuners.extend(tuners)
        return self

    def source_root(self, root: str) -> "RagBuilder":
        self._root = root
        return self

    def folder_extensions(self, exts: Iterable[str]) -> "RagBuilder":
        self._exts = list(exts)
        return self

    def add(self, text: str, id_: Optional[str] = None) -> "RagBuilder":
        self._ops.append(lambda L: L.add(text, id_))
        return self

    def add_all(self, texts: Iterable[str]) -> "RagBuilder":
        for t in texts:
            self.add(t)
        return self

    def add_file(self, path: str) -> "RagBuilder":
        self._ops.append(lambda L: L.add_file(path))
        return self

    def add_folder(self, path: str) -> "RagBuilder":
        if self._root is None:
            self._root = os.path.abspath(path)
        self._ops.append(lambda L: L.add_folder(path))
        return self

    def add_path(self, path: str) -> "RagBuilder":
        return self.add_folder(path) if os.path.isdir(path) else self.add_file(path)

    def add_resource(self, package: str, name: str) -> "RagBuilder":
        self._ops.append(lambda L: L.add_resource(package, name))
        return self

    def build(self, encoder=None):
        """BM25 index, or a BM25 + dense hybrid when an embedding ``encoder`` is given."""
        loader = CorpusLoader(self._opts, self._listener).add_tuner(*self._tuners)
        if self._exts is not None:
            loader.folder_extensions(self._exts)
        for op in self._ops:
            op(loader)
        lexical = PreparedRag(loader.build(), self._root, self._opts)
        return lexical if encoder is None else RagFactory.with_embeddings(lexical, encoder)
