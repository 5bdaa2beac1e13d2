"""Dense (embedding) and hybrid (reciprocal-rank fusion) retrieval.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/rag/DenseRagIndex.java:30-438 (cosine on
L2-normalised embeddings, hits below 0.45 x best dropped, "outside the corpus" when the best similarity is
< 0.28, ties to the shorter passage) and HybridRagIndex.java:30-315 (RRF with k=60 over each leaf index's
top ``4 x top_k``; outside only when every leaf says so; nested hybrids flattened, leaves must be distinct).

The reference embeds passages one at a time (optionally on an executor) and scores with a Java dot-product
loop.  Here the whole corpus goes through the encoder in packed batches and the passage matrix stays resident
on the encoder's device: a query is one encoder pass plus one [N, H] x [H] product.
"""
from __future__ import annotations

from typing import Callable, Dict, List, Optional, Sequence

import torch

from .corpus import TextChunk
from .lexical import HIT_FLOOR_RATIO, PreparedRag, RagHit, RagIndex

OUTSIDE_MAX_SIMILARITY = 0.28
RRF_K = 60
EMBED_BATCH = 256


class DenseRagIndex(RagIndex):
    def __init__(self, chunks: Sequence[TextChunk], encoder, vectors: Optional[torch.Tensor] = None,
                 on_passage_embedded: Optional[Callable[[int], None]] = None):
        if not chunks:
            raise ValueError("chunks must not be empty")
        if not hasattr(encoder, "is_embedding") or not encoder.is_embedding():
            raise ValueError(f"dense retrieval needs an embedding encoder (got {getattr(encoder, 'architecture_name', encoder)})")
        if getattr(encoder, "is_closed", lambda: False)():
            raise RuntimeError("embedding model is closed")
        self.chunks = list(chunks)
        self.encoder = encoder
        if vectors is None:
            parts = []
            texts = [c.text if c.text.strip() else c.id for c in self.chunks]
            for i in range(0, len(texts), EMBED_BATCH):
                parts.append(encoder.embed_batch(texts[i:i + EMBED_BATCH]))
                if on_passage_embedded is not None:
                    on_passage_embedded(min(i + EMBED_BATCH, len(texts)))
            vectors = torch.cat(parts, 0)
        if vectors.shape[0] != len(self.chunks):
            raise ValueError("vectors must match chunks")
        self.vectors = vectors.float().contiguous()
        self.dimensions = int(self.vectors.shape[1])
        self._lengths = torch.tensor([len(c.text) for c in self.chunks], dtype=torch.float64)

    @staticmethod
    def of(lexical_or_chunks, encoder, on_passage_embedded=None) -> "DenseRagIndex":
        chunks = lexical_or_chunks.chunks if isinstance(lexical_or_chunks, PreparedRag) else lexical_or_chunks
        return DenseRagIndex(chunks, encoder, on_passage_embedded=on_passage_embedded)

    def size(self) -> int:
        return len(self.chunks)

    def _scores(self, query: str) -> torch.Tensor:
        q = self.encoder.embed_batch([query if query.strip() else "_"])[0].to(self.vectors.device)
        return (self.vectors @ q).double().cpu()

    def is_outside_corpus(self, query: str) -> bool:
        if not query.strip():
            return True
        return float(self._scores(query).max()) < OUTSIDE_MAX_SIMILARITY

    def retrieve(self, query: str, top_k: int) -> List[RagHit]:
        if top_k <= 0:
            raise ValueError("top_k must be > 0")
        if not query.strip():
            return []
        s = self._scores(query)
        keep = torch.nonzero(s > 0.0).flatten().tolist()
        if not keep:
            return []
        keep.sort(key=lambda i: (-float(s[i]), len(self.chunks[i].text)))
        floor = float(s[keep[0]]) * HIT_FLOOR_RATIO
        return [RagHit(self.chunks[i], float(s[i])) for i in keep if float(s[i]) >= floor][:top_k]

    def __repr__(self) -> str:
        return f"DenseRagIndex(passages={self.size()}, dim={self.dimensions})"


def fuse(rankings: Sequence[Sequence[RagHit]], top_k: int) -> List[RagHit]:
    """Reciprocal-rank fusion: score(chunk) = sum over rankings of 1 / (k + rank)."""
    if not rankings:
        raise ValueError("rankings must not be empty")
    if top_k <= 0:
        raise ValueError("top_k must be > 0")
    acc: Dict[str, List] = {}
    for hits in rankings:
        for rank, h in enumerate(hits):
            r = 1.0 / (RRF_K + rank + 1)
            if h.chunk.id in acc:
                acc[h.chunk.id][1] += r
            else:
                acc[h.chunk.id] = [h.chunk, r]
    out = sorted(acc.values(), key=lambda a: (-a[1], len(a[0].text)))
    return [RagHit(c, s) for c, s in out[:top_k]]


class HybridRagIndex(RagIndex):
    def __init__(self, indexes: Sequence[RagIndex]):
        leaves: List[RagIndex] = []

        def add(ix):
            if isinstance(ix, HybridRagIndex):
                for leaf in ix.indexes:
                    add(leaf)
                return
            if any(ix is x for x in leaves):
                raise ValueError("hybrid indexes must be distinct")
            leaves.append(ix)

        for ix in indexes:
            add(ix)
        if len(leaves) < 2:
            raise ValueError("a hybrid index needs at least two indexes")
        self.indexes = leaves

    @staticmethod
    def of(lexical: PreparedRag, dense_or_encoder, on_passage_embedded=None) -> "HybridRagIndex":
        dense = dense_or_encoder if isinstance(dense_or_encoder, DenseRagIndex) else \
            DenseRagIndex.of(lexical, dense_or_encoder, on_passage_embedded)
        if lexical.size() != dense.size():
            raise ValueError("lexical and dense indexes must cover the same passages")
        return HybridRagIndex([lexical, dense])

    def lexical(self) -> PreparedRag:
        for ix in self.indexes:
            if isinstance(ix, PreparedRag):
                return ix
        raise RuntimeError("hybrid has no BM25 index")

    def dense(self) -> DenseRagIndex:
        for ix in self.indexes:
            if isinstance(ix, DenseRagIndex):
                return ix
        raise RuntimeError("hybrid has no dense index")

    def size(self) -> int:
        n = self.indexes[0].size()
        return n if all(ix.size() == n for ix in self.indexes) else -1

    def is_outside_corpus(self, query: str) -> bool:
        return all(ix.is_outside_corpus(query) for ix in self.indexes)

    def retrieve(self, query: str, top_k: int) -> List[RagHit]:
        if top_k <= 0:
            raise ValueError("top_k must be > 0")
        pool = max(top_k * 4, top_k)
        return fuse([ix.retrieve(query, pool) for ix in self.indexes], top_k)

    def __repr__(self) -> str:
        return f"HybridRagIndex(passages={self.size()}, sources={len(self.indexes)})"
