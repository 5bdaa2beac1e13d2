"""BM25 passage index with query-term selection, out-of-corpus detection and grounded re-scoring.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/rag/PreparedRag.java:40-632 (BM25 k1=1.2,
b=0.75, idf ln(1 + (N - df + .5)/(df + .5)); hits below 0.45 x best dropped; query terms: distinct surface
tokens, contentful (>= 3 chars) and known to the corpus, the longer ones (>= 5 chars) preferred, at most 5,
longest first then rarest; a passage qualifies when it holds ceil-half of the selected terms (1..2); a query is
"outside the corpus" when half or more of its salient (non-glue) contentful terms are unknown or its longest
one is; final score = bm25 x (1 + term coverage) x (1 + 200/(200 + len)), ties to the shorter passage).

Tokens are runs of letters/digits of length >= 2, lower-cased; Cyrillic tokens also index truncated stems
(drop 1 / 2 trailing letters, first 5 letters) as cheap inflection keys.  The first passage of each source also
indexes the source's file-name stem tokens.
"""
from __future__ import annotations

import math
import os
import re
import unicodedata
from collections import Counter, defaultdict
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

from .corpus import RagLoadOptions, TextChunk

K1 = 1.2
B = 0.75
HIT_FLOOR_RATIO = 0.45
SHORT_PASSAGE_CHARS = 200.0
MAX_SELECTED_TERMS = 5
CONTENTFUL_MIN_LEN = 3

_TOKEN = re.compile(r"[^\W_]+", re.UNICODE)
_STEM_SPLIT = re.compile(r"[\W_]+", re.UNICODE)
QUERY_GLUE = frozenset(
    "a an the and or but if then than so as at by for from in into of on to with without about over under up "
    "down out off not no yes do does did doing done be am is are was were been being have has had having can "
    "could may might must shall should will would i me my we our you your he she it they them their this that "
    "these those what which who whom whose where when why how please tell say said ask think know like want "
    "need get got just also only very too more most some any all own same other such".split())


@dataclass(frozen=True)
class RagHit:
    chunk: TextChunk
    score: float


class RagIndex:
    """Retrieval contract: ``retrieve(query, top_k) -> [RagHit]`` best first."""

    def retrieve(self, query: str, top_k: int) -> List[RagHit]:
        raise NotImplementedError

    def is_outside_corpus(self, query: str) -> bool:
        return False

    def size(self) -> int:
        return -1


def _cyrillic(tok: str) -> bool:
    return any(0x0400 <= ord(c) <= 0x04FF for c in tok)


def surface_tokens(text: str) -> List[str]:
    return [t for t in _TOKEN.findall(text.lower()) if len(t) > 1]


def tokenize(text: str) -> List[str]:
    out: List[str] = []
    for t in surface_tokens(text):
        out.append(t)
        if _cyrillic(t):
            if len(t) >= 3:
                out.append(t[:-1])
            if len(t) >= 5:
                out.append(t[:-2])
            if len(t) > 5:
                out.append(t[:5])
    return out


def normalize_model_text(raw: Optional[str]) -> str:
    if not raw or not raw.strip():
        return ""
    return re.sub(r"\s+", " ", unicodedata.normalize("NFC", raw).replace("\u00a0", " ")).strip()


def strip_section_prefix(text: str) -> str:
    sep = text.find(" — ")
    return text[sep + 3:].strip() if 0 < sep <= 80 else text


def source_stem_tokens(source: Optional[str]) -> List[str]:
    if not source or not source.strip():
        return []
    name = source.split(":", 1)[1] if source.startswith("resource:") else source
    name = os.path.basename(name.replace("\\", "/"))
    if "." in name[1:]:
        name = name[:name.rfind(".")]
    name = name.lower()
    toks = [p for p in _STEM_SPLIT.split(name) if len(p) > 1]
    return toks or ([name] if len(name) > 1 else [])


def term_coverage(text: str, terms: Sequence[str]) -> float:
    if not terms:
        return 0.0
    have = set(tokenize(text))
    return sum(1 for t in terms if t in have) / len(terms)


def grounded_score(hit: RagHit, terms: Sequence[str]) -> float:
    n = max(len(hit.chunk.text), 1)
    return hit.score * (1.0 + term_coverage(hit.chunk.text, terms)) * (1.0 + SHORT_PASSAGE_CHARS / (SHORT_PASSAGE_CHARS + n))


def keep_strong(scored: List[RagHit], top_k: int) -> List[RagHit]:
    if not scored:
        return []
    floor = scored[0].score * HIT_FLOOR_RATIO
    return [h for h in scored if h.score >= floor][:top_k]


@dataclass(frozen=True)
class Passage:
    chunk: TextChunk
    search_text: str
    tf: Dict[str, int]
    length: int


class PreparedRag(RagIndex):
    def __init__(self, chunks: Sequence[TextChunk], source_root: Optional[str] = None,
                 options: Optional[RagLoadOptions] = None):
        self.options = options or RagLoadOptions.defaults()
        self.source_root = source_root
        stems_done = set()
        ps: List[Passage] = []
        for c in chunks:
            if c.is_blank():
                continue
            text = normalize_model_text(c.text)
            search = strip_section_prefix(text)
            if c.source not in stems_done:
                stems_done.add(c.source)
                search = " ".join([search] + source_stem_tokens(c.source))
            tf = Counter(tokenize(search))
            ps.append(Passage(TextChunk(c.id, c.source, text), search, dict(tf), sum(tf.values())))
        if not ps:
            raise ValueError("no non-blank passages to index")
        self.passages = ps
        self.chunks = [p.chunk for p in ps]
        self.df: Dict[str, int] = Counter()
        self.postings: Dict[str, List[int]] = defaultdict(list)
        for i, p in enumerate(ps):
            for t in p.tf:
                self.df[t] += 1
                self.postings[t].append(i)
        n = len(ps)
        self.idf = {t: math.log(1.0 + (n - d + 0.5) / (d + 0.5)) for t, d in self.df.items()}
        self.avg_len = max(sum(p.length for p in ps) / n, 1.0)

    # ------------------------------------------------------------------ RagIndex
    def size(self) -> int:
        return len(self.passages)

    def is_outside_corpus(self, query: str) -> bool:
        return self._outside(list(dict.fromkeys(surface_tokens(query))))

    def retrieve(self, query: str, top_k: int) -> List[RagHit]:
        terms = self.select_terms(query)
        if not terms:
            return []
        hits = self._bm25(query, terms, max(top_k * 4, top_k))
        rescored = [RagHit(h.chunk, grounded_score(h, terms)) for h in hits
                    if term_coverage(h.chunk.text, terms) > 0.0]
        rescored.sort(key=lambda h: (-h.score, len(h.chunk.text)))
        return rescored[:top_k]

    def __repr__(self) -> str:
        return f"PreparedRag(passages={self.size()}, source={self.source_root or 'inline'})"

    # ------------------------------------------------------------------ query terms
    def _unknown(self, term: str) -> bool:
        if len(term) < CONTENTFUL_MIN_LEN or self.df.get(term, 0) > 0:
            return False
        return not any(self.df.get(k, 0) > 0 for k in tokenize(term))

    def _outside(self, surface: List[str]) -> bool:
        if not surface:
            return False
        salient = [t for t in surface if len(t) >= CONTENTFUL_MIN_LEN and t not in QUERY_GLUE]
        if not salient:
            return False
        oov = sum(1 for t in salient if self._unknown(t))
        if oov == 0:
            return False
        if oov * 2 >= len(salient):
            return True
        longest = max(len(t) for t in salient)
        return any(self._unknown(t) for t in salient if len(t) == longest)

    def select_terms(self, query: str) -> List[str]:
        surface = list(dict.fromkeys(surface_tokens(query)))
        if not surface or self._outside(surface):
            return []
        known = [t for t in dict.fromkeys(tokenize(query))
                 if len(t) >= CONTENTFUL_MIN_LEN and self.df.get(t, 0) > 0]
        if not known:
            return []
        longer = [t for t in known if len(t) >= 5]
        pool = longer or known
        pool.sort(key=lambda t: (-len(t), -self.idf.get(t, 0.0)))
        return pool[:MAX_SELECTED_TERMS]

    def _qualifies(self, p: Passage, terms: List[str]) -> bool:
        matched = sum(1 for t in terms if t in p.tf)
        need = min(max((len(terms) + 1) // 2, 1), 2)
        return matched >= need

    def _bm25(self, query: str, terms: List[str], top_k: int) -> List[RagHit]:
        raw = len(set(surface_tokens(query)))
        if raw >= 3 and not terms:
            return []
        cand = []
        seen = set()
        for t in terms:
            for d in self.postings.get(t, ()):
                if d not in seen:
                    seen.add(d)
                    cand.append(d)
        scored = []
        for d in cand:
            p = self.passages[d]
            if not self._qualifies(p, terms):
                continue
            s = 0.0
            norm = K1 * (1.0 - B + B * p.length / self.avg_len)
            for t in terms:
                f = p.tf.get(t, 0)
                if f:
                    s += self.idf.get(t, 0.0) * f * (K1 + 1.0) / (f + norm)
            if s > 0.0:
                scored.append(RagHit(p.chunk, s))
        scored.sort(key=lambda h: -h.score)
        return keep_strong(scored, top_k)
