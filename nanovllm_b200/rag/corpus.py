"""Corpus loading and chunking for retrieval.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/rag/{CorpusLoader.java:40-735, TextChunk.java,
RagLoadOptions.java:30-166, RagResource.java, RagTuner.java, RagTunerChain.java}.

Pipeline per document: tuner chain (allow? -> extract text -> preprocess text) -> cleanup into passages
(code fences removed, markdown headings become a ``section — `` prefix, links/images/inline code unwrapped,
bullets dropped, paragraphs split into sentences) -> chunking:
* ``atomic_sentences``: every passage its own chunk (long ones window-split without overlap);
* otherwise passages are packed greedily up to ``max_chunk_chars`` (a passage longer than that is window-split
  with overlap);
* no usable passages (or ``preprocess=False``): sliding windows of ``max_chunk_chars`` that prefer to break at a
  newline or space in the second half of the window, stepping ``max - overlap``.
Chunks are de-duplicated on a case/whitespace-folded fingerprint.  Budgets (bytes per file, file count, total
bytes) come from ``ResourceLimits``.  Package resources (``importlib.resources``) stand in for Java classpath
resources.
"""
from __future__ import annotations

import importlib.resources
import os
import re
from dataclasses import dataclass, field, replace
from typing import Callable, Iterable, List, Optional, Sequence

from ..chat.listeners import LlmListener, info
from ..utils.limits import ResourceLimits

DEFAULT_EXTENSIONS = frozenset({
    ".txt", ".md", ".markdown", ".rst", ".csv", ".tsv", ".json", ".xml", ".html", ".htm", ".properties", ".yml",
    ".yaml", ".log", ".java", ".kt", ".py", ".js", ".ts", ".css"})
_README = {"readme.md", "readme.txt", "readme.markdown"}


@dataclass(frozen=True)
class TextChunk:
    id: str
    source: str
    text: str = ""

    def __post_init__(self):
        if not self.id or not self.id.strip():
            raise ValueError("chunk id must not be blank")
        if self.text is None:
            object.__setattr__(self, "text", "")

    @staticmethod
    def of(id_: str, text: str) -> "TextChunk":
        return TextChunk(id_, id_, text)

    def is_blank(self) -> bool:
        return not self.text.strip()


@dataclass(frozen=True)
class RagLoadOptions:
    max_chunk_chars: int = 500
    chunk_overlap: int = 40
    preprocess: bool = True
    atomic_sentences: bool = False
    dedupe: bool = True
    limits: ResourceLimits = field(default_factory=ResourceLimits.current)

    def __post_init__(self):
        if self.max_chunk_chars < 64:
            raise ValueError("max_chunk_chars must be >= 64")
        if self.chunk_overlap < 0:
            raise ValueError("chunk_overlap must be >= 0")

    @staticmethod
    def defaults() -> "RagLoadOptions":
        return RagLoadOptions()

    @staticmethod
    def for_tiny_models() -> "RagLoadOptions":
        """Short atomic sentence chunks: small models ground better on one fact per passage."""
        return RagLoadOptions(max_chunk_chars=220, chunk_overlap=0, atomic_sentences=True)

    def with_(self, **kw) -> "RagLoadOptions":
        return replace(self, **kw)


@dataclass(frozen=True)
class RagResource:
    kind: str  # "file" | "resource"
    source: str
    path: Optional[str] = None
    content: Optional[bytes] = None

    @staticmethod
    def file(path: str, content: Optional[bytes] = None) -> "RagResource":
        p = os.path.abspath(path)
        return RagResource("file", p, p, content)

    @staticmethod
    def resource(name: str, content: Optional[bytes] = None) -> "RagResource":
        name = name.strip().lstrip("/")
        if not name:
            raise ValueError("resource path must not be blank")
        return RagResource("resource", "resource:" + name, name, content)

    def file_name(self) -> str:
        return os.path.basename(self.path or self.source)

    def is_file(self) -> bool:
        return self.kind == "file"


class RagTuner:
    """Hooks over corpus loading: filter resources, custom text extraction, text preprocessing."""

    def allows(self, resource: RagResource) -> bool:
        return True

    def extract(self, resource: RagResource) -> Optional[str]:
        return None

    def preprocess(self, text: str) -> str:
        return text

    @staticmethod
    def allowing(pred: Callable[[RagResource], bool]) -> "RagTuner":
        t = RagTuner()
        t.allows = pred  # type: ignore[method-assign]
        return t

    @staticmethod
    def extracting(fn: Callable[[RagResource], Optional[str]]) -> "RagTuner":
        t = RagTuner()
        t.extract = fn  # type: ignore[method-assign]
        return t

    @staticmethod
    def preprocessing(fn: Callable[[str], str]) -> "RagTuner":
        t = RagTuner()
        t.preprocess = fn  # type: ignore[method-assign]
        return t


class RagTunerChain:
    def __init__(self, tuners: Sequence[RagTuner] = ()):
        self.tuners = list(tuners)

    def plus(self, *more: RagTuner) -> "RagTunerChain":
        return RagTunerChain(self.tuners + list(more))

    def allows(self, r: RagResource) -> bool:
        return all(t.allows(r) for t in self.tuners)

    def extract(self, r: RagResource) -> Optional[str]:
        for t in self.tuners:
            got = t.extract(r)
            if got is not None:
                return got
        return None

    def preprocess(self, text: str) -> str:
        for t in self.tuners:
            text = t.preprocess(text)
        return text


# ----------------------------------------------------------------------------------------------- cleanup
_HEADING = re.compile(r"^#{1,6}\s+(.+?)\s*$")
_LINK = re.compile(r"\[([^\]]+)]\([^)]*\)")
_IMAGE = re.compile(r"!\[[^\]]*]\([^)]*\)")
_FENCE = re.compile(r"```.*?```", re.S)
_INLINE_CODE = re.compile(r"`([^`]+)`")
_BULLET = re.compile(r"^\s*[-*+]\s+")
_SENTENCE_END = re.compile(r"(?<=[.!?。！？])\s+(?=[^\W_]|[\"'(«])")


def _clean_inline(line: str) -> str:
    t = _IMAGE.sub("", line)
    t = _LINK.sub(r"\1", t)
    t = _INLINE_CODE.sub(r"\1", t)
    return re.sub(r" {2,}", " ", t.replace("\t", " "))


def passages(raw: Optional[str]) -> List[str]:
    """Sentence-level passages, each prefixed by its markdown section title (``title — sentence``)."""
    if not raw or not raw.strip():
        return []
    text = _FENCE.sub("\n", raw.replace("\r\n", "\n").replace("\r", "\n"))
    section, para, out = "", [], []

    def flush():
        if not para:
            return
        body = re.sub(r" +", " ", " ".join(para)).strip()
        para.clear()
        for s in _SENTENCE_END.split(body):
            s = s.strip()
            if s:
                out.append(f"{section} — {s}" if section else s)

    for line in text.split("\n"):
        h = _HEADING.match(line.strip())
        if h:
            flush()
            section = _clean_inline(h.group(1)).strip()
            continue
        if not line.strip():
            flush()
            continue
        cleaned = _clean_inline(_BULLET.sub("", line, count=1)).strip()
        if cleaned:
            para.append(cleaned)
    flush()
    return out


# ----------------------------------------------------------------------------------------------- chunking
def _prefer_break(body: str, start: int, end: int) -> int:
    lo = max(start + (end - start) // 2, start)
    nl = body.rfind("\n", 0, end)
    if nl >= lo:
        return nl + 1
    sp = body.rfind(" ", 0, end)
    if sp >= lo:
        return sp + 1
    return end


def window_split(base_id: str, source: str, body: str, max_chars: int, overlap: int) -> List[TextChunk]:
    if len(body) <= max_chars:
        return [TextChunk(base_id, source, body)]
    step = max(1, max_chars - min(overlap, max_chars - 1))
    out, start, part = [], 0, 0
    while start < len(body):
        end = min(len(body), start + max_chars)
        if end < len(body):
            end = _prefer_break(body, start, end)
        piece = body[start:end].strip()
        if piece:
            part += 1
            cid = base_id if (part == 1 and end >= len(body)) else f"{base_id}#{part}"
            out.append(TextChunk(cid, source, piece))
        if end >= len(body):
            break
        start = min(max(start + 1, end - (max_chars - step)), end)
    return out


def _atomic(base_id, source, units, max_chars) -> List[TextChunk]:
    out: List[TextChunk] = []
    for u in units:
        if len(u) <= max_chars:
            out.append(TextChunk(f"{base_id}#{len(out) + 1}", source, u))
            continue
        for w in window_split(f"{base_id}#{len(out) + 1}", source, u, max_chars, 0):
            out.append(TextChunk(f"{base_id}#{len(out) + 1}", source, w.text))
    if len(out) == 1:
        return [TextChunk(base_id, source, out[0].text)]
    return out


def _pack(base_id, source, units, max_chars, overlap) -> List[TextChunk]:
    out: List[TextChunk] = []
    buf: List[str] = []
    size = 0

    def emit():
        nonlocal size
        if buf:
            out.append(TextChunk(f"{base_id}#{len(out) + 1}", source, " ".join(buf)))
            buf.clear()
            size = 0

    for u in units:
        if len(u) > max_chars:
            emit()
            out.extend(window_split(f"{base_id}#w{len(out) + 1}", source, u, max_chars, overlap))
            continue
        if buf and size + 1 + len(u) > max_chars:
            emit()
        size = size + 1 + len(u) if buf else len(u)
        buf.append(u)
    emit()
    if len(out) == 1:
        return [TextChunk(base_id, out[0].source, out[0].text)]
    return out


def split(base_id: str, source: str, text: Optional[str], opts: RagLoadOptions) -> List[TextChunk]:
    if not text or not text.strip():
        return []
    if opts.preprocess:
        units = passages(text)
        if units:
            if opts.atomic_sentences:
                return _atomic(base_id, source, units, opts.max_chunk_chars)
            return _pack(base_id, source, units, opts.max_chunk_chars, opts.chunk_overlap)
    return window_split(base_id, source, text.strip(), opts.max_chunk_chars, opts.chunk_overlap)


def _fingerprint(text: str) -> str:
    return re.sub(r"\s+", " ", text.lower()).strip()


# ----------------------------------------------------------------------------------------------- loader
class CorpusLoader:
    def __init__(self, options: Optional[RagLoadOptions] = None, listener: Optional[LlmListener] = None):
        self.opts = options or RagLoadOptions.defaults()
        self.listener = listener
        self.tuners = RagTunerChain()
        self.extensions = DEFAULT_EXTENSIONS
        self.pending: List[TextChunk] = []
        self._anon = 0
        self._files = 0
        self._bytes = 0
        self._root: Optional[str] = None

    # knobs
    def options(self, opts: RagLoadOptions) -> "CorpusLoader":
        self.opts = opts
        return self

    def add_tuner(self, *tuners: RagTuner) -> "CorpusLoader":
        self.tuners = self.tuners.plus(*tuners)
        return self

    def folder_extensions(self, exts: Iterable[str]) -> "CorpusLoader":
        self.extensions = frozenset((e if e.startswith(".") else "." + e).lower() for e in exts)
        return self

    # sources
    def add(self, text: str, id_: Optional[str] = None, source: Optional[str] = None) -> "CorpusLoader":
        if id_ is None:
            self._anon += 1
            id_ = f"text-{self._anon}"
        self._append(id_, source or id_, text, None)
        return self

    def add_all(self, texts: Iterable[str]) -> "CorpusLoader":
        for t in texts:
            self.add(t)
        return self

    def add_file(self, path: str) -> "CorpusLoader":
        p = os.path.abspath(path)
        if not os.path.isfile(p):
            raise ValueError(f"not a regular file: {p}")
        res = RagResource.file(p)
        if not self.tuners.allows(res):
            info(self.listener, None, f"RAG skipped: {self._display(p)}\n")
            return self
        size = os.path.getsize(p)
        self._budget(p, size)
        with open(p, "rb") as f:
            data = f.read()
        self._account(size)
        self._index(RagResource.file(p, data), self._display(p))
        return self

    def add_files(self, *paths: str) -> "CorpusLoader":
        for p in paths:
            self.add_file(p)
        return self

    def add_folder(self, folder: str) -> "CorpusLoader":
        root = os.path.abspath(folder)
        if not os.path.isdir(root):
            raise ValueError(f"not a directory: {root}")
        self._root = root
        info(self.listener, None, f"RAG scanning {root} ...\n")
        for dirpath, dirnames, filenames in os.walk(root):
            dirnames.sort()
            for fn in sorted(filenames):
                if self._indexed(fn):
                    self.add_file(os.path.join(dirpath, fn))
        return self

    def add_resource(self, package: str, name: str) -> "CorpusLoader":
        """A data file shipped inside an importable package (the Python analogue of a classpath resource)."""
        ref = importlib.resources.files(package).joinpath(name)
        if not ref.is_file():
            raise ValueError(f"package resource not found: {package}/{name}")
        res = RagResource.resource(f"{package.replace('.', '/')}/{name}")
        if not self.tuners.allows(res):
            info(self.listener, None, f"RAG skipped: {res.source}\n")
            return self
        data = ref.read_bytes()
        self._budget(res.source, len(data))
        self._account(len(data))
        self._index(RagResource.resource(res.path, data), res.source)
        return self

    def build(self) -> List[TextChunk]:
        if self.opts.dedupe:
            seen = {}
            for c in self.pending:
                if not c.is_blank():
                    seen.setdefault(_fingerprint(c.text), c)
            out = list(seen.values())
        else:
            out = [c for c in self.pending if not c.is_blank()]
        if not out:
            raise ValueError("corpus has no non-blank chunks")
        return out

    # internals
    def _indexed(self, name: str) -> bool:
        low = name.lower()
        if low in _README or "." not in low:
            return False
        return low[low.rfind("."):] in self.extensions

    def _display(self, p: str) -> str:
        if self._root and p.startswith(self._root + os.sep):
            return os.path.relpath(p, self._root)
        return os.path.basename(p)

    def _budget(self, label: str, size: int) -> None:
        lim = self.opts.limits
        if size > lim.max_file_bytes:
            raise ValueError(f"file exceeds max_file_bytes ({lim.max_file_bytes}): {label}")
        if self._files >= lim.max_corpus_files:
            raise RuntimeError(f"corpus exceeds max_corpus_files ({lim.max_corpus_files})")
        if self._bytes + size > lim.max_total_corpus_bytes:
            raise RuntimeError(f"corpus exceeds max_total_corpus_bytes ({lim.max_total_corpus_bytes})")

    def _account(self, size: int) -> None:
        self._files += 1
        self._bytes += size

    def _index(self, res: RagResource, display: str) -> None:
        body = self.tuners.extract(res)
        if body is None:
            body = (res.content or b"").decode("utf-8", errors="replace")
        self._append(res.source, res.source, body, display)

    def _append(self, id_: str, source: str, text: Optional[str], display: Optional[str]) -> None:
        body = self.tuners.preprocess(text or "")
        chunks = split(id_, source, body, self.opts)
        self.pending.extend(chunks)
        if display is not None and self.listener is not None:
            info(self.listener, None, f"RAG {display}: {len(body)} char(s) -> {len(chunks)} chunk(s)\n")
            if not body:
                info(self.listener, None, f"RAG warning: no text extracted from {display}\n")
