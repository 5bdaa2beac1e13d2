"""Tokenizer codecs: text <-> token pieces.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/tokenizer/{Gpt2ByteBpeCodec, Gpt2Bytes,
MetaspaceBpeCodec, MetaspaceText, BpeMerges, WordPieceCodec, UnigramCodec, PrecompiledCharsMap, WordLevelCodec,
CharCodec, SentencePieceModel, TextNormalizer}.java.  Each codec maps a normalised string to vocabulary ids and
token pieces back to text:

* ``ByteBpe``      GPT-2 byte-level BPE: bytes -> printable code points, regex pre-split, rank-ordered merges;
* ``MetaspaceBpe`` SentencePiece-style BPE over text with spaces as U+2581 and optional <0xNN> byte fallback;
                   merges come from a merge list or, for GGUF "llama" vocabularies, from the piece scores;
* ``WordPiece``    BERT basic tokenisation (clean, CJK split, optional lower-case / accent strip, punctuation)
                   then greedy longest-match with a "##" continuation prefix;
* ``Unigram``      SentencePiece unigram: Viterbi over piece log-probabilities with byte fallback / unk;
* ``WordLevel``    whitespace words looked up whole;  ``Char`` one id per character.
"""
from __future__ import annotations

import heapq
import unicodedata
from functools import lru_cache
from typing import Dict, List, Optional, Sequence, Tuple

import regex

GPT2_PATTERN = r"""'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+"""
# Llama-3 / Qwen2-style split (case-insensitive contractions, single digits, newline runs)
QWEN2_PATTERN = (r"""(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|"""
                 r"""\s*[\r\n]+|\s+(?!\S)|\s+""")
LLAMA3_PATTERN = (r"""(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n]*|"""
                  r"""\s*[\r\n]+|\s+(?!\S)|\s+""")
SPIECE = "▁"


def bytes_to_unicode() -> Dict[int, str]:
    """The GPT-2 reversible byte -> printable character table: printable Latin-1 bytes map to themselves,
    the remaining 68 bytes to code points 256 and up, in byte order."""
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(ord("\xa1"), ord("\xac") + 1)) + \
        list(range(ord("\xae"), ord("\xff") + 1))
    table = {}
    extra = 0
    for b in range(256):
        if b in keep:
            table[b] = chr(b)
        else:
            table[b] = chr(256 + extra)
            extra += 1
    return table


BYTE_ENCODER = bytes_to_unicode()
BYTE_DECODER = {v: k for k, v in BYTE_ENCODER.items()}
_BYTE_CHARS = frozenset(BYTE_DECODER)
_TO_LATIN1 = {ord(ch): b for ch, b in BYTE_DECODER.items()}  # str.translate: byte symbol -> the byte as a char


def bpe_merge(symbols: List[str], ranks: Dict[Tuple[str, str], int]) -> List[str]:
    """Apply merges lowest rank first until no adjacent pair is mergeable (the pure-Python path; byte-level
    vocabularies use the C++ core in csrc/host/bpe.cpp when it is built)."""
    if len(symbols) < 2:
        return symbols
    while True:
        best = None
        best_rank = None
        for i in range(len(symbols) - 1):
            r = ranks.get((symbols[i], symbols[i + 1]))
            if r is not None and (best_rank is None or r < best_rank):
                best_rank, best = r, (symbols[i], symbols[i + 1])
        if best is None:
            return symbols
        merged = []
        i = 0
        while i < len(symbols):
            if i < len(symbols) - 1 and symbols[i] == best[0] and symbols[i + 1] == best[1]:
                merged.append(best[0] + best[1])
                i += 2
            else:
                merged.append(symbols[i])
                i += 1
        symbols = merged
        if len(symbols) == 1:
            return symbols


class Codec:
    def encode(self, text: str) -> List[int]:
        raise NotImplementedError

    def decode(self, pieces: Sequence[str]) -> str:
        raise NotImplementedError


def _native_core():
    try:
        import torch  # noqa: F401  (loads the libraries the extension links against)
        from .. import _host
        return _host
    except ImportError:  # the host helpers were not built: the pure-Python merge below runs instead
        return None


class ByteBpe(Codec):
    def __init__(self, vocab: Dict[str, int], merges: List[Tuple[str, str]], pattern: Optional[str] = GPT2_PATTERN,
                 unk_id: Optional[int] = None, native: Optional[bool] = None):
        self.vocab = vocab
        self.ranks = {m: i for i, m in enumerate(merges)}
        self.split = regex.compile(pattern) if pattern else None
        self.unk_id = unk_id
        self._cache: Dict[str, List[int]] = {}
        host = _native_core() if native is not False else None
        if native and host is None:
            raise ImportError("nanovllm_b200._host is not built (python setup.py build_ext --inplace)")
        self._core = self._build_core(host) if host is not None else None

    def _build_core(self, host):
        """Intern every symbol a merge can produce and hand the merge table to the C++ core (csrc/host/bpe.cpp)."""
        ids: Dict[str, int] = {}
        syms: List[str] = []

        def sid(x: str) -> int:
            i = ids.get(x)
            if i is None:
                i = ids[x] = len(syms)
                syms.append(x)
            return i

        byte_sym = [sid(BYTE_ENCODER[b]) for b in range(256)]
        left, right, rank, merged = [], [], [], []
        for (a, b), r in self.ranks.items():
            left.append(sid(a))
            right.append(sid(b))
            rank.append(r)
            merged.append(sid(a + b))
        vocab, unk = self.vocab, self.unk_id
        sym_vocab = [vocab.get(x, -1) for x in syms]
        fb_off, fb_ids = [0], []
        for x, v in zip(syms, sym_vocab):
            if v < 0:  # unknown merged piece: its single byte symbols (as the Python path does)
                fb_ids.extend(j for j in (vocab.get(ch, unk) for ch in x) if j is not None)
            fb_off.append(len(fb_ids))
        return host.ByteBpeCore(byte_sym, left, right, rank, merged, sym_vocab, fb_off, fb_ids)

    def _word(self, word: str) -> List[int]:
        hit = self._cache.get(word)
        if hit is not None:
            return hit
        if self._core is not None:
            ids = self._core.encode_word(word.encode("utf-8"))
            if len(self._cache) < 100_000:
                self._cache[word] = ids
            return ids
        mapped = "".join(BYTE_ENCODER[b] for b in word.encode("utf-8"))
        pieces = bpe_merge(list(mapped), self.ranks)
        ids = []
        for p in pieces:
            i = self.vocab.get(p)
            if i is None:
                # unknown merged piece: fall back to its single byte symbols
                for ch in p:
                    j = self.vocab.get(ch, self.unk_id)
                    if j is not None:
                        ids.append(j)
            else:
                ids.append(i)
        if len(self._cache) < 100_000:
            self._cache[word] = ids
        return ids

    def encode(self, text: str) -> List[int]:
        words = self.split.findall(text) if self.split is not None else [text]
        out: List[int] = []
        for w in words:
            out.extend(self._word(w))
        return out

    def decode(self, pieces: Sequence[str]) -> str:
        text = "".join(pieces)
        if _BYTE_CHARS.issuperset(text):  # every character is a byte symbol: translate and re-read as UTF-8
            return text.translate(_TO_LATIN1).encode("latin-1").decode("utf-8", errors="replace")
        data = bytearray()
        for p in pieces:
            for ch in p:
                b = BYTE_DECODER.get(ch)
                if b is None:
                    data.extend(ch.encode("utf-8"))
                else:
                    data.append(b)
        return data.decode("utf-8", errors="replace")


def _byte_piece(b: int) -> str:
    return f"<0x{b:02X}>"


class MetaspaceBpe(Codec):
    """SentencePiece-style BPE: ' ' -> U+2581, optional prefix, byte fallback.  ``scores`` (GGUF llama vocab)
    orders merges by the score of the merged piece when no merge list exists."""

    def __init__(self, vocab: Dict[str, int], merges: Optional[List[Tuple[str, str]]] = None,
                 scores: Optional[List[float]] = None, add_prefix: bool = True, byte_fallback: bool = True,
                 unk_id: Optional[int] = None, split_on_space: bool = False):
        self.vocab = vocab
        self.id_to_piece = {v: k for k, v in vocab.items()}
        self.ranks = {m: i for i, m in enumerate(merges)} if merges else None
        self.scores = scores
        self.add_prefix = add_prefix
        self.byte_fallback = byte_fallback
        self.unk_id = unk_id
        self.split_on_space = split_on_space
        # Merges never cross a boundary "x|▁" (x not ▁) when no piece holds a non-▁ character followed by ▁: the
        # text can then be cut there and each piece merged alone with the same result (and cached), instead of
        # running the merge over the whole text, whose cost grows with the square of its length.
        inner = regex.compile(f"[^{SPIECE}]{SPIECE}")
        self._chunk_safe = not any(inner.search(p) for p in vocab) and \
            not any(inner.search(a + b) for a, b in (self.ranks or ()))
        self._cut = regex.compile(f"(?<=[^{SPIECE}])(?={SPIECE})")
        self._cache: Dict[str, List[int]] = {}

    def _merge_by_score(self, symbols: List[str]) -> List[str]:
        """Highest-scoring adjacent merge first (leftmost among equal scores), one merge at a time, with a heap
        of candidate pairs over a linked list of symbols: O(n log n) for a whole unsplit text."""
        n = len(symbols)
        if n < 2:
            return symbols
        sym = list(symbols)
        nxt = list(range(1, n + 1))
        nxt[-1] = -1
        prv = list(range(-1, n - 1))
        alive = [True] * n
        vocab, scores = self.vocab, self.scores
        heap: List[Tuple[float, int, int, str]] = []

        def push(i: int) -> None:
            j = nxt[i]
            if j < 0:
                return
            cand = sym[i] + sym[j]
            k = vocab.get(cand)
            if k is not None:
                sc = scores[k] if scores is not None and k < len(scores) else 0.0
                heapq.heappush(heap, (-sc, i, j, cand))

        for i in range(n - 1):
            push(i)
        while heap:
            _, i, j, cand = heapq.heappop(heap)
            if not (alive[i] and alive[j] and nxt[i] == j and sym[i] + sym[j] == cand):
                continue  # stale: a neighbour merged since this pair was queued
            sym[i] = cand
            alive[j] = False
            nxt[i] = nxt[j]
            if nxt[j] >= 0:
                prv[nxt[j]] = i
            if prv[i] >= 0:
                push(prv[i])
            push(i)
        out, i = [], 0
        while i >= 0:
            out.append(sym[i])
            i = nxt[i]
        return out

    def _merge_by_score_rounds(self, symbols: List[str]) -> List[str]:
        """Reference form of ``_merge_by_score``: rescan every adjacent pair per merge (quadratic; for tests)."""
        while len(symbols) > 1:
            best = None
            best_score = None
            for i in range(len(symbols) - 1):
                cand = symbols[i] + symbols[i + 1]
                j = self.vocab.get(cand)
                if j is not None:
                    s = self.scores[j] if self.scores is not None and j < len(self.scores) else 0.0
                    if best_score is None or s > best_score:
                        best_score, best = s, i
            if best is None:
                break
            symbols = symbols[:best] + [symbols[best] + symbols[best + 1]] + symbols[best + 2:]
        return symbols

    def _pieces_to_ids(self, pieces: List[str]) -> List[int]:
        out = []
        for p in pieces:
            i = self.vocab.get(p)
            if i is not None:
                out.append(i)
            elif self.byte_fallback:
                for b in p.encode("utf-8"):
                    j = self.vocab.get(_byte_piece(b))
                    if j is not None:
                        out.append(j)
                    elif self.unk_id is not None:
                        out.append(self.unk_id)
            elif self.unk_id is not None:
                out.append(self.unk_id)
        return out

    def encode(self, text: str) -> List[int]:
        if not text:
            return []
        t = text.replace(" ", SPIECE)
        if self.add_prefix and not t.startswith(SPIECE):
            t = SPIECE + t
        chunks = [t]
        if self.split_on_space:
            chunks = [c for c in regex.split(f"(?={SPIECE})", t) if c]
        elif self._chunk_safe:
            chunks = [c for c in self._cut.split(t) if c]
        out: List[int] = []
        cache = self._cache
        for c in chunks:
            ids = cache.get(c)
            if ids is None:
                syms = list(c)
                syms = bpe_merge(syms, self.ranks) if self.ranks is not None else self._merge_by_score(syms)
                ids = self._pieces_to_ids(syms)
                if len(cache) < 100_000 and len(c) <= 256:
                    cache[c] = ids
            out.extend(ids)
        return out

    def decode(self, pieces: Sequence[str]) -> str:
        data = bytearray()
        for p in pieces:
            if len(p) == 6 and p.startswith("<0x") and p.endswith(">"):
                try:
                    data.append(int(p[3:5], 16))
                    continue
                except ValueError:
                    pass
            data.extend(p.replace(SPIECE, " ").encode("utf-8"))
        s = data.decode("utf-8", errors="replace")
        return s[1:] if (self.add_prefix and s.startswith(" ")) else s


def _is_punct(ch: str) -> bool:
    cp = ord(ch)
    if 33 <= cp <= 47 or 58 <= cp <= 64 or 91 <= cp <= 96 or 123 <= cp <= 126:
        return True
    return unicodedata.category(ch).startswith("P")


def _is_cjk(cp: int) -> bool:
    return (0x4E00 <= cp <= 0x9FFF or 0x3400 <= cp <= 0x4DBF or 0x20000 <= cp <= 0x2A6DF or 0x2A700 <= cp <= 0x2B73F
            or 0x2B740 <= cp <= 0x2B81F or 0x2B820 <= cp <= 0x2CEAF or 0xF900 <= cp <= 0xFAFF or
            0x2F800 <= cp <= 0x2FA1F)


# ASCII fast path of the BERT basic tokeniser: runs of ASCII are cleaned by one str.translate (control characters
# are category Cc and dropped; tab / newline / CR stay as whitespace) and split into words and single punctuation
# characters by one regex, at C speed; the other characters take the per-character path below.
_ASCII_CLEAN = {c: None for c in list(range(0, 9)) + [11, 12] + list(range(14, 32)) + [127]}
_ASCII_PUNCT = r"!-/:-@\[-`{-~"
_ASCII_WORDS = regex.compile(rf"[{_ASCII_PUNCT}]|[^\s{_ASCII_PUNCT}]+")
_ASCII_RUN = regex.compile(r"([\x00-\x7f]+)")


def bert_basic_tokenize(text: str, lowercase: bool = True, strip_accents: Optional[bool] = None) -> List[str]:
    """BERT basic tokenisation: drop control characters, space out CJK ideographs, split on whitespace, optional
    lower-case and accent strip, then split off every punctuation character."""
    if text.isascii():
        t = text.translate(_ASCII_CLEAN)
        return _ASCII_WORDS.findall(t.lower() if lowercase else t)
    parts = _ASCII_RUN.split(text)  # non-ASCII runs at even indices, ASCII runs at odd ones
    for i in range(1, len(parts), 2):
        parts[i] = parts[i].translate(_ASCII_CLEAN)
    for i in range(0, len(parts), 2):
        if parts[i]:
            parts[i] = _clean_chars(parts[i])
    words = []
    strip = strip_accents or (strip_accents is None and lowercase)
    for w in "".join(parts).split():
        if w.isascii():
            words.extend(_ASCII_WORDS.findall(w.lower() if lowercase else w))
            continue
        if lowercase:
            w = w.lower()
        if strip:
            w = "".join(c for c in unicodedata.normalize("NFD", w) if unicodedata.category(c) != "Mn")
        cur = ""
        for ch in w:
            if _is_punct(ch):
                if cur:
                    words.append(cur)
                    cur = ""
                words.append(ch)
            else:
                cur += ch
        if cur:
            words.append(cur)
    return words


def _clean_chars(text: str) -> str:
    out = []
    for ch in text:
        cp = ord(ch)
        if cp == 0 or cp == 0xFFFD or (unicodedata.category(ch).startswith("C") and ch not in "\t\n\r"):
            continue
        if _is_cjk(cp):
            out.append(f" {ch} ")
        elif ch in "\t\n\r" or unicodedata.category(ch) == "Zs":
            out.append(" ")
        else:
            out.append(ch)
    return "".join(out)


class WordPiece(Codec):
    def __init__(self, vocab: Dict[str, int], unk_token: str = "[UNK]", prefix: str = "##",
                 lowercase: bool = True, strip_accents: Optional[bool] = None, max_chars: int = 100):
        self.vocab = vocab
        self.unk_id = vocab.get(unk_token, 0)
        self.prefix = prefix
        self.lowercase = lowercase
        self.strip_accents = strip_accents
        self.max_chars = max_chars
        self._cache: Dict[str, List[int]] = {}

    def _word(self, w: str) -> List[int]:
        hit = self._cache.get(w)
        if hit is not None:
            return hit
        ids = self._match(w)
        if len(self._cache) < 200_000:
            self._cache[w] = ids
        return ids

    def _match(self, w: str) -> List[int]:
        if len(w) > self.max_chars:
            return [self.unk_id]
        out = []
        start = 0
        while start < len(w):
            end = len(w)
            found = None
            while start < end:
                sub = w[start:end]
                if start > 0:
                    sub = self.prefix + sub
                if sub in self.vocab:
                    found = self.vocab[sub]
                    break
                end -= 1
            if found is None:
                return [self.unk_id]
            out.append(found)
            start = end
        return out

    def encode(self, text: str) -> List[int]:
        out: List[int] = []
        for w in bert_basic_tokenize(text, self.lowercase, self.strip_accents):
            out.extend(self._word(w))
        return out

    def decode(self, pieces: Sequence[str]) -> str:
        s = ""
        for p in pieces:
            if p.startswith(self.prefix):
                s += p[len(self.prefix):]
            else:
                s += (" " if s else "") + p
        return s


class Unigram(Codec):
    """Viterbi segmentation maximising the sum of piece log-probabilities (SentencePiece unigram)."""

    def __init__(self, pieces: List[Tuple[str, float]], unk_id: Optional[int] = 0, byte_fallback: bool = False,
                 add_prefix: bool = True, normalizer=None):
        self.pieces = pieces
        self.vocab = {p: i for i, (p, _) in enumerate(pieces)}
        self.scores = [s for _, s in pieces]
        self.unk_id = unk_id
        self.byte_fallback = byte_fallback
        self.add_prefix = add_prefix
        self.normalizer = normalizer
        self.max_len = max((len(p) for p, _ in pieces), default=1)
        finite = [s for s in self.scores if s > -1e30]
        self.unk_penalty = (min(finite) if finite else 0.0) - 10.0

    def encode(self, text: str) -> List[int]:
        if self.normalizer is not None:
            text = self.normalizer(text)
        if not text:
            return []
        t = text.replace(" ", SPIECE)
        if self.add_prefix and not t.startswith(SPIECE):
            t = SPIECE + t
        n = len(t)
        best = [float("-inf")] * (n + 1)
        back: List[Optional[Tuple[int, int]]] = [None] * (n + 1)
        best[0] = 0.0
        for i in range(n):
            if best[i] == float("-inf"):
                continue
            matched = False
            for j in range(i + 1, min(n, i + self.max_len) + 1):
                pid = self.vocab.get(t[i:j])
                if pid is not None:
                    matched = True
                    sc = best[i] + self.scores[pid]
                    if sc > best[j]:
                        best[j], back[j] = sc, (i, pid)
            if not matched or best[i + 1] == float("-inf"):
                sc = best[i] + self.unk_penalty
                if sc > best[i + 1]:
                    best[i + 1], back[i + 1] = sc, (i, -1)
        out: List[int] = []
        j = n
        while j > 0:
            i, pid = back[j]
            if pid == -1:
                ch = t[i:j]
                if self.byte_fallback:
                    ids = [self.vocab.get(_byte_piece(b)) for b in ch.encode("utf-8")]
                    if all(x is not None for x in ids):
                        out.extend(reversed(ids))
                    elif self.unk_id is not None:
                        out.append(self.unk_id)
                elif self.unk_id is not None:
                    if not out or out[-1] != self.unk_id:
                        out.append(self.unk_id)
            else:
                out.append(pid)
            j = i
        out.reverse()
        return out

    def decode(self, pieces: Sequence[str]) -> str:
        data = bytearray()
        for p in pieces:
            if len(p) == 6 and p.startswith("<0x") and p.endswith(">"):
                try:
                    data.append(int(p[3:5], 16))
                    continue
                except ValueError:
                    pass
            data.extend(p.replace(SPIECE, " ").encode("utf-8"))
        s = data.decode("utf-8", errors="replace")
        return s[1:] if (self.add_prefix and s.startswith(" ")) else s


class WordLevel(Codec):
    def __init__(self, vocab: Dict[str, int], unk_token: str = "[UNK]", pattern: str = r"\w+|[^\w\s]+"):
        self.vocab = vocab
        self.unk_id = vocab.get(unk_token, 0)
        self.split = regex.compile(pattern)

    def encode(self, text: str) -> List[int]:
        return [self.vocab.get(w, self.unk_id) for w in self.split.findall(text)]

    def decode(self, pieces: Sequence[str]) -> str:
        return " ".join(pieces)


class Char(Codec):
    def __init__(self, vocab: Dict[str, int], unk_id: int = 0):
        self.vocab = vocab
        self.unk_id = unk_id

    def encode(self, text: str) -> List[int]:
        return [self.vocab.get(c, self.unk_id) for c in text]

    def decode(self, pieces: Sequence[str]) -> str:
        return "".join(pieces)
