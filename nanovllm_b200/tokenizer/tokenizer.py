"""``Tokenizer``: the public tokenizer façade and its loaders.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/tokenizer/Tokenizer.java:79-449 and
TokenizerLoader.java:34-504:
* loading: a folder's ``tokenizer.json`` (HF tokenizers format), else ``tokenizer.model`` (SentencePiece), plus
  ``tokenizer_config.json`` / ``generation_config.json`` / ``config.json`` for special tokens and EOS ids; GGUF
  metadata (``tokenizer.ggml.*``: gpt2 byte-BPE, llama SentencePiece, bert WordPiece, t5 unigram);
* added / special tokens are atomic in ``encode`` (matched before the codec sees the text);
* ``decode`` optionally skips special tokens; ``StreamDecoder`` emits only complete UTF-8 characters;
* stop ids: EOS, then ``<|endoftext|>``, ``<eos>``, ``<end_of_turn>``, ``<turn|>``, ``<|im_end|>`` when present,
  then generation_config EOS ids (TokenizerLoader.java:485-504);
* chat format detection (ChatML, Gemma ``<start_of_turn>`` / Gemma4 ``<|turn>`` turns, plain) and the hand-coded
  templates of Tokenizer.java:311-435 -- including the ChatML "think-skip" seed ``<think>\\n\\n</think>\\n\\n`` when
  thinking is off but the vocabulary has both tags, and Gemma's folding of the system text into the first user
  turn.  There is no Jinja.
"""
from __future__ import annotations

import json
import os
import unicodedata
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import regex

from ..exceptions import ModelLoadException
from ..utils.limits import ResourceLimits
from . import codecs as C

CHATML, TURN_BASED, PLAIN = "chatml", "turn_based", "plain"


class Tokenizer:
    def __init__(self, codec: C.Codec, id_to_token: List[str], *, special_ids: Iterable[int] = (),
                 added: Optional[Dict[str, int]] = None, bos_id: Optional[int] = None, eos_id: Optional[int] = None,
                 pad_id: Optional[int] = None, unk_id: Optional[int] = None, extra_eos: Sequence[int] = (),
                 chat_template: Optional[str] = None, normalizers: Sequence = (), add_bos: bool = False,
                 cls_id: Optional[int] = None, sep_id: Optional[int] = None, metaspace: bool = False):
        self.codec = codec
        self.id_to_token = id_to_token
        self.vocab = {t: i for i, t in enumerate(id_to_token) if t is not None}
        self.special_ids = set(special_ids)
        self.added = dict(added or {})
        for t, i in self.added.items():
            self.vocab.setdefault(t, i)
        self.bos_id, self.pad_id, self.unk_id = bos_id, pad_id, unk_id
        self.eos_id = eos_id if eos_id is not None else -1
        self.chat_template = chat_template
        self.normalizers = list(normalizers)
        self.add_bos = add_bos
        self.cls_id, self.sep_id = cls_id, sep_id
        self._added_sorted = sorted(self.added.keys(), key=len, reverse=True)
        # leftmost match, longest token first at a position: one alternation in that order scans at C speed
        self._added_re = (regex.compile("|".join(regex.escape(t) for t in self._added_sorted))
                          if self._added_sorted else None)
        self.stop_ids = self._stop_ids(extra_eos)
        self.chat_format = self._detect_format(metaspace)

    # ------------------------------------------------------------------ basics
    @property
    def vocab_size(self) -> int:
        return len(self.id_to_token)

    def token_id(self, token: str) -> Optional[int]:
        return self.vocab.get(token)

    def token(self, i: int) -> Optional[str]:
        return self.id_to_token[i] if 0 <= i < len(self.id_to_token) else None

    def eos_token_id(self) -> int:
        return self.eos_id

    def pad_token_id(self) -> int:
        return self.pad_id if self.pad_id is not None else self.eos_id

    def stop_token_ids(self) -> List[int]:
        return list(self.stop_ids)

    def _stop_ids(self, extra: Sequence[int]) -> List[int]:
        ids = [self.eos_id] if self.eos_id is not None and self.eos_id >= 0 else []
        for t in ("<|endoftext|>", "<eos>", "<end_of_turn>", "<turn|>", "<|im_end|>"):
            i = self.vocab.get(t)
            if i is not None and i not in ids:
                ids.append(i)
        for i in extra:
            if i is not None and i >= 0 and i not in ids:
                ids.append(int(i))
        return ids

    # ------------------------------------------------------------------ encode / decode
    def _normalize(self, text: str) -> str:
        for n in self.normalizers:
            text = n(text)
        return text

    def _split_added(self, text: str) -> List[Tuple[str, bool]]:
        if not self._added_sorted:
            return [(text, False)]
        out: List[Tuple[str, bool]] = []
        start = 0
        for m in self._added_re.finditer(text):
            if start < m.start():
                out.append((text[start:m.start()], False))
            out.append((m.group(0), True))
            start = m.end()
        if start < len(text):
            out.append((text[start:], False))
        return out

    def encode(self, text: str, allow_special: bool = True, add_bos: Optional[bool] = None) -> List[int]:
        ids: List[int] = []
        if (self.add_bos if add_bos is None else add_bos) and self.bos_id is not None:
            ids.append(self.bos_id)
        segs = self._split_added(text) if allow_special else [(text, False)]
        for seg, is_added in segs:
            if is_added:
                ids.append(self.added[seg])
            elif seg:
                ids.extend(self.codec.encode(self._normalize(seg)))
        return ids

    def decode(self, ids: Sequence[int], skip_special: bool = False) -> str:
        out = []
        buf: List[str] = []
        for i in ids:
            i = int(i)
            if skip_special and i in self.special_ids:
                continue
            tok = self.token(i)
            if tok is None:
                continue
            if tok in self.added and i in self.special_ids:
                if buf:
                    out.append(self.codec.decode(buf))
                    buf = []
                out.append(tok)
            else:
                buf.append(tok)
        if buf:
            out.append(self.codec.decode(buf))
        return "".join(out)

    def stream_decoder(self, skip_special: bool = True) -> "StreamDecoder":
        return StreamDecoder(self, skip_special)

    # ------------------------------------------------------------------ chat
    def _detect_format(self, metaspace: bool) -> str:
        tpl = self.chat_template or ""
        if "<|turn>" in tpl or "<|turn>" in self.vocab:
            return TURN_BASED
        if "start_of_turn" in tpl or "<start_of_turn>" in self.vocab:
            return TURN_BASED
        if "<|im_start|>" in tpl or "<|im_start|>" in self.vocab:
            return CHATML
        if metaspace and "<bos>" in self.vocab:
            return TURN_BASED
        return PLAIN

    def is_turn_based_chat(self) -> bool:
        return self.chat_format == TURN_BASED

    def invites_thinking(self, think_open: str = "<think>", think_close: str = "</think>") -> bool:
        return think_open in self.vocab and think_close in self.vocab

    def skip_special_tokens_on_chat_decode(self) -> bool:
        return True

    def apply_chat_template(self, messages, add_generation_prompt: bool = True, enable_thinking: bool = False,
                            think_open: str = "<think>", think_close: str = "</think>") -> str:
        msgs = [m if isinstance(m, dict) else {"role": m.role, "content": m.content} for m in messages]
        if self.chat_format == TURN_BASED:
            if "<|turn>" in self.vocab or "<|turn>" in (self.chat_template or ""):
                return self._angle_turns(msgs, add_generation_prompt, enable_thinking)
            return self._gemma_turns(msgs, add_generation_prompt)
        if self.chat_format == CHATML:
            s = "".join(f"<|im_start|>{m.get('role', 'user')}\n{m.get('content', '')}<|im_end|>\n" for m in msgs)
            if add_generation_prompt:
                s += "<|im_start|>assistant\n"
                if not enable_thinking and self.invites_thinking(think_open, think_close):
                    s += f"{think_open}\n\n{think_close}\n\n"
            return s
        s = "".join(f"{m.get('role', 'user')}: {m.get('content', '')}\n" for m in msgs)
        if add_generation_prompt:
            s += "assistant: "
        return s

    def _gemma_turns(self, msgs, add_generation_prompt: bool) -> str:
        system = None
        turns = []
        for m in msgs:
            if m.get("role") == "system":
                system = m.get("content", "")
            else:
                turns.append(m)
        s = "<bos>" if "<bos>" in self.vocab else ""
        first_user = True
        for m in turns:
            role = "model" if m.get("role") == "assistant" else m.get("role", "user")
            content = m.get("content", "")
            if role == "user":
                if first_user and system and system.strip():
                    content = f"{system}\n\n{content}"
                first_user = False
            s += f"<start_of_turn>{role}\n{content}<end_of_turn>\n"
        if add_generation_prompt:
            s += "<start_of_turn>model\n"
        return s

    def _angle_turns(self, msgs, add_generation_prompt: bool, enable_thinking: bool) -> str:
        system = None
        turns = []
        for m in msgs:
            if m.get("role") in ("system", "developer"):
                system = m.get("content", "")
            else:
                turns.append(m)
        s = "<bos>" if "<bos>" in self.vocab else ""
        if enable_thinking or (system and system.strip()):
            s += "<|turn>system\n"
            if enable_thinking:
                s += "<|think|>\n"
            if system and system.strip():
                s += system.strip()
            s += "<turn|>\n"
        for m in turns:
            role = "model" if m.get("role") == "assistant" else m.get("role", "user")
            s += f"<|turn>{role}\n{m.get('content', '').strip()}<turn|>\n"
        if add_generation_prompt:
            s += "<|turn>model\n"
        return s

    # ------------------------------------------------------------------ embeddings
    def cls_sep_ids(self) -> Tuple[Optional[int], Optional[int]]:
        if self.cls_id is not None or self.sep_id is not None:
            return self.cls_id, self.sep_id
        for a, b in (("[CLS]", "[SEP]"), ("<s>", "</s>")):
            if a in self.vocab and b in self.vocab:
                return self.vocab[a], self.vocab[b]
        return self.bos_id, (self.eos_id if self.eos_id is not None and self.eos_id >= 0 else None)

    # ------------------------------------------------------------------ loaders
    @staticmethod
    def from_pretrained(model_dir: str) -> "Tokenizer":
        return _load_folder(model_dir)

    @staticmethod
    def from_gguf(meta: dict) -> "Tokenizer":
        return _load_gguf(meta)

    @staticmethod
    def from_sentencepiece(path: str, **kw) -> "Tokenizer":
        from .spm_model import load_sentencepiece
        return load_sentencepiece(path, **kw)

    @staticmethod
    def from_json(tokenizer_json: dict, tokenizer_config: Optional[dict] = None, extra_eos: Sequence[int] = ()):
        return _from_tokenizer_json(tokenizer_json, tokenizer_config or {}, extra_eos)


class StreamDecoder:
    """Incremental detokeniser that only emits text once the bytes form complete UTF-8 characters.

    A push decodes only the tokens since the previous emission plus the ones before it back to the emission
    before that (``prefix`` .. end), and emits what that window decodes to beyond its already-emitted part
    (``prefix`` .. ``read``).  Both decodes start at the same token, so word joins, leading-space rules and
    multi-byte characters come out as in a decode of the whole reply, at a cost that does not grow with the
    reply's length."""

    def __init__(self, tok: Tokenizer, skip_special: bool = True):
        self.tok = tok
        self.skip = skip_special
        self.ids: List[int] = []
        self.prefix = 0  # window start: a token boundary whose preceding text is emitted
        self.read = 0    # tokens whose text is emitted

    def push(self, token_id: int) -> str:
        self.ids.append(int(token_id))
        head = self.tok.decode(self.ids[self.prefix:self.read], self.skip)
        full = self.tok.decode(self.ids[self.prefix:], self.skip)
        # hold back a trailing replacement character: it is usually an incomplete multi-byte sequence
        if len(full) <= len(head) or full.endswith("\ufffd"):
            return ""
        self.prefix, self.read = self.read, len(self.ids)
        return full[len(head):]

    def flush(self) -> str:
        head = self.tok.decode(self.ids[self.prefix:self.read], self.skip)
        full = self.tok.decode(self.ids[self.prefix:], self.skip)
        self.prefix = self.read = len(self.ids)
        return full[len(head):]


def utf8_complete_prefix(data: bytes) -> Tuple[str, bytes]:
    """Split bytes into (decoded complete characters, incomplete tail)."""
    cut = len(data)
    i = len(data) - 1
    back = 0
    while i >= 0 and back < 4:
        b = data[i]
        if b & 0xC0 == 0x80:
            i -= 1
            back += 1
            continue
        need = 1 if b < 0x80 else 2 if b >> 5 == 0x6 else 3 if b >> 4 == 0xE else 4 if b >> 3 == 0x1E else 1
        if len(data) - i < need:
            cut = i
        break
    return data[:cut].decode("utf-8", errors="replace"), data[cut:]


# ----------------------------------------------------------------------------------------------- folder loader
def _read_json(path: str) -> Optional[dict]:
    if not os.path.isfile(path):
        return None
    from ..utils.json_limits import load_file
    return load_file(path)


def _token_content(v):
    if isinstance(v, dict):
        return v.get("content")
    return v


def _eos_list(v) -> List[int]:
    if v is None:
        return []
    if isinstance(v, list):
        return [int(x) for x in v]
    return [int(v)]


def _load_folder(d: str) -> Tokenizer:
    tj = _read_json(os.path.join(d, "tokenizer.json"))
    tc = _read_json(os.path.join(d, "tokenizer_config.json")) or {}
    gc = _read_json(os.path.join(d, "generation_config.json")) or {}
    cfg = _read_json(os.path.join(d, "config.json")) or {}
    extra = _eos_list(gc.get("eos_token_id")) + _eos_list(cfg.get("eos_token_id"))
    if tj is not None:
        return _from_tokenizer_json(tj, tc, extra)
    spm = os.path.join(d, "tokenizer.model")
    if os.path.isfile(spm):
        from .spm_model import load_sentencepiece
        return load_sentencepiece(spm, tokenizer_config=tc, extra_eos=extra)
    raise ModelLoadException(f"no tokenizer.json or tokenizer.model in {d}")


def _normalizer_fns(spec) -> Tuple[List, bool, bool]:
    """-> (functions, lowercase flag for WordPiece, has_precompiled)"""
    fns = []
    lower = False
    if not spec:
        return fns, lower, False
    kind = spec.get("type")
    if kind == "Sequence":
        pre = False
        for s in spec.get("normalizers", []):
            f, l2, p2 = _normalizer_fns(s)
            fns += f
            lower = lower or l2
            pre = pre or p2
        return fns, lower, pre
    if kind in ("NFC", "NFD", "NFKC", "NFKD"):
        fns.append(lambda t, k=kind: unicodedata.normalize(k, t))
    elif kind == "Lowercase":
        fns.append(str.lower)
        lower = True
    elif kind == "BertNormalizer":
        lower = bool(spec.get("lowercase", True))
    elif kind == "Replace":
        pat = spec.get("pattern", {})
        src = pat.get("String") if isinstance(pat, dict) else None
        dst = spec.get("content", "")
        if src is not None:
            fns.append(lambda t, a=src, b=dst: t.replace(a, b))
        elif isinstance(pat, dict) and pat.get("Regex"):
            import regex
            rx = regex.compile(pat["Regex"])
            fns.append(lambda t, r=rx, b=dst: r.sub(b, t))
    elif kind == "Prepend":
        p = spec.get("prepend", "")
        fns.append(lambda t, pp=p: pp + t if t else t)
    elif kind == "StripAccents":
        fns.append(lambda t: "".join(c for c in unicodedata.normalize("NFD", t) if unicodedata.category(c) != "Mn"))
    elif kind == "Strip":
        fns.append(str.strip)
    elif kind == "Precompiled":
        from .charsmap import PrecompiledCharsMap
        import base64
        blob = spec.get("precompiled_charsmap")
        if blob:
            cm = PrecompiledCharsMap(base64.b64decode(blob))
            fns.append(cm.normalize)
        return fns, lower, True
    return fns, lower, False


def _pretok_info(spec) -> dict:
    info = {"byte_level": False, "pattern": None, "metaspace": False, "prepend": True, "bert": False,
            "split_ws": False}
    if not spec:
        return info
    kind = spec.get("type")
    if kind == "Sequence":
        for s in spec.get("pretokenizers", []):
            sub = _pretok_info(s)
            for k, v in sub.items():
                if v and k != "prepend":
                    info[k] = v
            if sub.get("metaspace"):
                info["prepend"] = sub["prepend"]
        return info
    if kind == "ByteLevel":
        info["byte_level"] = True
        if spec.get("use_regex", True) and info["pattern"] is None:
            info["pattern"] = C.GPT2_PATTERN
    elif kind == "Split":
        pat = spec.get("pattern", {})
        info["pattern"] = pat.get("Regex") if isinstance(pat, dict) and pat.get("Regex") else None
    elif kind == "Metaspace":
        info["metaspace"] = True
        info["prepend"] = spec.get("prepend_scheme", "always") != "never" and spec.get("add_prefix_space", True)
        info["split_ws"] = bool(spec.get("split", False))
    elif kind in ("BertPreTokenizer", "Whitespace", "WhitespaceSplit"):
        info["bert"] = True
    return info


def _from_tokenizer_json(tj: dict, tc: dict, extra_eos: Sequence[int]) -> Tokenizer:
    model = tj.get("model", {})
    mtype = model.get("type")
    norms, lower, precompiled = _normalizer_fns(tj.get("normalizer"))
    pre = _pretok_info(tj.get("pre_tokenizer"))
    dec = tj.get("decoder") or {}
    dec_kinds = json.dumps(dec)
    metaspace = pre["metaspace"] or "Metaspace" in dec_kinds or ("\\u2581" in dec_kinds or "▁" in dec_kinds)
    added = {}
    special = set()
    for a in tj.get("added_tokens", []) or []:
        added[a["content"]] = int(a["id"])
        if a.get("special", False):
            special.add(int(a["id"]))
    if mtype == "BPE":
        vocab = {k: int(v) for k, v in model.get("vocab", {}).items()}
        merges = []
        for m in model.get("merges", []):
            if isinstance(m, str):
                a, b = m.split(" ", 1)
            else:
                a, b = m
            merges.append((a, b))
        unk = model.get("unk_token")
        unk_id = vocab.get(unk) if unk else None
        if pre["byte_level"] or (not metaspace and "ByteLevel" in dec_kinds):
            codec = C.ByteBpe(vocab, merges, pre["pattern"] or C.GPT2_PATTERN, unk_id)
        else:
            # legacy SentencePiece-BPE exports use a Prepend + Replace normalizer instead of a Metaspace split
            has_prepend = "Prepend" in json.dumps(tj.get("normalizer") or {})
            codec = C.MetaspaceBpe(vocab, merges, None, add_prefix=(pre["prepend"] if pre["metaspace"] else False),
                                   byte_fallback=bool(model.get("byte_fallback", False)), unk_id=unk_id)
            if has_prepend:
                # the normalizer already prepended U+2581 and replaced spaces
                codec.add_prefix = False
    elif mtype == "WordPiece":
        vocab = {k: int(v) for k, v in model.get("vocab", {}).items()}
        normalizer = tj.get("normalizer") or {}
        lower = bool(normalizer.get("lowercase", lower)) if normalizer.get("type") == "BertNormalizer" else lower
        strip = normalizer.get("strip_accents") if normalizer.get("type") == "BertNormalizer" else None
        codec = C.WordPiece(vocab, model.get("unk_token", "[UNK]"), model.get("continuing_subword_prefix", "##"),
                            lowercase=lower, strip_accents=strip)
        norms = [f for f in norms if f is not str.lower]
    elif mtype == "Unigram":
        pieces = [(p, float(s)) for p, s in model.get("vocab", [])]
        vocab = {p: i for i, (p, _) in enumerate(pieces)}
        codec = C.Unigram(pieces, model.get("unk_id", 0), bool(model.get("byte_fallback", False)),
                          add_prefix=pre["prepend"] if pre["metaspace"] else True)
        metaspace = True
    elif mtype == "WordLevel":
        vocab = {k: int(v) for k, v in model.get("vocab", {}).items()}
        codec = C.WordLevel(vocab, model.get("unk_token", "[UNK]"))
    else:
        raise ModelLoadException(f"unsupported tokenizer.json model type {mtype!r}")
    size = max(list(vocab.values()) + list(added.values()) + [-1]) + 1
    id_to_token: List[Optional[str]] = [None] * size
    for t, i in vocab.items():
        id_to_token[i] = t
    for t, i in added.items():
        id_to_token[i] = t
    id_to_token = [t if t is not None else f"<unused{i}>" for i, t in enumerate(id_to_token)]

    def tid(name):
        v = _token_content(tc.get(name))
        return added.get(v, vocab.get(v)) if v is not None else None

    eos = tid("eos_token")
    if eos is None:
        for cand in ("<|endoftext|>", "</s>", "<eos>", "[SEP]"):
            if cand in added or cand in vocab:
                eos = added.get(cand, vocab.get(cand))
                break
    return Tokenizer(codec, id_to_token, special_ids=special, added=added, bos_id=tid("bos_token"), eos_id=eos,
                     pad_id=tid("pad_token"), unk_id=tid("unk_token"), extra_eos=extra_eos,
                     chat_template=tc.get("chat_template") if isinstance(tc.get("chat_template"), str) else None,
                     normalizers=norms, add_bos=bool(tc.get("add_bos_token", False)), cls_id=tid("cls_token"),
                     sep_id=tid("sep_token"), metaspace=metaspace)


# ----------------------------------------------------------------------------------------------- GGUF loader
def _load_gguf(meta: dict) -> Tokenizer:
    model = meta.get("tokenizer.ggml.model", "gpt2")
    tokens: List[str] = list(meta.get("tokenizer.ggml.tokens") or [])
    if not tokens:
        raise ModelLoadException("GGUF file has no tokenizer.ggml.tokens")
    types = list(meta.get("tokenizer.ggml.token_type") or [1] * len(tokens))
    scores = list(meta.get("tokenizer.ggml.scores") or [])
    vocab = {t: i for i, t in enumerate(tokens)}
    special = {i for i, ty in enumerate(types) if ty in (3, 4)}  # control, user-defined
    added = {tokens[i]: i for i, ty in enumerate(types) if ty in (3, 4) and tokens[i]}

    def g(key):
        v = meta.get(f"tokenizer.ggml.{key}")
        return int(v) if v is not None else None

    bos, eos, unk, pad = g("bos_token_id"), g("eos_token_id"), g("unknown_token_id"), g("padding_token_id")
    sep, cls = g("seperator_token_id"), g("cls_token_id")
    add_bos = bool(meta.get("tokenizer.ggml.add_bos_token", model == "llama"))
    tpl = meta.get("tokenizer.chat_template")
    metaspace = False
    if model == "gpt2":
        merges = []
        for m in meta.get("tokenizer.ggml.merges") or []:
            a, b = m.split(" ", 1)
            merges.append((a, b))
        pre = (meta.get("tokenizer.ggml.pre") or "default").lower()
        pattern = {"qwen2": C.QWEN2_PATTERN, "llama-bpe": C.LLAMA3_PATTERN, "llama3": C.LLAMA3_PATTERN,
                   "lfm2": C.LLAMA3_PATTERN, "smaug-bpe": C.LLAMA3_PATTERN}.get(pre, C.GPT2_PATTERN)
        codec = C.ByteBpe(vocab, merges, pattern, unk)
        add_bos = bool(meta.get("tokenizer.ggml.add_bos_token", False))
    elif model == "llama":
        codec = C.MetaspaceBpe(vocab, None, scores or [0.0] * len(tokens), add_prefix=True, byte_fallback=True,
                               unk_id=unk)
        metaspace = True
    elif model == "bert":
        codec = C.WordPiece(vocab, tokens[unk] if unk is not None else "[UNK]", "##", lowercase=True)
        add_bos = False
    elif model == "t5":
        codec = C.Unigram(list(zip(tokens, scores or [0.0] * len(tokens))), unk, True)
        metaspace = True
    else:
        raise ModelLoadException(f"unsupported GGUF tokenizer model {model!r}")
    return Tokenizer(codec, tokens, special_ids=special, added=added, bos_id=bos, eos_id=eos, pad_id=pad, unk_id=unk,
                     chat_template=tpl, add_bos=add_bos, cls_id=cls, sep_id=sep, metaspace=metaspace)
