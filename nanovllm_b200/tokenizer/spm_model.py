"""SentencePiece ``tokenizer.model`` (protobuf ModelProto) reader.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/tokenizer/SentencePieceModel.java:1-300.
Fields used: pieces (1: piece, score, type), trainer_spec (2: model_type 3, byte_fallback 35, unk/bos/eos/pad ids
40-43) and normalizer_spec (3: precompiled charsmap 2, add_dummy_prefix 3, remove_extra_whitespaces 4).  Unigram
models decode with Viterbi, BPE models with score-ordered merges.
"""
from __future__ import annotations

from typing import Optional, Sequence

from ..exceptions import ModelLoadException
from ..utils import protowire as pw
from . import codecs as C

NORMAL, UNKNOWN, CONTROL, USER_DEFINED, UNUSED, BYTE = 1, 2, 3, 4, 5, 6
UNIGRAM, BPE, WORD, CHAR = 1, 2, 3, 4


def parse_model(data: bytes) -> dict:
    pieces = []
    trainer = {"model_type": UNIGRAM, "byte_fallback": False, "unk_id": 0, "bos_id": 1, "eos_id": 2, "pad_id": -1}
    norm = {"charsmap": b"", "add_dummy_prefix": True, "remove_extra_whitespaces": True}
    for f, wt, v in pw.iter_fields(data):
        if f == 1 and wt == pw.LEN:
            piece, score, typ = "", 0.0, NORMAL
            for f2, w2, v2 in pw.iter_fields(v):
                if f2 == 1:
                    piece = pw.as_str(v2)
                elif f2 == 2:
                    score = pw.as_float(v2)
                elif f2 == 3:
                    typ = v2
            pieces.append((piece, score, typ))
        elif f == 2 and wt == pw.LEN:
            for f2, w2, v2 in pw.iter_fields(v):
                if f2 == 3:
                    trainer["model_type"] = v2
                elif f2 == 35:
                    trainer["byte_fallback"] = bool(v2)
                elif f2 == 40:
                    trainer["unk_id"] = pw.signed64(v2) if v2 >= (1 << 63) else v2
                elif f2 == 41:
                    trainer["bos_id"] = pw.signed64(v2)
                elif f2 == 42:
                    trainer["eos_id"] = pw.signed64(v2)
                elif f2 == 43:
                    trainer["pad_id"] = pw.signed64(v2)
        elif f == 3 and wt == pw.LEN:
            for f2, w2, v2 in pw.iter_fields(v):
                if f2 == 2:
                    norm["charsmap"] = bytes(v2)
                elif f2 == 3:
                    norm["add_dummy_prefix"] = bool(v2)
                elif f2 == 4:
                    norm["remove_extra_whitespaces"] = bool(v2)
    if not pieces:
        raise ModelLoadException("SentencePiece model has no pieces")
    return {"pieces": pieces, "trainer": trainer, "normalizer": norm}


def load_sentencepiece(path: str, tokenizer_config: Optional[dict] = None, extra_eos: Sequence[int] = ()):
    from .charsmap import PrecompiledCharsMap
    from .tokenizer import Tokenizer
    with open(path, "rb") as f:
        m = parse_model(f.read())
    pieces = m["pieces"]
    tr, nm = m["trainer"], m["normalizer"]
    tokens = [p for p, _, _ in pieces]
    scores = [s for _, s, _ in pieces]
    vocab = {t: i for i, t in enumerate(tokens)}
    special = {i for i, (_, _, t) in enumerate(pieces) if t in (CONTROL, USER_DEFINED, UNKNOWN)}
    added = {p: i for i, (p, _, t) in enumerate(pieces) if t in (CONTROL, USER_DEFINED) and p}
    cm = PrecompiledCharsMap(nm["charsmap"]) if nm["charsmap"] else None
    norms = []
    if cm is not None:
        norms.append(cm.normalize)
    if nm["remove_extra_whitespaces"]:
        norms.append(lambda t: " ".join(t.split()))
    unk = tr["unk_id"] if tr["unk_id"] >= 0 else None
    if tr["model_type"] == BPE:
        codec = C.MetaspaceBpe(vocab, None, scores, add_prefix=nm["add_dummy_prefix"],
                               byte_fallback=tr["byte_fallback"], unk_id=unk)
    elif tr["model_type"] == CHAR:
        codec = C.Char(vocab, unk or 0)
    elif tr["model_type"] == WORD:
        codec = C.WordLevel(vocab, tokens[unk] if unk is not None else "<unk>")
    else:
        codec = C.Unigram([(p, s) for p, s, _ in pieces], unk, tr["byte_fallback"], add_prefix=nm["add_dummy_prefix"])
    tc = tokenizer_config or {}
    bos = tr["bos_id"] if tr["bos_id"] >= 0 else None
    eos = tr["eos_id"] if tr["eos_id"] >= 0 else None
    return Tokenizer(codec, tokens, special_ids=special, added=added, bos_id=bos, eos_id=eos,
                     pad_id=tr["pad_id"] if tr["pad_id"] >= 0 else None, unk_id=unk, extra_eos=extra_eos,
                     chat_template=tc.get("chat_template") if isinstance(tc.get("chat_template"), str) else None,
                     normalizers=norms, add_bos=bool(tc.get("add_bos_token", True)), metaspace=True)
