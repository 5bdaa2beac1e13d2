"""Tokenizer codecs vs the HF ``tokenizers`` library (oracle) on tokenizers trained in-test, GGUF vocabularies,
special-token atomicity, streaming decode, stop ids and the hand-coded chat templates (reference analogues:
TokenizerCodecTest and the chat/template cases of CoreUnitTest)."""
import json
import os

import pytest

from nanovllm_b200.tokenizer.tokenizer import CHATML, PLAIN, TURN_BASED, Tokenizer

tk = pytest.importorskip("tokenizers")

CORPUS = [
    "The quick brown fox jumps over the lazy dog. Über naïve café! 東京タワー 123 4567.",
    "Hello, world! It's a test's test; we'll see: x=1+2*3 (ok?) \n\n  indented\tTabs",
    "Emoji 🙂🚀 and accents àéîõü, numbers 3.14159 and 2026, CAPS and MiXeD case.",
] * 20
SAMPLES = ["The quick brown fox", "Hello,  world!\n\nNew para", "naïve café 東京 🙂", "x=1+2*3 (ok?)",
           "  leading and trailing  ", "It's 2026; we'll see."]


def _save(t, tmp_path, name="tokenizer.json", config=None):
    d = tmp_path / name.replace(".json", "")
    d.mkdir()
    t.save(str(d / "tokenizer.json"))
    if config is not None:
        (d / "tokenizer_config.json").write_text(json.dumps(config))
    return str(d)


def _train_bytelevel(tmp_path):
    from tokenizers import Tokenizer as T, decoders, models, pre_tokenizers, trainers
    t = T(models.BPE())
    t.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    t.decoder = decoders.ByteLevel()
    t.train_from_iterator(CORPUS, trainers.BpeTrainer(vocab_size=400, special_tokens=["<|endoftext|>", "<|im_start|>",
                                                                                       "<|im_end|>", "<think>",
                                                                                       "</think>"],
                                                      initial_alphabet=pre_tokenizers.ByteLevel.alphabet()))
    return t


def test_byte_level_bpe_matches_oracle(tmp_path):
    t = _train_bytelevel(tmp_path)
    ours = Tokenizer.from_pretrained(_save(t, tmp_path, config={"eos_token": "<|endoftext|>"}))
    for s in SAMPLES:
        assert ours.encode(s) == t.encode(s).ids, s
        assert ours.decode(ours.encode(s)) == s


def test_special_tokens_are_atomic_and_chatml(tmp_path):
    t = _train_bytelevel(tmp_path)
    ours = Tokenizer.from_pretrained(_save(t, tmp_path, config={"eos_token": "<|endoftext|>"}))
    ids = ours.encode("<|im_start|>user\nhi<|im_end|>")
    assert ids[0] == ours.token_id("<|im_start|>") and ours.token_id("<|im_end|>") in ids
    assert ours.chat_format == CHATML
    p = ours.apply_chat_template([{"role": "user", "content": "hi"}], add_generation_prompt=True)
    assert p == "<|im_start|>user\nhi<|im_end|>\n<|im_start|>assistant\n<think>\n\n</think>\n\n"
    p2 = ours.apply_chat_template([{"role": "user", "content": "hi"}], enable_thinking=True)
    assert p2.endswith("<|im_start|>assistant\n")
    assert ours.stop_token_ids()[:2] == [ours.token_id("<|endoftext|>"), ours.token_id("<|im_end|>")]
    assert ours.decode(ids, skip_special=True) == "user\nhi"


def test_wordpiece_matches_oracle(tmp_path):
    from tokenizers import Tokenizer as T, decoders, models, normalizers, pre_tokenizers, trainers
    t = T(models.WordPiece(unk_token="[UNK]"))
    t.normalizer = normalizers.BertNormalizer(lowercase=True)
    t.pre_tokenizer = pre_tokenizers.BertPreTokenizer()
    t.decoder = decoders.WordPiece()
    t.train_from_iterator(CORPUS, trainers.WordPieceTrainer(vocab_size=300, special_tokens=["[UNK]", "[CLS]", "[SEP]",
                                                                                            "[PAD]", "[MASK]"]))
    ours = Tokenizer.from_pretrained(_save(t, tmp_path))
    for s in SAMPLES:
        assert ours.encode(s) == t.encode(s, add_special_tokens=False).ids, s
    assert ours.cls_sep_ids() == (t.token_to_id("[CLS]"), t.token_to_id("[SEP]"))


def test_unigram_and_metaspace_bpe_match_oracle(tmp_path):
    from tokenizers import Tokenizer as T, decoders, models, pre_tokenizers, trainers
    u = T(models.Unigram())
    u.pre_tokenizer = pre_tokenizers.Metaspace()
    u.decoder = decoders.Metaspace()
    u.train_from_iterator(CORPUS, trainers.UnigramTrainer(vocab_size=200, special_tokens=["<unk>"], unk_token="<unk>"))
    ours = Tokenizer.from_pretrained(_save(u, tmp_path, "uni.json"))
    for s in ["The quick brown fox", "lazy dog jumps", "Hello world"]:
        assert ours.encode(s) == u.encode(s).ids, s
        assert ours.decode(ours.encode(s)) == u.decode(u.encode(s).ids)
    b = T(models.BPE(byte_fallback=True, unk_token="<unk>"))
    b.pre_tokenizer = pre_tokenizers.Metaspace()
    b.decoder = decoders.Metaspace()
    b.train_from_iterator(CORPUS, trainers.BpeTrainer(vocab_size=300, special_tokens=["<unk>"] +
                                                      [f"<0x{i:02X}>" for i in range(256)]))
    ours_b = Tokenizer.from_pretrained(_save(b, tmp_path, "msp.json"))
    for s in ["The quick brown fox", "jumps over", "Hello, world!"]:
        assert ours_b.encode(s) == b.encode(s).ids, s


def test_gguf_gpt2_vocab_matches_json(tmp_path):
    t = _train_bytelevel(tmp_path)
    tj = json.loads(t.to_str())
    vocab = tj["model"]["vocab"]
    tokens = [None] * (max(vocab.values()) + 1)
    for k, v in vocab.items():
        tokens[v] = k
    for a in tj["added_tokens"]:
        tokens[a["id"]] = a["content"]
    types = [3 if a in ("<|endoftext|>", "<|im_start|>", "<|im_end|>", "<think>", "</think>") else 1 for a in tokens]
    merges = [m if isinstance(m, str) else " ".join(m) for m in tj["model"]["merges"]]
    meta = {"tokenizer.ggml.model": "gpt2", "tokenizer.ggml.pre": "default", "tokenizer.ggml.tokens": tokens,
            "tokenizer.ggml.token_type": types, "tokenizer.ggml.merges": merges,
            "tokenizer.ggml.eos_token_id": vocab.get("<|endoftext|>", 0)}
    g = Tokenizer.from_gguf(meta)
    for s in SAMPLES:
        assert g.encode(s) == t.encode(s).ids


def test_turn_based_and_plain_templates():
    from nanovllm_b200.tokenizer.codecs import Char
    vocab = {c: i for i, c in enumerate(["<bos>", "<start_of_turn>", "<end_of_turn>", "a", "b"])}
    tok = Tokenizer(Char(vocab), list(vocab.keys()), added={"<bos>": 0, "<start_of_turn>": 1, "<end_of_turn>": 2},
                    special_ids=[0, 1, 2], eos_id=2)
    assert tok.chat_format == TURN_BASED
    p = tok.apply_chat_template([{"role": "system", "content": "S"}, {"role": "user", "content": "U"},
                                 {"role": "assistant", "content": "A"}, {"role": "user", "content": "V"}])
    assert p == ("<bos><start_of_turn>user\nS\n\nU<end_of_turn>\n<start_of_turn>model\nA<end_of_turn>\n"
                 "<start_of_turn>user\nV<end_of_turn>\n<start_of_turn>model\n")
    angle = {c: i for i, c in enumerate(["<bos>", "<|turn>", "<turn|>"])}
    t4 = Tokenizer(Char(angle), list(angle.keys()), added=dict(angle), eos_id=2)
    p4 = t4.apply_chat_template([{"role": "system", "content": " sys "}, {"role": "user", "content": "q"}],
                                enable_thinking=True)
    assert p4 == "<bos><|turn>system\n<|think|>\nsys<turn|>\n<|turn>user\nq<turn|>\n<|turn>model\n"
    plain = Tokenizer(Char({"a": 0}), ["a"], eos_id=0)
    assert plain.chat_format == PLAIN
    assert plain.apply_chat_template([{"role": "user", "content": "hi"}]) == "user: hi\nassistant: "


def test_stream_decoder_emits_complete_characters(tmp_path):
    t = _train_bytelevel(tmp_path)
    ours = Tokenizer.from_pretrained(_save(t, tmp_path))
    text = "café 東京 🙂 ok"
    ids = ours.encode(text)
    sd = ours.stream_decoder()
    out = "".join(sd.push(i) for i in ids) + sd.flush()
    assert out == text
    assert "�" not in out


def _basic_by_definition(text, lowercase=True, strip_accents=None):
    """BERT basic tokenisation written per character (the definition the fast path must reproduce)."""
    import unicodedata
    from nanovllm_b200.tokenizer.codecs import _is_cjk, _is_punct
    out = []
    for ch in text:
        cp = ord(ch)
        if cp == 0 or cp == 0xFFFD or (unicodedata.category(ch).startswith("C") and ch not in "\t\n\r"):
            continue
        out.append(f" {ch} " if _is_cjk(cp) else " " if ch in "\t\n\r" or unicodedata.category(ch) == "Zs" else ch)
    words = []
    for w in "".join(out).split():
        if lowercase:
            w = w.lower()
        if strip_accents or (strip_accents is None and lowercase):
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


@pytest.mark.parametrize("lowercase,strip", [(True, None), (False, None), (True, False), (False, True)])
def test_bert_basic_tokenize_fast_path_matches_definition(lowercase, strip):
    import random
    from nanovllm_b200.tokenizer.codecs import bert_basic_tokenize
    alphabet = (list("abcXYZ019 ,.;!?-_'\"()[]{}@#$%^&*+=~`|\\/<>:") +
                ["\t", "\n", "\r", "\x00", "\x01", "\x0b", "\x0c", "\x1c", "\x1f", "\x7f",  # ASCII controls
                 "\x85", "\u00a0", "\u3000", "\u2028", "\u200b", "\ufffd",  # NEL, Zs, Zs, Zl, Cf, replacement
                 "\u00e9", "\u00c4", "\u00f1", "e\u0301", "\u0301",  # accents, combining acute
                 "\u4e2d", "\u6587", "\uff0c", "\u3002", "\u201c", "\u201d", "\u2014",  # CJK, CJK / other punct
                 "\u212a", "\u0130", "\u00df", "\u03a9", "\U0001f600", "\U00020001"])  # Kelvin, dotted I, ...
    rng = random.Random(11)
    for n in range(600):
        pool = alphabet[:52] if n % 3 == 0 else alphabet  # a third of the cases are pure ASCII
        text = "".join(rng.choice(pool) for _ in range(rng.randint(0, 40)))
        assert bert_basic_tokenize(text, lowercase, strip) == _basic_by_definition(text, lowercase, strip), repr(text)


def test_native_byte_bpe_core_matches_python_merge(tmp_path):
    """The C++ merge core (csrc/host/bpe.cpp) gives the pure-Python merge's ids: trained merges, random byte
    strings (multi-byte UTF-8, rare bytes) and a merged piece missing from the vocabulary (byte fallback)."""
    import random
    from nanovllm_b200.tokenizer import codecs as C
    if C._native_core() is None:
        pytest.skip("host extension not built")
    t = _train_bytelevel(tmp_path)
    j = json.loads(t.to_str())
    vocab = dict(j["model"]["vocab"])
    merges = [tuple(m.split(" ")) if isinstance(m, str) else tuple(m) for m in j["model"]["merges"]]
    # drop one merged piece from the vocabulary: both paths must fall back to its byte symbols
    gone = next(m for m in reversed(merges) if (m[0] + m[1]).isascii() and (m[0] + m[1]).isalpha())
    vocab.pop(gone[0] + gone[1])
    py = C.ByteBpe(vocab, merges, C.GPT2_PATTERN, native=False)
    nat = C.ByteBpe(vocab, merges, C.GPT2_PATTERN, native=True)
    assert py._core is None and nat._core is not None
    rng = random.Random(5)
    texts = SAMPLES + CORPUS[:3] + [gone[0] + gone[1] + " " + gone[0] + gone[1]]
    for _ in range(300):
        texts.append("".join(chr(rng.choice([rng.randrange(32, 127), rng.randrange(0xa0, 0x800),
                                              rng.randrange(0x3000, 0x9fff), rng.randrange(0x1f300, 0x1f64f)]))
                             for _ in range(rng.randint(1, 30))))
    for s in texts:
        assert nat.encode(s) == py.encode(s), s
    assert len(nat.encode(gone[0] + gone[1])) == len(gone[0] + gone[1])  # the fallback ran: one id per byte


def _spm_vocab(rng, inner_space: bool):
    import string
    letters = "abcde"
    vocab = {"<unk>": 0}
    for i in range(256):
        vocab[f"<0x{i:02X}>"] = len(vocab)
    for c in letters + "▁":
        vocab.setdefault(c, len(vocab))
    for _ in range(120):
        p = "".join(rng.choice(letters) for _ in range(rng.randint(2, 4)))
        vocab.setdefault(p, len(vocab))
        vocab.setdefault("▁" + p[:rng.randint(1, len(p))], len(vocab))
    vocab.setdefault("▁▁", len(vocab))
    if inner_space:  # pieces across a word boundary: the text may not be cut
        vocab.setdefault("a▁b", len(vocab))
        vocab.setdefault("e▁", len(vocab))
    return vocab


@pytest.mark.parametrize("inner_space", [False, True])
def test_sentencepiece_bpe_heap_merge_and_word_cuts_match_full_rescans(inner_space):
    """Score-ordered SentencePiece merging: the heap form equals the rescan-every-pair form (ties: leftmost),
    and cutting the text before each word (only when no piece spans a word boundary) changes no id."""
    import random
    from nanovllm_b200.tokenizer import codecs as C
    rng = random.Random(3 + inner_space)
    vocab = _spm_vocab(rng, inner_space)
    scores = [float(rng.randint(0, 6)) for _ in range(len(vocab))]  # many ties
    cod = C.MetaspaceBpe(vocab, None, scores, add_prefix=True, byte_fallback=True, unk_id=0)
    assert cod._chunk_safe == (not inner_space)
    for _ in range(300):
        text = "".join(rng.choice("abcde  é") for _ in range(rng.randint(1, 60)))
        t = text.replace(" ", C.SPIECE)
        t = t if t.startswith(C.SPIECE) else C.SPIECE + t  # the codec's prefix rule
        want = cod._pieces_to_ids(cod._merge_by_score_rounds(list(t)))
        assert cod._merge_by_score(list(t)) == cod._merge_by_score_rounds(list(t)), t
        assert cod.encode(text) == want, text


def test_stream_decoder_windows_concatenate_to_the_full_decode(tmp_path):
    """Pushing a reply token by token (random ids: partial UTF-8 bytes, special tokens, word joins) emits text
    whose concatenation with the flush is the decode of the whole reply, for byte-level BPE, SentencePiece BPE
    and WordPiece vocabularies."""
    import random
    from tokenizers import Tokenizer as T, decoders, models, pre_tokenizers, trainers
    toks = [Tokenizer.from_pretrained(_save(_train_bytelevel(tmp_path), tmp_path, "bl.json"))]
    b = T(models.BPE(byte_fallback=True, unk_token="<unk>"))
    b.pre_tokenizer = pre_tokenizers.Metaspace()
    b.decoder = decoders.Metaspace()
    b.train_from_iterator(CORPUS, trainers.BpeTrainer(vocab_size=300, special_tokens=["<unk>"] +
                                                      [f"<0x{i:02X}>" for i in range(256)]))
    toks.append(Tokenizer.from_pretrained(_save(b, tmp_path, "msp.json")))
    w = T(models.WordPiece(unk_token="[UNK]"))
    w.pre_tokenizer = pre_tokenizers.BertPreTokenizer()
    w.decoder = decoders.WordPiece()
    w.train_from_iterator(CORPUS, trainers.WordPieceTrainer(vocab_size=300, special_tokens=["[UNK]", "[CLS]", "[SEP]"]))
    toks.append(Tokenizer.from_pretrained(_save(w, tmp_path, "wp.json")))
    rng = random.Random(9)
    for tok in toks:
        for _ in range(40):
            ids = tok.encode(rng.choice(CORPUS)[:rng.randint(5, 120)]) + [rng.randrange(tok.vocab_size)
                                                                         for _ in range(rng.randint(0, 12))]
            for skip in (True, False):
                sd = tok.stream_decoder(skip_special=skip)
                parts = [sd.push(i) for i in ids]
                assert "".join(parts) + sd.flush() == tok.decode(ids, skip_special=skip)
                assert not any(p.endswith("�") for p in parts)


def test_byte_level_decode_fast_path_matches_per_symbol_decode():
    """Pieces made only of byte symbols decode through one translate; mixed pieces (added tokens with other
    characters) through the per-symbol loop; both give the per-symbol loop's text."""
    import random
    from nanovllm_b200.tokenizer import codecs as C

    def slow(pieces):
        data = bytearray()
        for p in pieces:
            for ch in p:
                b = C.BYTE_DECODER.get(ch)
                data.extend(ch.encode("utf-8") if b is None else bytes([b]))
        return data.decode("utf-8", errors="replace")

    cod = C.ByteBpe({}, [], C.GPT2_PATTERN, native=False)
    rng = random.Random(4)
    syms = list(C.BYTE_DECODER)
    for _ in range(300):
        pieces = ["".join(rng.choice(syms) for _ in range(rng.randint(1, 4))) for _ in range(rng.randint(0, 12))]
        if rng.random() < 0.3:
            pieces.insert(rng.randrange(len(pieces) + 1), rng.choice(["<|im_end|>", "\n", "é", "中"]))
        assert cod.decode(pieces) == slow(pieces)
