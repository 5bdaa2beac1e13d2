"""RAG: chunking, BM25 selection / outside-corpus rules, dense + hybrid fusion on a tiny BERT, RagSession turns."""
import pytest
import torch

from nanovllm_b200.chat import prompts
from nanovllm_b200.rag import (CorpusLoader, DenseRagIndex, HybridRagIndex, PreparedRag, RagFactory, RagHit,
                               RagLoadOptions, RagSession, RagTuner, TextChunk, format_user_message)
from nanovllm_b200.rag.corpus import passages, window_split
from nanovllm_b200.rag.dense import fuse
from nanovllm_b200.rag.session import parse_rewrite, prefer_prior_source, short_follow_up
from nanovllm_b200.sampling_params import SamplingParams

GRIMM = """# The Brothers Grimm
The brothers Jacob Grimm and Wilhelm Grimm were German scholars who collected folk tales. The father of the
brothers was Philipp Wilhelm Grimm, a lawyer. Jacob was awarded a position as librarian in Kassel.

# Little Red Riding Hood
A girl in a red hood walks through the forest to her grandmother. A wolf meets her on the way and runs ahead to the
grandmother's house.
"""
PARIS = "Paris is the capital of France. It is also the largest city of the country."


def test_passages_sections_sentences_and_markup():
    ps = passages("# Title\nSome `code` and a [link](http://x). Second sentence!\n\n```\nfenced\n```\n- bullet item")
    assert ps == ["Title — Some code and a link.", "Title — Second sentence!", "Title — bullet item"]


def test_chunking_modes(tmp_path):
    tiny = CorpusLoader(RagLoadOptions.for_tiny_models()).add(GRIMM, "g").build()
    assert all(len(c.text) <= 220 for c in tiny) and len(tiny) >= 5
    packed = CorpusLoader(RagLoadOptions(max_chunk_chars=300)).add(GRIMM, "g").build()
    assert len(packed) < len(tiny) and all(len(c.text) <= 300 for c in packed)
    raw = CorpusLoader(RagLoadOptions(max_chunk_chars=64, chunk_overlap=16, preprocess=False)).add(" ".join(f"w{i}" for i in range(80))).build()
    assert len(raw) > 3 and all(len(c.text) <= 64 for c in raw)
    w = window_split("x", "x", "abcdefgh " * 30, 100, 20)
    assert all(len(c.text) <= 100 for c in w) and w[0].id == "x#1"
    dup = CorpusLoader().add("Same text here.").add("same   TEXT here.").build()
    assert len(dup) == 1
    with pytest.raises(ValueError):
        RagLoadOptions(max_chunk_chars=10)


def test_folder_loading_tuners_and_budgets(tmp_path):
    (tmp_path / "grimm.md").write_text(GRIMM)
    (tmp_path / "paris.txt").write_text(PARIS)
    (tmp_path / "README.md").write_text("ignored readme")
    (tmp_path / "image.png").write_bytes(b"\x89PNG")
    ix = RagFactory.make(str(tmp_path), RagLoadOptions.for_tiny_models())
    srcs = {c.source for c in ix.chunks}
    assert any(s.endswith("grimm.md") for s in srcs) and any(s.endswith("paris.txt") for s in srcs)
    assert not any("README" in s for s in srcs)
    only_txt = RagFactory.builder().add_processor(RagTuner.allowing(lambda r: r.file_name().endswith(".txt"))) \
        .add_folder(str(tmp_path)).build()
    assert all(c.source.endswith(".txt") for c in only_txt.chunks)
    upper = RagFactory.builder().add_processor(RagTuner.preprocessing(str.upper)).add("hello world text").build()
    assert upper.chunks[0].text == "HELLO WORLD TEXT"
    from nanovllm_b200.utils.limits import ResourceLimits
    with pytest.raises(ValueError):
        CorpusLoader(RagLoadOptions(limits=ResourceLimits(max_file_bytes=10))).add_file(str(tmp_path / "grimm.md"))
    assert RagFactory.try_make(str(tmp_path / "missing")) is None


def _grimm_index():
    return RagFactory.builder().for_tiny_models().add(GRIMM, "grimm.md").add(PARIS, "paris.txt").build()


def test_bm25_retrieval_and_outside_corpus():
    ix = _grimm_index()
    hits = ix.retrieve("who was the father of the Grimm brothers", 2)
    assert hits and "Philipp" in hits[0].chunk.text
    assert "Paris is the capital" in ix.retrieve("capital of France", 1)[0].chunk.text
    assert ix.retrieve("Little Red Riding Hood wolf grandmother", 2)
    for off in ("what do you think about estonia?", "I would like to discuss about cars",
                "please write any Java program"):
        assert ix.is_outside_corpus(off) or not ix.retrieve(off, 3), off
    assert not ix.retrieve("what do you think about BMW?", 3)
    terms = ix.select_terms("grandmother wolf forest girl")
    assert len(terms) <= 5 and terms[0] == "grandmother"


def test_fuse_and_prior_source():
    a, b, c = (TextChunk(i, i, t) for i, t in (("a", "aaaa"), ("b", "bb"), ("c", "c")))
    fused = fuse([[RagHit(a, 9), RagHit(b, 5)], [RagHit(b, 0.9), RagHit(c, 0.8)]], 3)
    assert fused[0].chunk.id == "b"
    assert fused[0].score == pytest.approx(1 / 62 + 1 / 61)
    g1, g2, p = TextChunk("g1", "grimm", "x"), TextChunk("g2", "grimm", "y"), TextChunk("p", "paris", "z")
    cands = [RagHit(p, 1.0), RagHit(g1, 0.6), RagHit(g2, 0.5)]
    assert [h.chunk.id for h in prefer_prior_source(cands, "grimm", 1)] == ["g1"]
    assert [h.chunk.id for h in prefer_prior_source([RagHit(p, 1.0), RagHit(g1, 0.3)], "grimm", 1)] == ["p"]


def test_query_helpers():
    assert short_follow_up("what are their names?")
    assert not short_follow_up("what are the names of the famous German brothers who collected tales")
    assert parse_rewrite('Search: "grimm father"') == "grimm father"
    assert parse_rewrite("NONE") is None and parse_rewrite("") is None
    hits = [RagHit(TextChunk("a", "a", "first passage " * 20), 1.0), RagHit(TextChunk("b", "b", "second"), 0.5)]
    msg = format_user_message(hits, "q?", 100)
    assert prompts.question(msg) == "q?" and len(prompts.facts(msg)) <= 100
    assert format_user_message([], "plain?") == "plain?"


def _bert_model():
    from test_models_cpu import bert_tiny
    from nanovllm_b200.api.model import LlmModel
    from nanovllm_b200.models.registry import init_random_weights
    from nanovllm_b200.models.writers import byte_level_tokenizer_json
    from nanovllm_b200.tokenizer.tokenizer import Tokenizer
    hf = bert_tiny()
    tok = Tokenizer.from_json(byte_level_tokenizer_json(hf.vocab_size))
    return LlmModel(hf, init_random_weights(hf, 2), tokenizer=tok)


def test_dense_and_hybrid_on_tiny_bert_cpu():
    model = _bert_model()
    lex = _grimm_index()
    seen = []
    dense = DenseRagIndex.of(lex, model, on_passage_embedded=seen.append)
    assert dense.size() == lex.size() and seen[-1] == lex.size()
    assert torch.allclose(dense.vectors.norm(dim=1), torch.ones(dense.size()), atol=1e-3)
    # a passage's own text is its nearest neighbour (cosine 1)
    target = lex.chunks[2]
    top = dense.retrieve(target.text, 1)
    assert top[0].chunk.id == target.id and top[0].score == pytest.approx(1.0, abs=2e-3)
    hybrid = HybridRagIndex.of(lex, dense)
    assert hybrid.size() == lex.size() and hybrid.lexical() is lex and hybrid.dense() is dense
    assert hybrid.retrieve("father of the Grimm brothers", 2)
    with pytest.raises(ValueError):
        HybridRagIndex([lex, lex])


def test_rag_session_turns_with_scripted_engine():
    from test_chat import ScriptedLLM
    llm = ScriptedLLM(["Philipp Wilhelm Grimm.", "grimm father names", "Jacob and Wilhelm.", "I do not know."])
    rag = RagSession(llm, _grimm_index(), sampling=SamplingParams(temperature=0.8, max_tokens=32))
    r = rag.send("Who was the father of the Grimm brothers?")
    assert r.answer == "Philipp Wilhelm Grimm."
    prompt, sp = llm.calls[0][0][0], llm.calls[0][1]
    assert prompts.GROUNDING in prompt and "Philipp" in prompt
    assert sp.temperature == pytest.approx(0.15)  # grounded turns cap temperature
    assert rag.chat.history[-2].content == "Who was the father of the Grimm brothers?"
    rag.send("why so?")  # short follow-up without a direct hit -> the model rewrites it into keywords
    assert "Follow-up: why so?" in llm.calls[1][0][0]
    assert rag.last_retrieval_query == "grimm father names" and rag.last_hits
    assert llm.calls[1][1].max_tokens == 48 and llm.calls[1][1].temperature == pytest.approx(0.1)
    r = rag.send("Tell me about quantum chromodynamics lattice simulations")
    assert rag.last_hits == [] and llm.calls[-1][1].max_tokens >= 384


def test_rag_session_fluent_knobs():
    """RagSession.open and its knobs (RagSession.java:96-400): RAG knobs act on the turn, chat knobs reach the
    underlying ChatSession, format_user_message builds the grounded turn."""
    from test_chat import ScriptedLLM
    from nanovllm_b200.chat import ChatSession
    llm = ScriptedLLM(["I do not know.", "Philipp."])
    diag = []
    rag = (RagSession.open(llm, _grimm_index(), 16).max_tokens_when_no_hits(99).isolate_generation(True)
           .timeout(2.0).max_history_messages(6).diagnostics(diag.append).emit_debug_prompts(False))
    assert rag.chat.timeout_s == 2.0 and rag.chat.max_history == 6 and not rag.chat.thinking_enabled()
    rag.send("Tell me about quantum chromodynamics lattice simulations")
    assert llm.calls[-1][1].max_tokens == 99
    chat = ChatSession(llm)
    rag2 = RagSession.open(chat, _grimm_index())
    assert rag2.chat is chat
    rag2.send("Who was the father of the Grimm brothers?")
    hits = _grimm_index().retrieve("father Grimm brothers", 2)
    msg = RagSession.format_user_message(hits, "Who was the father?")
    assert "Who was the father?" in msg and "Philipp" in msg
    with pytest.raises(ValueError):
        rag.max_tokens_when_no_hits(0)
