"""Chat layer: think-tag parsing and salvage, prompt layouts, history truncation, advisors and ChatSession turns.

Scripted-engine tests pin the turn logic exactly; one test drives a real tiny Qwen3 through the engine on CPU.
"""
from dataclasses import dataclass
from typing import List

import pytest

from nanovllm_b200.api.model import LlmModel
from nanovllm_b200.chat import (ChatMessage, ChatSession, LlmAdvisor, LlmListeners, LlmTextKind, ThinkTags,
                                parse, salvage_from_thinking, truncate_history)
from nanovllm_b200.chat import prompts
from nanovllm_b200.chat.markup import ChatReply, clean_assistant_text
from nanovllm_b200.config import EngineConfig
from nanovllm_b200.llm import LLM
from nanovllm_b200.models.writers import byte_level_tokenizer_json
from nanovllm_b200.sampling_params import SamplingParams
from nanovllm_b200.tokenizer.tokenizer import Tokenizer


# ------------------------------------------------------------------------------------------------- markup
def test_parse_closed_and_unclosed_think_blocks():
    p = parse("<think>plan it</think>The answer is 4.")
    assert (p.thinking, p.answer, p.think_open) == ("plan it", "The answer is 4.", False)
    p = parse("<think>still going")
    assert (p.thinking, p.answer, p.think_open) == ("still going", "", True)
    p = parse("<think>a</think>x<think>b</think>y")
    assert p.thinking == "a\nb" and p.answer == "x\ny"
    # a close tag with no open tag: everything before it was thinking
    p = parse("hmm</think>ok")
    assert p.thinking == "hmm" and p.answer == "ok"


def test_parse_holds_partial_markers_and_cuts_specials():
    assert parse("Hello <thi").answer == "Hello"
    assert parse("Hello <|im_e").answer == "Hello"
    assert parse("Done.<|im_end|>garbage").answer == "Done."
    custom = ThinkTags.of("[[t]]", "[[/t]]")
    p = parse("[[t]]why[[/t]]because", custom)
    assert p.thinking == "why" and p.answer == "because"
    with pytest.raises(ValueError):
        ThinkTags.of("x", "x")


def test_salvage_from_thinking():
    assert salvage_from_thinking("Let me think.\nSo the answer is: 42.") == "42"
    assert salvage_from_thinking("long reasoning line\nParis") == "Paris"
    assert salvage_from_thinking("") == ""
    r = ChatReply.parse("<think>Work.\nFinal answer: blue</think>")
    assert r.answer == "blue" and r.salvaged
    assert clean_assistant_text("<think>x</think>  fine  ") == "fine"


# ------------------------------------------------------------------------------------------------- prompts
def test_rag_layout_round_trip():
    doc = prompts.with_context("who wrote it?", "- passage one\n- passage two")
    assert prompts.question(doc) == "who wrote it?"
    assert prompts.facts(doc) == "- passage one\n- passage two"
    assert prompts.has_facts(doc) and not prompts.has_facts("plain question")
    assert prompts.question("plain question") == "plain question"


def test_mix_notes_before_question_dedupe_and_skip_empty():
    mixed = prompts.mix("What is the capital of France?", ["Paris is in France.", "Paris is the capital.", "",
                                                          "Paris is in France."])
    assert mixed.endswith("capital of France?")
    assert mixed.count(prompts.note_line("Paris is in France.")) == 1
    assert mixed.index("Paris is the capital.") < mixed.index("capital of France?")
    assert prompts.mix("  Q?  ", ["", "   "]) == "Q?"
    grounded = prompts.with_context("who are the grimm brothers?", "- The Brothers Grimm were Jacob and Wilhelm.")
    mixed = prompts.mix(grounded, ["Wilhelm Grimm was a folklorist."])
    assert mixed.startswith(prompts.GROUNDING) and mixed.endswith("who are the grimm brothers?")
    assert prompts.note_line("Wilhelm Grimm was a folklorist.") in prompts.facts(mixed)


def test_select_notes_keeps_grounded_only():
    grounded = prompts.with_context("q?", "- The Brothers Grimm were Jacob Grimm and Wilhelm Grimm.")
    sel = prompts.select_notes(grounded, ["The Brothers Grimm were Jacob Grimm and Wilhelm Grimm.",
                                          "Bananas contain potassium minerals.", ""])
    assert sel == ["The Brothers Grimm were Jacob Grimm and Wilhelm Grimm."]
    assert prompts.select_notes("plain?", ["a note", "a note", " "]) == ["a note"]
    assert prompts.is_abstention("I do not know.") and not prompts.is_abstention("I do not knowledge")


# ------------------------------------------------------------------------------------------------- scripted engine
def _tokenizer():
    return Tokenizer.from_json(byte_level_tokenizer_json(300))


@dataclass
class _Out:
    token_ids: List[int]


class ScriptedLLM:
    """Engine stand-in: replies come from a script, prompts are recorded."""

    def __init__(self, replies, max_model_len=4096):
        self.tokenizer = _tokenizer()
        self.cfg = EngineConfig(max_model_len=max_model_len)
        self.default_sampling = SamplingParams(max_tokens=64)
        self.replies = list(replies)
        self.calls = []

    def generate_token_ids(self, prompts_, sampling, on_token=None, timeout_s=None):
        self.calls.append(([self.tokenizer.decode(p) for p in prompts_], sampling))
        outs = []
        for i, _ in enumerate(prompts_):
            ids = self.tokenizer.encode(self.replies.pop(0), allow_special=True)
            if on_token is not None:
                for t in ids:
                    on_token(i, i, t)
            outs.append(_Out(ids))
        return outs


def test_session_history_keeps_answer_and_streams_events():
    llm = ScriptedLLM(["<think>consider</think>Four.", "Five."])
    listener, events = LlmListeners.collecting()
    s = ChatSession(llm, system_prompt="Be brief.", listener=listener)
    r = s.send("2+2?")
    assert r.answer == "Four." and r.thinking == "consider"
    assert [m.role for m in s.history] == ["system", "user", "assistant"]
    assert s.history[-1].content == "Four."
    answer_text = "".join(e.text for e in events if e.kind == LlmTextKind.TEXT_ASSISTANT and not e.snapshot)
    think_text = "".join(e.text for e in events if e.kind == LlmTextKind.TEXT_THINKING and not e.snapshot)
    assert answer_text == "Four." and think_text == "consider"
    s.send("and 2+3?")
    prompt = llm.calls[-1][0][0]
    assert "2+2?" in prompt and "Four." in prompt and "consider" not in prompt  # history keeps answer only
    s.clear()
    assert [m.role for m in s.history] == ["system"]


def test_session_salvages_unclosed_thinking_and_falls_back():
    llm = ScriptedLLM(["<think>Work it out.\nAnswer: blue", ""])
    diag, events = LlmListeners.collecting([LlmTextKind.TEXT_DIAGNOSTICS])
    s = ChatSession(llm, listener=diag)
    r = s.send("color?")
    assert r.answer == "blue" and r.salvaged
    assert any("unclosed thinking" in e.text for e in events)
    r = s.send("again?")
    assert r.answer == s.fallback_reply


def test_session_history_cap_and_truncation():
    llm = ScriptedLLM(["ok"] * 6)
    s = ChatSession(llm, system_prompt="sys", max_history_messages=4)
    for i in range(3):
        s.send(f"message {i}")
    assert len(s.history) == 4 and s.history[0].role == "system"
    tok = _tokenizer()
    hist = [ChatMessage.system("s")] + [ChatMessage.user("x" * 40), ChatMessage.assistant("y" * 40)] * 6 + \
           [ChatMessage.user("last")]
    truncate_history(hist, tok, max_model_len=200, max_tokens=16)
    assert hist[0].role == "system" and hist[-1].content == "last"
    assert len(tok.encode(tok.apply_chat_template(hist))) <= 200 - 16 - 16
    assert all(hist[i].role != "assistant" for i in (1,))  # never starts the dialog with a dangling reply


def test_advisors_run_as_one_batch_and_mix_into_prompt():
    llm = ScriptedLLM(["Paris is the capital.", "<think>hm</think>It is in Europe.", "Paris."])
    notes, events = LlmListeners.collecting([LlmTextKind.TEXT_ADVISOR_NOTE])
    s = ChatSession(llm, advisors=[LlmAdvisor("facts", "State one fact."), LlmAdvisor("geo", "Give geography.")],
                    sampling=SamplingParams(temperature=0.9, max_tokens=500), listener=notes)
    r = s.send("What is the capital of France?")
    assert r.answer == "Paris."
    adv_prompts, adv_sp = llm.calls[0]
    assert len(adv_prompts) == 2  # one batched generate for both advisors
    assert adv_sp.temperature == pytest.approx(0.3) and adv_sp.max_tokens == 256
    assert "State one fact." in adv_prompts[0] and "Give geography." in adv_prompts[1]
    main_prompt = llm.calls[1][0][0]
    assert main_prompt.index("Paris is the capital.") < main_prompt.index("What is the capital of France?")
    assert "It is in Europe." in main_prompt and "hm" not in main_prompt
    assert s.history[0].content == "What is the capital of France?"  # history keeps the raw question
    assert len(events) == 2
    with pytest.raises(ValueError):
        LlmAdvisor(" ", "x")


def test_unusable_answer_recovery_uses_advisor_notes():
    llm = ScriptedLLM(["Helpful note.", "facts", "facts"])
    s = ChatSession(llm, advisors=[LlmAdvisor("facts", "Give facts.")], recover_unusable_answers=True)
    r = s.send("question?")
    assert r.answer == "Helpful note."  # both main answers equal the advisor's name -> notes used


# ------------------------------------------------------------------------------------------------- real engine
def test_chat_session_on_tiny_model_cpu():
    from test_cpu_model import tiny
    from nanovllm_b200.models.registry import init_random_weights
    hf = tiny(vocab_size=300)
    w = init_random_weights(hf, 0)
    model = LlmModel(hf, w, tokenizer=_tokenizer())
    llm = LLM(model, EngineConfig(max_num_seqs=2, max_model_len=512, num_kvcache_blocks=8,
                                  max_num_batched_tokens=512), device="cpu")
    raw, events = LlmListeners.collecting([LlmTextKind.TEXT_RAW])
    s = ChatSession(llm, system_prompt="hi", sampling=SamplingParams(max_tokens=12, ignore_eos=True).deterministic(),
                    listener=raw)
    r = s.send("hello there")
    streamed = "".join(e.text for e in events if not e.snapshot)
    assert streamed == r.raw
    assert s.history[-1].role == "assistant" and s.history[-1].content == r.answer
    s.send("again")
    assert [m.role for m in s.history] == ["system", "user", "assistant", "user", "assistant"]


def test_session_uses_the_models_chat_specials():
    """A checkpoint's own end-of-answer marker (LlmModel option ``chat_specials``) ends the visible answer, both
    in the streamed events and in the final reply."""
    from nanovllm_b200.chat.markup import ChatSpecials
    llm = ScriptedLLM(["Six. [[stop]] trailing junk"])
    llm.chat_specials = lambda: ChatSpecials(("[[stop]]",))
    listener, events = LlmListeners.collecting()
    r = ChatSession(llm, listener=listener).send("3+3?")
    assert r.answer == "Six."
    shown = "".join(e.text for e in events if e.kind == LlmTextKind.TEXT_ASSISTANT and not e.snapshot)
    assert shown.strip() == "Six."


def test_reply_scanner_streams_token_by_token_like_a_single_parse():
    from nanovllm_b200.chat.markup import ReplyScanner
    raw = "<think>plan: add\nthe numbers</think>The answer is 4.<|im_end|>tail"
    sc = ReplyScanner()
    shown = []
    for i in range(0, len(raw), 3):  # 3-character chunks split every marker somewhere
        shown.append(sc.feed(raw[i:i + 3]).snapshot().answer)
    final = sc.snapshot()
    assert final == parse(raw)
    assert final.answer == "The answer is 4." and final.thinking == "plan: add\nthe numbers"
    assert all("<" not in s for s in shown), "a partial marker leaked into the displayed answer"
    # answers only ever grow while streaming
    assert all(b.startswith(a) for a, b in zip(shown, shown[1:]))


class FrontDoorLLM(ScriptedLLM):
    """Scripted engine carrying the real ``LLM`` front-door methods (chat / rag / run_advisors)."""
    from nanovllm_b200.llm import LLM as _LLM
    chat = _LLM.chat
    rag = _LLM.rag
    run_advisors = _LLM.run_advisors
    new_conversation = _LLM.new_conversation
    _assert_open = _LLM._assert_open

    def __init__(self, replies, advisors=(), system_prompt=""):
        super().__init__(replies)
        self._closed = False
        self.advisors = list(advisors)
        self.advisor_mixer = None
        self.think_tags = None
        self.system_prompt = system_prompt
        self.listener = None


def test_llm_front_door_chat_rag_and_advisors():
    from nanovllm_b200.rag import RagFactory
    llm = FrontDoorLLM(["Four.", "Paris lies on the Seine.", "note A", "note B"], system_prompt="Be brief.")
    s = llm.chat(7)  # int: max new tokens per turn, engine defaults otherwise
    assert s.sampling_params().max_tokens == 7 and s.sampling_params().temperature == llm.default_sampling.temperature
    assert s.send("2+2?").answer == "Four."
    ix = RagFactory.of("Paris is the capital of France. It lies on the Seine river.")
    r = llm.rag(ix, max_tokens=32)
    assert r.send("Where does Paris lie?").answer == "Paris lies on the Seine."
    assert r.base_sampling.max_tokens == 32  # (turns without hits raise it to the no-hits floor, as designed)
    llm.advisors = [LlmAdvisor("a", "Say A."), LlmAdvisor("b", "Say B.")]
    enr = llm.run_advisors("What is the capital?", [], SamplingParams(max_tokens=100))
    assert [x.advisor_name for x in enr.responses] == ["a", "b"] and len(llm.calls[-1][0]) == 2  # one batched generate
    conv = llm.new_conversation()
    assert [m.role for m in conv] == ["system"] and conv[0].content == "Be brief."
    with pytest.raises(ValueError):
        llm.chat(0)
    llm._closed = True
    with pytest.raises(Exception):
        llm.chat()


def test_chat_session_fluent_knobs():
    """ChatSession setters of the reference (ChatSession.java:99-405) return the session and take effect."""
    import io
    llm = ScriptedLLM(["<think>hmm</think>Ten.", "x", "Eleven.", "", ""])
    think, answer, diag = io.StringIO(), io.StringIO(), []
    s = (ChatSession.open(llm, 9).deterministic().max_tokens(5).timeout(3.0).enable_thinking(True)
         .max_history_messages(4).emit_debug_prompts(False).recover_unusable_answers(True)
         .unusable_answer(lambda a: a.strip() in ("", "x")).unusable_answer_fallback("n/a")
         .diagnostics(diag.append).stream_to(think, answer)
         .seed(ChatMessage.user("5+5?"), ChatMessage.assistant("Ten.")))
    assert s.sampling_params().max_tokens == 5 and s.sampling_params().top_k == 1  # deterministic kept
    assert s.thinking_enabled() and s.timeout_s == 3.0 and s.think_tags() is s.tags
    assert [m.role for m in s.history] == ["user", "assistant"]
    r = s.send("5+5 again?")
    assert r.answer == "Ten." and think.getvalue() == "hmm" and answer.getvalue() == "Ten."
    assert s.send("6+5?").answer == "Eleven." and any("retrying" in d for d in diag)  # "x" is unusable
    assert s.send("and?").answer == "n/a"  # still unusable after the retry: the fallback reply
    assert len(s.history) <= 4
    with pytest.raises(ValueError):
        s.max_history_messages(1)
