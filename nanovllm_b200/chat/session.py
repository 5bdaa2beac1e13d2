"""Advisors and ``ChatSession`` (multi-turn chat with streaming, salvage and history management).

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/chat/ChatSession.java:73-845 and
llm/{AdvisorRunner.java:20-110, LlmAdvisor.java, LlmAdvisorMixer.java, DefaultAdvisorMixer.java,
AdvisorEnrichment.java}.  One turn:

1. append the user text to history, cap the history length, truncate it to the prompt budget;
2. advisors (when configured): every advisor gets its own dialog -- its role prompt as system, the earlier USER
   turns, then the advisor-facing question -- and ALL advisor prompts run as ONE batched generate (temperature
   ``min(main, 0.3)``, or 0.3 when main is greedy; ``min(main max_tokens, 256)``); the mixer folds their notes into
   the model's user text;
3. generate with a token callback that streams TEXT_RAW / TEXT_THINKING / TEXT_ASSISTANT deltas (a snapshot event
   when the parse rewrote already-shown text; assistant text is held while a think block is open);
4. optional unusable-answer recovery (retry once without matching filler turns, then advisor notes, then a fixed
   fallback);
5. salvage an answer from the thinking when the visible answer is blank, or tiny (<= 12 chars) after long
   thinking (>= 120 chars); keep only the answer in history.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence

from ..sampling_params import SamplingParams
from ..utils.limits import ResourceLimits
from . import prompts
from .listeners import LlmListener, LlmTextKind, emit
from .markup import ChatReply, ChatSpecials, ReplyScanner, ThinkTags, parse, salvage_from_thinking
from .messages import ChatMessage, truncate_history

MAX_ADVISOR_TOKENS = 256
ADVISOR_TEMPERATURE = 0.3
DEFAULT_FALLBACK_REPLY = "Sorry, I could not produce an answer."


# ----------------------------------------------------------------------------------------------- advisors
@dataclass(frozen=True)
class LlmAdvisor:
    name: str
    prompt: str

    def __post_init__(self):
        if not self.name or not self.name.strip():
            raise ValueError("advisor name must not be blank")
        if not self.prompt or not self.prompt.strip():
            raise ValueError("advisor prompt must not be blank")
        object.__setattr__(self, "name", self.name.strip())
        object.__setattr__(self, "prompt", self.prompt.strip())


@dataclass(frozen=True)
class AdvisorResponse:
    advisor_name: str
    text: str


@dataclass
class AdvisorEnrichment:
    model_user_text: str
    responses: List[AdvisorResponse] = field(default_factory=list)
    salvage_notes: List[str] = field(default_factory=list)

    @staticmethod
    def passthrough(text: str) -> "AdvisorEnrichment":
        return AdvisorEnrichment(text)

    def has_advisor_notes(self) -> bool:
        return any(r.text and r.text.strip() for r in self.responses)

    def answer_salvage_notes(self) -> List[str]:
        src = self.salvage_notes or [r.text for r in self.responses]
        out: List[str] = []
        for n in src:
            n = (n or "").strip()
            if n and n not in out:
                out.append(n)
        return out


class DefaultAdvisorMixer:
    """Mixer contract: ``mix_prompt(llm, responses, history, prompt) -> model user text``."""

    def mix_prompt(self, llm, responses: Sequence[AdvisorResponse], history, prompt: str) -> str:
        return prompts.mix(prompt, [r.text for r in responses])


def dialog_turn(role_prompt: str, prior_dialog: Sequence[ChatMessage], model_user_text: str) -> List[ChatMessage]:
    system = (role_prompt or "").strip()
    if not system:
        raise ValueError("role prompt must not be blank")
    user = prompts.advisor_facing_user_text(model_user_text)
    if not user:
        raise ValueError("model user text must not be blank")
    return [ChatMessage.system(system)] + [m for m in prior_dialog if m.role == "user"] + [ChatMessage.user(user)]


def advisor_sampling(main: SamplingParams) -> SamplingParams:
    t = min(main.temperature, ADVISOR_TEMPERATURE)
    if t <= 1e-10:
        t = ADVISOR_TEMPERATURE
    return main.with_(temperature=t, max_tokens=min(main.max_tokens, MAX_ADVISOR_TOKENS), ignore_eos=False)


class AdvisorRunner:
    @staticmethod
    def enrich(llm, advisors: Sequence[LlmAdvisor], model_user_text: str, prior_dialog: Sequence[ChatMessage],
               main_sampling: SamplingParams, mixer=None, tags: ThinkTags = ThinkTags(),
               note_filter: Optional[Callable[[str], bool]] = None) -> AdvisorEnrichment:
        if not advisors:
            return AdvisorEnrichment.passthrough(model_user_text)
        tok = llm.tokenizer
        sp = advisor_sampling(main_sampling)
        batch = []
        for a in advisors:
            turn = dialog_turn(a.prompt, prior_dialog, model_user_text)
            truncate_history(turn, tok, llm.cfg.max_model_len, sp.max_tokens, False, tags)
            text = tok.apply_chat_template(turn, True, False, tags.open, tags.close)
            batch.append(tok.encode(text, allow_special=True))
        outs = llm.generate_token_ids(batch, sp)  # one batched generate for every advisor
        responses = []
        for a, o in zip(advisors, outs):
            raw = tok.decode(o.token_ids, skip_special=True)
            answer = ChatReply.parse(raw, tags).answer.strip()
            responses.append(AdvisorResponse(a.name, prompts.usable_note(answer, note_filter)))
        salvage = prompts.select_notes(model_user_text, [r.text for r in responses])
        mixed = (mixer or DefaultAdvisorMixer()).mix_prompt(llm, responses, list(prior_dialog), model_user_text)
        return AdvisorEnrichment(mixed, responses, salvage)


# ----------------------------------------------------------------------------------------------- streaming
class _TurnStream:
    def __init__(self):
        self.raw = ""
        self.think = ""
        self.answer = ""

    @staticmethod
    def _one(listener, source, kind, current, shown):
        if current == shown:
            return
        if len(current) > len(shown) and current.startswith(shown):
            emit(listener, source, kind, current[len(shown):])
        else:
            emit(listener, source, kind, current, snapshot=True)

    def push(self, listener, source, raw: str, thinking: str, answer: str, think_open: bool):
        self._one(listener, source, LlmTextKind.TEXT_RAW, raw, self.raw)
        self.raw = raw
        self._one(listener, source, LlmTextKind.TEXT_THINKING, thinking, self.think)
        self.think = thinking
        if not think_open:
            self._one(listener, source, LlmTextKind.TEXT_ASSISTANT, answer, self.answer)
            self.answer = answer


def should_salvage(answer: str, thinking: str) -> bool:
    if not thinking.strip():
        return False
    if not answer.strip():
        return True
    return len(answer) <= 12 and len(thinking) >= 120


def _engine_think_tags(llm) -> ThinkTags:
    handle = getattr(llm, "model_handle", None)
    tags = getattr(handle, "think_tags", None)
    return tags() if callable(tags) else ThinkTags()


# ----------------------------------------------------------------------------------------------- session
class ChatSession:
    def __init__(self, llm, system_prompt: Optional[str] = None, sampling: Optional[SamplingParams] = None,
                 think_tags: Optional[ThinkTags] = None, enable_thinking: bool = False,
                 max_history_messages: int = ResourceLimits.MAX_HISTORY_MESSAGES,
                 timeout_s: Optional[float] = None, advisors: Optional[Sequence[LlmAdvisor]] = None, mixer=None,
                 listener: Optional[LlmListener] = None, emit_debug_prompts: bool = False,
                 seed_messages: Sequence[ChatMessage] = (), recover_unusable_answers: bool = False,
                 unusable_answer: Optional[Callable[[str], bool]] = None,
                 fallback_reply: str = DEFAULT_FALLBACK_REPLY):
        if llm.tokenizer is None:
            raise ValueError("ChatSession needs an engine with a tokenizer")
        if max_history_messages < 2:
            raise ValueError("max_history_messages must be >= 2")
        self.llm = llm
        self.tok = llm.tokenizer
        self._sp = sampling or llm.default_sampling
        self.tags = think_tags or getattr(llm, "think_tags", None) or _engine_think_tags(llm)
        specials = getattr(llm, "chat_specials", None)
        self.specials = (specials() if callable(specials) else None) or ChatSpecials.default()
        self._thinking = enable_thinking
        self.max_history = max_history_messages
        self.timeout_s = timeout_s
        self.advisors = list(advisors if advisors is not None else (getattr(llm, "advisors", None) or []))
        self.mixer = mixer or getattr(llm, "advisor_mixer", None) or DefaultAdvisorMixer()
        self.listener = listener if listener is not None else getattr(llm, "listener", None)
        if system_prompt is None:
            system_prompt = getattr(llm, "system_prompt", "") or ""
        self.debug = emit_debug_prompts
        self.recover = recover_unusable_answers
        self.unusable = unusable_answer or (lambda s: not s.strip())
        self.fallback_reply = fallback_reply
        self.history: List[ChatMessage] = []
        if system_prompt and system_prompt.strip():
            self.history.append(ChatMessage.system(system_prompt.strip()))
        self.history.extend(seed_messages)
        self.last_reply: Optional[ChatReply] = None
        self.last_advisor_s = 0.0
        self.last_generate_s = 0.0
        self._stream: Optional[_TurnStream] = None

    # -------------------------------------------------------------------------------------- knobs
    # fluent setters of the reference session (ChatSession.java:99-405); each returns the session
    @staticmethod
    def open(llm, max_tokens: int) -> "ChatSession":
        """A session with the engine's default sampling and ``max_tokens`` new tokens per turn."""
        return ChatSession(llm, sampling=llm.default_sampling.with_(max_tokens=int(max_tokens)))

    def listen(self, listener: Optional[LlmListener]) -> "ChatSession":
        self.listener = listener
        return self

    def sampling(self, sp: SamplingParams) -> "ChatSession":
        if sp is None:
            raise ValueError("sampling must not be None")
        self._sp = sp
        return self

    def sampling_params(self) -> SamplingParams:
        return self._sp

    def deterministic(self) -> "ChatSession":
        return self.sampling(self._sp.deterministic())

    def max_tokens(self, n: int) -> "ChatSession":
        return self.sampling(self._sp.with_(max_tokens=int(n)))

    def seed(self, *messages: ChatMessage) -> "ChatSession":
        """Append prior turns (e.g. a few-shot dialog) to the history."""
        for m in messages:
            self.history.extend(m if isinstance(m, (list, tuple)) else [m])
        self._cap()
        return self

    def timeout(self, seconds: Optional[float]) -> "ChatSession":
        self.timeout_s = None if seconds is None else float(seconds)
        return self

    def enable_thinking(self, on: bool = True) -> "ChatSession":
        self._thinking = bool(on)
        return self

    def thinking_enabled(self) -> bool:
        return self._thinking

    def think_tags(self, tags: Optional[ThinkTags] = None):
        """With ``tags``: set them and return the session; without: the session's think tags."""
        if tags is None:
            return self.tags
        self.tags = tags
        return self

    def recover_unusable_answers(self, on: bool = True) -> "ChatSession":
        self.recover = bool(on)
        return self

    def unusable_answer(self, predicate: Callable[[str], bool]) -> "ChatSession":
        if not callable(predicate):
            raise TypeError("unusable_answer needs a callable")
        self.unusable = predicate
        return self

    def unusable_answer_fallback(self, text: str) -> "ChatSession":
        self.fallback_reply = text or DEFAULT_FALLBACK_REPLY
        return self

    def max_history_messages(self, n: int) -> "ChatSession":
        if n < 2:
            raise ValueError("max_history_messages must be >= 2")
        self.max_history = int(n)
        self._cap()
        return self

    def emit_debug_prompts(self, on: bool = True) -> "ChatSession":
        self.debug = bool(on)
        return self

    def diagnostics(self, consumer: Optional[Callable[[str], None]]) -> "ChatSession":
        """Send the session's diagnostic lines (retries, salvage) to ``consumer`` besides the listener."""
        self._diag_sink = consumer
        return self

    def stream_to(self, think_out=None, answer_out=None) -> "ChatSession":
        """Write streamed thinking / answer text to file-like objects (e.g. sys.stdout) as it arrives."""
        def listener(_source, event):
            out = think_out if event.kind == LlmTextKind.TEXT_THINKING else \
                answer_out if event.kind == LlmTextKind.TEXT_ASSISTANT else None
            if out is not None and not event.snapshot:
                out.write(event.text)
                if hasattr(out, "flush"):
                    out.flush()
        self.listener = listener
        return self

    def last_generate_stats(self):
        return getattr(self.llm, "last_stats", None)

    def clear(self) -> None:
        self.history = [m for m in self.history[:1] if m.role == "system"]

    def _diag(self, text: str) -> None:
        emit(self.listener, self, LlmTextKind.TEXT_DIAGNOSTICS, text)
        sink = getattr(self, "_diag_sink", None)
        if sink is not None:
            sink(text)

    def _cap(self) -> None:
        while len(self.history) > self.max_history:
            at = 0
            if self.history and self.history[0].role == "system":
                if len(self.history) == 1:
                    break
                at = 1
            self.history.pop(at)

    def _prior_users(self) -> List[ChatMessage]:
        users = [m for m in self.history if m.role == "user"]
        return users[:-1] if len(users) > 1 else []

    # -------------------------------------------------------------------------------------- turns
    def send(self, user_text: str) -> ChatReply:
        return self.send_prepared(user_text, user_text)

    def ask(self, user_text: str) -> str:
        return self.send(user_text).answer

    def send_prepared(self, history_user_text: str, model_user_text: str, isolate: bool = False,
                      sampling: Optional[SamplingParams] = None) -> ChatReply:
        """History keeps ``history_user_text``; the model sees ``model_user_text`` (e.g. a grounded RAG turn).
        ``isolate`` generates from the system prompt plus this turn only (no earlier dialog)."""
        hist_user, model_user = (history_user_text or "").strip(), (model_user_text or "").strip()
        if not hist_user or not model_user:
            raise ValueError("user text must not be blank")
        sp = sampling or self._sp
        self.history.append(ChatMessage.user(hist_user))
        self._cap()
        truncate_history(self.history, self.tok, self.llm.cfg.max_model_len, sp.max_tokens,
                         self._thinking, self.tags)
        t0 = time.perf_counter()
        if self.advisors:
            enr = AdvisorRunner.enrich(self.llm, self.advisors, model_user, self._prior_users(), sp,
                                       self.mixer, self.tags, getattr(self.llm, "advisor_note_filter", None))
            for r in enr.responses:
                if r.text:
                    emit(self.listener, self, LlmTextKind.TEXT_ADVISOR_NOTE, f"[{r.advisor_name}] {r.text}\n")
        else:
            enr = AdvisorEnrichment.passthrough(model_user)
        self.last_advisor_s = time.perf_counter() - t0 if self.advisors else 0.0
        if self.debug:
            emit(self.listener, self, LlmTextKind.TEXT_DEBUG, enr.model_user_text)
        t1 = time.perf_counter()
        reply = self._generate(enr.model_user_text, isolate, sp)
        if self.recover and self._unusable(reply.answer):
            self._scrub_filler()
            self._diag("(unusable main answer: retrying without filler history)\n")
            reply = self._generate(enr.model_user_text, isolate, sp)
            if self._unusable(reply.answer):
                notes = " ".join(enr.answer_salvage_notes()).strip()
                if notes:
                    self._diag("(unusable main answer: used advisor notes)\n")
                    reply = ChatReply(notes, "", reply.raw, reply.stats)
                else:
                    self._diag("(unusable main answer: used fallback reply)\n")
                    reply = ChatReply(self.fallback_reply, "", reply.raw, reply.stats)
        self.last_generate_s = time.perf_counter() - t1
        return self._finish(reply)

    def _unusable(self, answer: str) -> bool:
        body = (answer or "").strip()
        return self.unusable(body) or any(a.name.lower() == body.lower() for a in self.advisors)

    def _scrub_filler(self) -> None:
        self.history = [m for m in self.history if not (m.role == "assistant" and self.unusable(m.content.strip()))]

    def _turn_messages(self, model_user_text: str, isolate: bool, sp: SamplingParams) -> List[ChatMessage]:
        if isolate:
            msgs = [m for m in self.history[:1] if m.role == "system"] + [ChatMessage.user(model_user_text)]
        else:
            msgs = list(self.history)
            if msgs and msgs[-1].role == "user" and msgs[-1].content != model_user_text:
                msgs[-1] = ChatMessage.user(model_user_text)
        truncate_history(msgs, self.tok, self.llm.cfg.max_model_len, sp.max_tokens, self._thinking,
                         self.tags)
        return msgs

    def _generate(self, model_user_text: str, isolate: bool, sp: SamplingParams) -> ChatReply:
        msgs = self._turn_messages(model_user_text, isolate, sp)
        prompt = self.tok.apply_chat_template(msgs, True, self._thinking, self.tags.open, self.tags.close)
        if self.debug:
            emit(self.listener, self, LlmTextKind.TEXT_DEBUG, prompt)
        ids = self.tok.encode(prompt, allow_special=True)
        dec = self.tok.stream_decoder(skip_special=True)
        stream = self._stream = _TurnStream()
        raw: List[str] = []
        scanner = ReplyScanner(self.tags, self.specials)  # fed one decoded delta per token, never rescanned

        def on_token(_i, _sid, token):
            delta = dec.push(token)
            if not delta:
                return
            raw.append(delta)
            p = scanner.feed(delta).snapshot()
            stream.push(self.listener, self, "".join(raw), p.thinking, p.answer, p.think_open)

        out = self.llm.generate_token_ids([ids], sp, on_token=on_token if self.listener else None,
                                          timeout_s=self.timeout_s)[0]
        full = self.tok.decode(out.token_ids, skip_special=True)
        p = parse(full, self.tags, self.specials)
        return ChatReply(p.answer, p.thinking, full, getattr(self.llm, "last_stats", None), think_open=p.think_open)

    def _finish(self, reply: ChatReply) -> ChatReply:
        answer, thinking = reply.answer.strip(), reply.thinking
        salvaged = False
        if should_salvage(answer, thinking):
            answer = salvage_from_thinking(thinking)
            salvaged = True
            self._diag("(reply recovered from unclosed thinking)\n" if reply.think_open else
                       "(reply recovered from thinking: the visible answer was missing or truncated)\n")
        if not answer.strip():
            answer = self.fallback_reply
            self._diag("(empty reply: used fallback)\n")
        done = ChatReply(answer, thinking, reply.raw, reply.stats, salvaged=salvaged)
        if self._stream is not None:
            self._stream.push(self.listener, self, reply.raw, thinking, answer, False)
        self.history.append(ChatMessage.assistant(done.answer))
        self._cap()
        self.last_reply = done
        return done
