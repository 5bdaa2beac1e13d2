"""Retrieval-augmented chat on top of ``ChatSession``.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/rag/RagSession.java:40-865.  A turn:

1. resolve the retrieval query: nothing when the index says the question is outside the corpus; a short
   follow-up (< 6 index tokens) with an anchor from an earlier turn is used as-is when it already hits, else
   rewritten by the model into search keywords (temperature 0.1, <= 48 tokens; "NONE" means no search) or,
   failing that, expanded as ``anchor + "\\n" + question``;
2. retrieve ``4 x top_k`` candidates; a short follow-up prefers passages from the previous turn's source when
   that source's best hit is within 55% of the overall best; clip to ``top_k``;
3. format the model turn: ``- passage`` lines capped at ``max_context_chars`` behind a grounding line, question
   last (plain question when nothing was found);
4. sampling: grounded turns cap temperature at 0.15, turns without hits get at least ``max_tokens_when_no_hits``;
   a turn without hits (or with ``isolate_generation``) is generated without earlier dialog;
5. history keeps the raw question (``ChatSession.send_prepared``).
"""
from __future__ import annotations

import re
from typing import List, Optional

from ..chat import prompts
from ..chat.markup import ChatReply, ThinkTags
from ..chat.messages import ChatMessage
from ..chat.session import ChatSession
from ..sampling_params import SamplingParams
from .lexical import RagHit, RagIndex, tokenize

GROUNDED_TEMPERATURE_CAP = 0.15
SHORT_FOLLOW_UP_MAX_TOKENS = 6
PRIOR_SOURCE_COMPETITIVE = 0.55
_SEARCH_PREFIX = re.compile(r"(?i)^\s*(?:search\s*:\s*)?")
_WRAP_QUOTES = re.compile(r"^[\"'`]+|[\"'`]+$")


def short_follow_up(question: str) -> bool:
    return len(tokenize(question)) < SHORT_FOLLOW_UP_MAX_TOKENS


def format_user_message(hits: List[RagHit], question: str, max_context_chars: int = 1 << 30) -> str:
    q = question.strip()
    if not q:
        raise ValueError("question must not be blank")
    if max_context_chars < 64:
        raise ValueError("max_context_chars must be >= 64")
    parts, used = [], 0
    for h in hits:
        block = "- " + h.chunk.text.strip()
        nxt = len(block) if used == 0 else used + 2 + len(block)
        if nxt > max_context_chars and used > 0:
            break
        if len(block) > max_context_chars and used == 0:
            parts.append(block[:max_context_chars])
            break
        parts.append(block)
        used = nxt
    context = "\n".join(parts)
    return prompts.with_context(q, context) if context.strip() else prompts.without_context(q)


def parse_rewrite(raw: Optional[str], tags: ThinkTags = ThinkTags()) -> Optional[str]:
    if not raw or not raw.strip():
        return None
    answer = ChatReply.parse(raw, tags).answer.strip()
    first = next((ln.strip() for ln in answer.splitlines() if ln.strip()), "")
    cleaned = _WRAP_QUOTES.sub("", _SEARCH_PREFIX.sub("", first, count=1)).strip()
    if not cleaned or cleaned.lower() == "none":
        return None
    return cleaned[:240].strip()


def prefer_prior_source(cands: List[RagHit], prior: str, top_k: int) -> List[RagHit]:
    if not cands:
        return []
    if not prior:
        return cands[:top_k]
    same = [h for h in cands if h.chunk.source == prior]
    if same and same[0].score >= cands[0].score * PRIOR_SOURCE_COMPETITIVE:
        return same[:top_k]
    return cands[:top_k]


class RagSession:
    def __init__(self, llm, index: RagIndex, chat: Optional[ChatSession] = None, top_k: int = 4,
                 max_context_chars: int = 3500, max_tokens_when_no_hits: int = 384, isolate_generation: bool = False,
                 sampling: Optional[SamplingParams] = None):
        self.llm = llm
        self.index = index
        self.chat = chat or ChatSession(llm)
        self.chat.enable_thinking(False)
        self.base_sampling = sampling or self.chat.sampling_params()
        self.top_k(top_k).max_context(max_context_chars)
        if max_tokens_when_no_hits < 1:
            raise ValueError("max_tokens_when_no_hits must be >= 1")
        self._no_hit_tokens = max_tokens_when_no_hits
        self._isolate = isolate_generation
        self.last_hits: List[RagHit] = []
        self.anchor_query = ""
        self.last_source = ""
        self.last_retrieval_query = ""

    # knobs
    def top_k(self, k: int) -> "RagSession":
        if k <= 0:
            raise ValueError("top_k must be > 0")
        self._top_k = k
        return self

    def max_context(self, chars: int) -> "RagSession":
        if chars < 64:
            raise ValueError("max_context_chars must be >= 64")
        self.max_context_chars = chars
        return self

    def sampling(self, sp: SamplingParams) -> "RagSession":
        self.base_sampling = sp
        return self

    def deterministic(self) -> "RagSession":
        return self.sampling(self.base_sampling.deterministic())

    def seed(self, *messages: ChatMessage) -> "RagSession":
        self.chat.history.extend(messages)
        return self

    def listen(self, listener) -> "RagSession":
        self.chat.listen(listener)
        return self

    # the reference session's other knobs (RagSession.java:96-400): RAG ones here, chat ones forwarded
    @staticmethod
    def open(llm_or_chat, index: RagIndex, max_tokens: Optional[int] = None) -> "RagSession":
        """``open(llm, index[, max_tokens])`` or ``open(chat_session, index)`` (reuses its dialog and knobs)."""
        if isinstance(llm_or_chat, ChatSession):
            return RagSession(llm_or_chat.llm, index, chat=llm_or_chat)
        chat = ChatSession.open(llm_or_chat, max_tokens) if max_tokens is not None else None
        return RagSession(llm_or_chat, index, chat=chat)

    @staticmethod
    def format_user_message(hits: List[RagHit], question: str, max_context_chars: Optional[int] = None) -> str:
        """The model-facing grounded turn: retrieved passages, then the question."""
        return format_user_message(hits, question, max_context_chars if max_context_chars is not None else 1 << 30)

    def max_tokens_when_no_hits(self, n: int) -> "RagSession":
        if n < 1:
            raise ValueError("max_tokens_when_no_hits must be >= 1")
        self._no_hit_tokens = int(n)
        return self

    def isolate_generation(self, on: bool = True) -> "RagSession":
        self._isolate = bool(on)
        return self

    def _forward(self, name: str, *args) -> "RagSession":
        getattr(self.chat, name)(*args)
        return self

    def timeout(self, seconds: Optional[float]) -> "RagSession":
        return self._forward("timeout", seconds)

    def enable_thinking(self, on: bool = True) -> "RagSession":
        return self._forward("enable_thinking", on)

    def think_tags(self, tags: ThinkTags) -> "RagSession":
        return self._forward("think_tags", tags)

    def max_history_messages(self, n: int) -> "RagSession":
        return self._forward("max_history_messages", n)

    def recover_unusable_answers(self, on: bool = True) -> "RagSession":
        return self._forward("recover_unusable_answers", on)

    def unusable_answer(self, predicate) -> "RagSession":
        return self._forward("unusable_answer", predicate)

    def unusable_answer_fallback(self, text: str) -> "RagSession":
        return self._forward("unusable_answer_fallback", text)

    def emit_debug_prompts(self, on: bool = True) -> "RagSession":
        return self._forward("emit_debug_prompts", on)

    def diagnostics(self, consumer) -> "RagSession":
        return self._forward("diagnostics", consumer)

    def stream_to(self, think_out=None, answer_out=None) -> "RagSession":
        return self._forward("stream_to", think_out, answer_out)

    def clear(self) -> None:
        self.chat.clear()
        self.last_hits, self.anchor_query, self.last_source, self.last_retrieval_query = [], "", "", ""

    # turns
    def ask(self, question: str) -> str:
        return self.send(question).answer

    def send(self, question: str) -> ChatReply:
        q = (question or "").strip()
        if not q:
            raise ValueError("question must not be blank")
        if self.index.size() == 0:
            self.last_hits, self.last_retrieval_query = [], ""
            return self.chat.send(q)
        self.last_hits = self._retrieve(q)
        if short_follow_up(q):
            if self.last_hits and self.last_retrieval_query.strip():
                self.anchor_query = self.last_retrieval_query
        else:
            self.anchor_query = q
        if self.last_hits:
            self.last_source = self.last_hits[0].chunk.source
        prompt = format_user_message(self.last_hits, q, self.max_context_chars)
        base = self.base_sampling
        if not self.last_hits:
            sp = base.with_(max_tokens=max(base.max_tokens, self._no_hit_tokens))
        else:
            sp = base.with_(temperature=min(base.temperature, GROUNDED_TEMPERATURE_CAP))
        isolate = not self.last_hits or self._isolate
        return self.chat.send_prepared(q, prompt, isolate=isolate, sampling=sp)

    def _retrieve(self, q: str) -> List[RagHit]:
        query = self._resolve_query(q)
        if query is None:
            self.last_retrieval_query = ""
            return []
        self.last_retrieval_query = query
        cands = self.index.retrieve(query, max(self._top_k * 4, self._top_k))
        if short_follow_up(q) and self.last_source:
            return prefer_prior_source(cands, self.last_source, self._top_k)
        return cands[:self._top_k]

    def _resolve_query(self, q: str) -> Optional[str]:
        if self.index.is_outside_corpus(q):
            return None
        if short_follow_up(q) and self.anchor_query.strip():
            if self.index.retrieve(q, 1):
                return q
            rewritten = self._rewrite(self.anchor_query, q)
            if rewritten is not None and not self.index.is_outside_corpus(rewritten):
                return rewritten
            return f"{self.anchor_query}\n{q}"
        return q

    def _rewrite(self, prior: str, follow_up: str) -> Optional[str]:
        tok = self.llm.tokenizer
        user = prompts.rewrite_follow_up(prior.strip(), follow_up.strip()) if prior.strip() else \
            prompts.rewrite_standalone(follow_up.strip())
        tags = self.chat.tags
        text = tok.apply_chat_template([ChatMessage.user(user)], True, False, tags.open, tags.close)
        out = self.llm.generate_token_ids([tok.encode(text, allow_special=True)],
                                          SamplingParams(temperature=0.1, max_tokens=48))[0]
        return parse_rewrite(tok.decode(out.token_ids, skip_special=True), tags)
