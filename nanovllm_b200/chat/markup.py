"""Assistant-reply markup: think tags, chat special markers, reply parsing and salvage.

Observable behaviour follows the reference's chat layer (nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/
chat/AssistantParts.java, ChatReply.java, ThinkTags.java, ChatSpecials.java): text inside think tags is thinking
(several blocks, or a block still open at the end), the rest is the answer; a chat special marker ends the
answer; an incomplete marker at the end of a streaming buffer is held back so it never reaches the screen; an
answer can be salvaged from the thinking when the model never produced one.

The implementation is an incremental scanner (``ReplyScanner``): text is fed chunk by chunk as tokens stream in,
every complete marker is consumed exactly once as a state transition (lead -> think / answer -> done), and only
the unconsumed tail that could still grow into a marker is kept between feeds.  ``parse`` is a scanner fed once.
"""
from __future__ import annotations

import re
from dataclasses import dataclass, field
from typing import List, Optional, Tuple


@dataclass(frozen=True)
class ThinkTags:
    open: str = "<think>"
    close: str = "</think>"

    @staticmethod
    def default() -> "ThinkTags":
        return ThinkTags()

    @staticmethod
    def of(open_tag: str, close_tag: str) -> "ThinkTags":
        if not open_tag or not close_tag or open_tag == close_tag:
            raise ValueError("think tags must be two different non-empty strings")
        return ThinkTags(open_tag, close_tag)


DEFAULT_SPECIALS = ("<|im_end|>", "<|im_start|>", "<|endoftext|>", "<end_of_turn>", "<start_of_turn>", "<turn|>",
                    "<|turn>", "</s>", "<eos>", "<|eot_id|>")


@dataclass(frozen=True)
class ChatSpecials:
    markers: Tuple[str, ...] = DEFAULT_SPECIALS

    @staticmethod
    def default() -> "ChatSpecials":
        return ChatSpecials()

    def search_markers(self, tags: ThinkTags) -> List[str]:
        return list(self.markers) + [tags.open, tags.close]


@dataclass(frozen=True)
class AssistantParts:
    thinking: str
    answer: str
    think_open: bool


# scanner states
_LEAD, _THINK, _ANSWER, _DONE = "lead", "think", "answer", "done"


@dataclass
class ReplyScanner:
    """Streaming splitter of raw assistant text into thinking and answer.

    States: ``lead`` (no tag seen yet: the text is provisional -- a first close tag turns it into thinking, a
    first open tag or a special marker into answer), ``think``, ``answer`` and ``done`` (a special marker or a
    stray close tag ended the answer; later text is ignored).  Think and answer text accumulate as segments, one
    per block; ``snapshot`` joins them."""
    tags: ThinkTags = field(default_factory=ThinkTags)
    specials: ChatSpecials = field(default_factory=ChatSpecials)
    state: str = _LEAD
    _tail: str = ""
    _lead: List[str] = field(default_factory=list)
    _think: List[List[str]] = field(default_factory=list)
    _answer: List[List[str]] = field(default_factory=list)

    def __post_init__(self):
        self._markers = self.specials.search_markers(self.tags)
        self._pattern = re.compile("|".join(re.escape(m) for m in sorted(set(self._markers), key=len, reverse=True)))

    # -------------------------------------------------------------------------------- feeding
    def feed(self, chunk: str) -> "ReplyScanner":
        text = self._tail + (chunk or "")
        pos = 0
        for m in self._pattern.finditer(text):
            self._emit(text[pos:m.start()])
            self._on_marker(m.group(0))
            pos = m.end()
        rest = text[pos:]
        keep = self._marker_prefix_len(rest)
        self._emit(rest[:len(rest) - keep])
        self._tail = rest[len(rest) - keep:]
        return self

    def _marker_prefix_len(self, text: str) -> int:
        """Length of the longest suffix of ``text`` that is a proper prefix of some marker (held back)."""
        best = 0
        for m in self._markers:
            for k in range(min(len(m) - 1, len(text)), best, -1):
                if text.endswith(m[:k]):
                    best = k
                    break
        return best

    def _emit(self, s: str) -> None:
        if not s or self.state == _DONE:
            return
        if self.state == _LEAD:
            self._lead.append(s)
        elif self.state == _THINK:
            self._think[-1].append(s)
        else:
            self._answer[-1].append(s)

    def _on_marker(self, mk: str) -> None:
        st = self.state
        if st == _DONE:
            return
        if mk == self.tags.open:
            if st == _LEAD:
                self._answer.append(self._lead)
                self._lead = []
            if st != _THINK:  # an open tag inside thinking is dropped
                self._think.append([])
                self.state = _THINK
        elif mk == self.tags.close:
            if st == _LEAD:  # everything before a first, unopened close tag was thinking
                self._think.append(self._lead)
                self._lead = []
            if st in (_LEAD, _THINK):
                self._answer.append([])
                self.state = _ANSWER
            else:  # a stray close tag in the answer ends it
                self.state = _DONE
        else:  # chat special marker: ends the answer, dropped from thinking
            if st == _LEAD:
                self._answer.append(self._lead)
                self._lead = []
                self.state = _DONE
            elif st == _ANSWER:
                self.state = _DONE

    # -------------------------------------------------------------------------------- results
    def snapshot(self) -> AssistantParts:
        think = [("".join(seg)).strip() for seg in self._think]
        thinking = "\n".join(t for t in think if t)
        segments = list(self._answer)
        if self.state == _LEAD:
            segments = segments + [self._lead]
        answer = ""
        for seg in segments:
            piece = "".join(seg)
            if not piece.strip():
                continue
            answer = piece if not answer.strip() else answer.rstrip() + "\n" + piece.lstrip()
        return AssistantParts(thinking, answer.strip(), self.state == _THINK)


def parse(raw: Optional[str], tags: ThinkTags = ThinkTags(), specials: ChatSpecials = ChatSpecials()) -> AssistantParts:
    """Split complete (or partially streamed) assistant text into thinking, answer and think-still-open."""
    if raw is None or not raw.strip():
        return AssistantParts("", "", False)
    return ReplyScanner(tags, specials).feed(raw).snapshot()


def strip_chat_markup(text: str, tags: ThinkTags = ThinkTags(), specials: ChatSpecials = ChatSpecials()) -> str:
    out = text or ""
    for m in specials.search_markers(tags):
        out = out.replace(m, "")
    return out.strip()


# -------------------------------------------------------------------------------------------- salvage
# A line that states its result: "answer: X", "final answer = X", "so the answer is - X", "therefore: X".
_STATED = re.compile(r"(?i)\b(?:final answer|answer|so the answer is|therefore)\s*[:=\-]\s*(.+)$")


def _stated_value(line: str) -> str:
    m = _STATED.search(line)
    return re.sub(r"[.\"']+$", "", m.group(1).strip()) if m else ""


def salvage_from_thinking(thinking: Optional[str]) -> str:
    """Recover a short answer from thinking text when the model never produced one.

    Candidate lines are the non-empty ones that are not list continuations ("+ ...").  Walking back from the
    last candidate, the first line that states a result gives that result, and the first brief line (at most
    120 characters, not a question) is taken as is; with neither, the last candidate is returned, cut to 200
    characters."""
    if not thinking or not thinking.strip():
        return ""
    candidates = [ln.strip() for ln in thinking.strip().splitlines()]
    candidates = [ln for ln in candidates if ln and not ln.startswith("+")]
    for ln in reversed(candidates):
        stated = _stated_value(ln)
        if stated:
            return stated
        if len(ln) <= 120 and not ln.endswith("?"):
            return ln
    if not candidates:
        return ""
    last = candidates[-1]
    return last if len(last) <= 200 else last[:200].strip() + "…"


def clean_assistant_text(raw: Optional[str], tags: ThinkTags = ThinkTags(),
                         specials: ChatSpecials = ChatSpecials()) -> str:
    p = parse(raw, tags, specials)
    return p.answer if p.answer else salvage_from_thinking(p.thinking)


def stream_display_text(raw: Optional[str], tags: ThinkTags = ThinkTags(),
                        specials: ChatSpecials = ChatSpecials()) -> str:
    return parse(raw, tags, specials).answer


@dataclass
class ChatReply:
    """Final result of one chat turn (ChatReply.java:49-318)."""
    answer: str
    thinking: str = ""
    raw: str = ""
    stats: Optional[object] = None
    salvaged: bool = False
    think_open: bool = False

    @staticmethod
    def parse(raw: str, tags: ThinkTags = ThinkTags(), specials: ChatSpecials = ChatSpecials()) -> "ChatReply":
        p = parse(raw, tags, specials)
        if p.answer:
            return ChatReply(p.answer, p.thinking, raw, think_open=p.think_open)
        return ChatReply(salvage_from_thinking(p.thinking), p.thinking, raw, salvaged=True, think_open=p.think_open)

    def has_answer(self) -> bool:
        return bool(self.answer.strip())
