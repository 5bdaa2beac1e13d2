"""Assistant-reply markup: think tags, chat special markers, reply parsing and salvage.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/chat/{AssistantParts.java:23-261, ChatReply.java,
ThinkTags.java:27-75, ChatSpecials.java:30-90}.  ``parse`` splits raw model output into (thinking, answer,
think-still-open): text inside ``<think>..</think>`` (also several or an unclosed block) is thinking, the rest is
the answer; chat special markers end the answer; an incomplete marker at the end of a streaming buffer is held
back so it never flashes on screen.  ``salvage_from_thinking`` recovers a short answer from the thinking when the
model never closed its think block (a stated "answer: ..." line, else the last brief line).
"""
from __future__ import annotations

import re
from dataclasses import dataclass
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


def _hold_incomplete_suffix(text: str, markers: List[str]) -> str:
    """Drop a trailing prefix of any marker (the rest may still be streaming in)."""
    best = 0
    for m in markers:
        for k in range(min(len(m) - 1, len(text)), 0, -1):
            if text.endswith(m[:k]):
                best = max(best, k)
                break
    return text[:-best] if best else text


def _join_think(a: str, b: str) -> str:
    a, b = (a or "").strip(), (b or "").strip()
    if not a:
        return b
    if not b:
        return a
    return a + "\n" + b


def _join_answer(a: str, b: str) -> str:
    a, b = a or "", b or ""
    if not a.strip():
        return b
    if not b.strip():
        return a
    return a.rstrip() + "\n" + b.lstrip()


def _split_rest(text: str, tags: ThinkTags, markers: List[str]) -> Tuple[str, str, bool]:
    """-> (thinking, answer, open) of the text after a closed think block."""
    text = _hold_incomplete_suffix(text, markers)
    s = text.find(tags.open)
    if s < 0:
        return "", text, False
    before, inner = text[:s], text[s + len(tags.open):]
    e = inner.find(tags.close)
    if e < 0:
        return inner, before, True
    t2, a2, o2 = _split_rest(inner[e + len(tags.close):], tags, markers)
    return _join_think(inner[:e], t2), _join_answer(before, a2), o2


def strip_chat_markup(text: str, tags: ThinkTags = ThinkTags(), specials: ChatSpecials = ChatSpecials()) -> str:
    out = text or ""
    for m in specials.search_markers(tags):
        out = out.replace(m, "")
    return out.strip()


def _sanitize_answer(text: str, markers: List[str]) -> str:
    cleaned = _hold_incomplete_suffix(text, markers)
    for m in markers:
        at = cleaned.find(m)
        if at >= 0:
            cleaned = cleaned[:at]
    return cleaned.strip()


def parse(raw: Optional[str], tags: ThinkTags = ThinkTags(), specials: ChatSpecials = ChatSpecials()) -> AssistantParts:
    if raw is None or not raw.strip():
        return AssistantParts("", "", False)
    markers = specials.search_markers(tags)
    text = _hold_incomplete_suffix(raw, markers)
    s = text.find(tags.open)
    e = text.find(tags.close, s + len(tags.open)) if s >= 0 else text.find(tags.close)
    if s >= 0 and e > s:
        thinking = text[s + len(tags.open):e]
        t2, after, is_open = _split_rest(text[e + len(tags.close):], tags, markers)
        thinking = _join_think(thinking, t2)
    elif s >= 0:
        thinking, after, is_open = text[s + len(tags.open):], "", True
    elif e >= 0:
        thinking, after, is_open = _split_rest(text[e + len(tags.close):], tags, markers)
        thinking = _join_think(text[:e], thinking)
    else:
        thinking, after, is_open = "", text, False
    return AssistantParts(strip_chat_markup(thinking, tags, specials), _sanitize_answer(after, markers), is_open)


_STATED = re.compile(r"(?i)\b(?:final answer|answer|so the answer is|therefore)\s*[:=\-]\s*(.+)$")


def _brief(line: str) -> bool:
    return 0 < len(line) <= 120 and not line.endswith("?")


def salvage_from_thinking(thinking: Optional[str]) -> str:
    if not thinking or not thinking.strip():
        return ""
    lines = re.split(r"\r?\n", thinking.strip())
    for line in reversed(lines):
        line = line.strip()
        if not line or line.startswith("+"):
            continue
        m = _STATED.search(line)
        if m:
            got = re.sub(r"[.\"']+$", "", m.group(1).strip())
            if got:
                return got
        if _brief(line):
            return line
    for line in reversed(lines):
        line = line.strip()
        if line and not line.startswith("+"):
            return line[:200].strip() + "…" if len(line) > 200 else line
    return ""


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
