"""Listener / event bus for streamed text and status.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/chat/{LlmTextKind.java:13-45, LlmListener.java,
LlmTextEvent.java, LlmListeners.java:22-291}: events carry a kind (thinking, assistant, raw, advisor note,
diagnostics, debug, status info / progress) and text; helpers build silent, print-stream and composed listeners.
"""
from __future__ import annotations

import enum
import sys
import time
from dataclasses import dataclass, field
from typing import Callable, Iterable, Optional, TextIO


class LlmTextKind(enum.Enum):
    TEXT_THINKING = "thinking"
    TEXT_ASSISTANT = "assistant"
    TEXT_RAW = "raw"
    TEXT_ADVISOR_NOTE = "advisor_note"
    TEXT_DIAGNOSTICS = "diagnostics"
    TEXT_DEBUG = "debug"
    STATUS_INFO = "status_info"
    STATUS_PROGRESS = "status_progress"

    def is_status(self) -> bool:
        return self in (LlmTextKind.STATUS_INFO, LlmTextKind.STATUS_PROGRESS)


@dataclass(frozen=True)
class LlmTextEvent:
    """``snapshot`` is True when ``text`` REPLACES what was shown for this kind (the parse changed earlier text,
    e.g. a held marker resolved), False when it is a delta appended to it."""
    kind: LlmTextKind
    text: str
    snapshot: bool = False
    timestamp: float = field(default_factory=time.time)


LlmListener = Callable[[object, LlmTextEvent], None]


class LlmListeners:
    @staticmethod
    def silent() -> LlmListener:
        return lambda source, ev: None

    @staticmethod
    def to_print_streams(out: Optional[TextIO] = None, err: Optional[TextIO] = None) -> LlmListener:
        """Assistant text to ``out``; thinking, status and diagnostics to ``err`` (default: the process's
        stdout / stderr at the time of each event)."""
        def listener(source, ev: LlmTextEvent):
            if ev.kind == LlmTextKind.TEXT_ASSISTANT:
                stream = out if out is not None else sys.stdout
            else:
                stream = err if err is not None else sys.stderr
            if ev.kind in (LlmTextKind.TEXT_RAW, LlmTextKind.TEXT_DEBUG):
                return
            stream.write(ev.text)
            stream.flush()
        return listener

    @staticmethod
    def to_system() -> LlmListener:
        return LlmListeners.to_print_streams(sys.stdout, sys.stderr)

    @staticmethod
    def compose(*listeners: Optional[LlmListener]) -> LlmListener:
        ls = [x for x in listeners if x is not None]

        def listener(source, ev):
            for x in ls:
                x(source, ev)
        return listener

    @staticmethod
    def collecting(kinds: Optional[Iterable[LlmTextKind]] = None):
        """-> (listener, list) that appends matching events to the list (tests, transcripts)."""
        events = []
        allowed = set(kinds) if kinds is not None else None

        def listener(source, ev):
            if allowed is None or ev.kind in allowed:
                events.append(ev)
        return listener, events


def info(listener: Optional[LlmListener], source, text: str) -> None:
    if listener is not None:
        listener(source, LlmTextEvent(LlmTextKind.STATUS_INFO, text))


def progressf(listener: Optional[LlmListener], source, fmt: str, *args) -> None:
    if listener is not None:
        listener(source, LlmTextEvent(LlmTextKind.STATUS_PROGRESS, fmt % args if args else fmt))


def emit(listener: Optional[LlmListener], source, kind: LlmTextKind, text: str, snapshot: bool = False) -> None:
    if listener is not None and (text or snapshot):
        listener(source, LlmTextEvent(kind, text, snapshot))
