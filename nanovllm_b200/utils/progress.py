"""In-place load progress (percent, ETA, current item) reported through the listener bus.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/llmcontainer/LoadProgress.java:13-88
(a 24-cell bar, percent, (i/n), ETA from the elapsed rate, the tail of the current item name, and a closing
"done in Xs" line; silent listeners cost nothing).
"""
from __future__ import annotations

import time
from typing import Optional

from ..chat.listeners import LlmListener, LlmTextEvent, LlmTextKind


def _fmt_seconds(s: float) -> str:
    return f"{s:.0f}s" if s < 60 else f"{int(s // 60)}m{int(s % 60):02d}s"


class LoadProgress:
    WIDTH = 24

    def __init__(self, label: str, total: int, listener: Optional[LlmListener] = None, source=None):
        self.label = label
        self.total = max(1, int(total))
        self.listener = listener
        self.source = source
        self.current = 0
        self.detail = ""
        self.finished = False
        self.t0 = time.perf_counter()
        self._render()

    def _emit(self, kind: LlmTextKind, text: str) -> None:
        if self.listener is not None:
            self.listener(self.source, LlmTextEvent(kind, text))

    def step(self, detail: str = "") -> None:
        self.current = min(self.current + 1, self.total)
        self.detail = detail or ""
        self._render()

    def finish(self, message: str = "") -> None:
        if self.finished:
            return
        self.finished = True
        took = time.perf_counter() - self.t0
        self._emit(LlmTextKind.STATUS_INFO, f"\r{self.label}: done in {took:.1f}s" + (f" - {message}" if message else "") + "\n")

    def line(self) -> str:
        frac = self.current / self.total
        filled = int(round(frac * self.WIDTH))
        bar = "=" * filled + " " * (self.WIDTH - filled)
        el = time.perf_counter() - self.t0
        eta = "--" if self.current <= 0 else _fmt_seconds(el * (1.0 - frac) / frac)
        d = self.detail if len(self.detail) <= 48 else "..." + self.detail[-45:]
        return f"\r{self.label}: [{bar}] {frac * 100:3.0f}% ({self.current}/{self.total}) ETA {eta}  {d}   "

    def _render(self) -> None:
        if self.finished or self.listener is None:
            return
        self._emit(LlmTextKind.STATUS_PROGRESS, self.line())
