"""Chat messages and prompt-budget history truncation.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/chat/ChatMessages.java:59-130 -- the prompt
budget is ``max(64, max_model_len - max_tokens - 16)`` tokens of the templated history; while over budget the
oldest non-system message is dropped, together with the assistant reply that answered it, and the system
message plus the newest user turn always stay.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List

from .markup import ThinkTags

PROMPT_MARGIN = 16


@dataclass
class ChatMessage:
    role: str
    content: str

    @staticmethod
    def system(text: str) -> "ChatMessage":
        return ChatMessage("system", text)

    @staticmethod
    def user(text: str) -> "ChatMessage":
        return ChatMessage("user", text)

    @staticmethod
    def assistant(text: str) -> "ChatMessage":
        return ChatMessage("assistant", text)


def truncate_history(history: List[ChatMessage], tokenizer, max_model_len: int, max_tokens: int,
                     enable_thinking: bool = False, tags: ThinkTags = ThinkTags()) -> None:
    budget = max(64, max_model_len - max_tokens - PROMPT_MARGIN)
    min_keep = 2 if history and history[0].role == "system" else 1
    while len(history) > min_keep:
        prompt = tokenizer.apply_chat_template(history, True, enable_thinking, tags.open, tags.close)
        if len(tokenizer.encode(prompt)) <= budget:
            return
        drop = 1 if history[0].role == "system" else 0
        if drop >= len(history):
            return
        history.pop(drop)
        if drop < len(history) and history[drop].role == "assistant":
            history.pop(drop)
