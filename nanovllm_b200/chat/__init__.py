"""Chat layer: messages and truncation, think-tag markup, listeners, advisors, ``ChatSession``."""
from .listeners import LlmListeners, LlmTextEvent, LlmTextKind
from .markup import AssistantParts, ChatReply, ChatSpecials, ThinkTags, clean_assistant_text, parse, salvage_from_thinking
from .messages import ChatMessage, truncate_history
from .session import AdvisorRunner, ChatSession, DefaultAdvisorMixer, LlmAdvisor

__all__ = ["LlmListeners", "LlmTextEvent", "LlmTextKind", "AssistantParts", "ChatReply", "ChatSpecials", "ThinkTags",
           "clean_assistant_text", "parse", "salvage_from_thinking", "ChatMessage", "truncate_history",
           "AdvisorRunner", "ChatSession", "DefaultAdvisorMixer", "LlmAdvisor"]
