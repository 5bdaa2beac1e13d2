"""Prompt layouts shared by RAG and advisors.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/prompts/{RagPrompts.java:12-97,
AdvisorPrompts.java:14-76, ChatPrompts.java:10-44} and llm/AdvisorPrompt.java:27-257.

A grounded user turn has the layout ``<grounding line>\\n\\n<facts block>\\n\\n<question>``: the question is
always the text after the LAST blank line and the facts are everything before it (minus the grounding line).
Advisor notes become ``- note`` lines appended to the facts block (or to a new one), so the question stays last
and RAG passages keep coming first.  A note is only mixed into a grounded turn when at least 60% of its
contentful terms (letters/digits runs of length >= 4) also occur in the passages.
"""
from __future__ import annotations

import re
from typing import Iterable, List, Optional, Sequence, Set

ABSTAIN_REPLY = "I do not know"
GROUNDING = "Answer from the passages below only; do not make up titles, people or sources."
REWRITE_STANDALONE = ("Turn this question into a few search keywords for a document index.\n"
                      "Reply with the keywords only, or NONE when there is nothing to search for.\n"
                      "Question: {q}")
REWRITE_FOLLOW_UP = ("Turn this follow-up into a few search keywords for a document index.\n"
                     "Where the follow-up says it, they or that, name what it means, taken from Prior.\n"
                     "Reply with the keywords only, or NONE when the follow-up has nothing to do with Prior.\n"
                     "Prior: {prior}\n"
                     "Follow-up: {q}")

_ABSTAIN_RE = re.compile(r"(?i)^\s*" + re.escape(ABSTAIN_REPLY) + r"\.?\s*$")
_TERM = re.compile(r"[^\W_]+", re.UNICODE)
CONTENTFUL_MIN_LEN = 4
GROUNDING_COVERAGE = 0.6


# ------------------------------------------------------------------------------------------------ RAG layout
def with_context(question: str, context: str) -> str:
    return f"{GROUNDING}\n\n{context.strip()}\n\n{question.strip()}"


def without_context(question: str) -> str:
    return question.strip()


def _strip_grounding(block: str) -> str:
    if block == GROUNDING:
        return ""
    if block.startswith(GROUNDING):
        return block[len(GROUNDING):].strip()
    return block


def facts(document: Optional[str]) -> str:
    if not document or not document.strip():
        return ""
    text = document.strip()
    sep = text.rfind("\n\n")
    return _strip_grounding(text[:sep].strip()) if sep >= 0 else ""


def question(document: Optional[str]) -> str:
    if not document or not document.strip():
        return ""
    text = document.strip()
    sep = text.rfind("\n\n")
    return text[sep + 2:].strip() if sep >= 0 else text


def has_facts(document: Optional[str]) -> bool:
    return bool(facts(document).strip())


def rewrite_standalone(q: str) -> str:
    return REWRITE_STANDALONE.format(q=q).strip()


def rewrite_follow_up(prior: str, q: str) -> str:
    return REWRITE_FOLLOW_UP.format(prior=prior, q=q).strip()


def fold_system_into_first_user(system: Optional[str], user: Optional[str], first_user: bool) -> str:
    """For templates without a system role: the system text leads the first user turn."""
    content = user or ""
    if not first_user or not system or not system.strip():
        return content
    return f"{system}\n\n{content}"


# ------------------------------------------------------------------------------------------------ advisor notes
def note_line(note: str) -> str:
    return "- " + note.strip().replace('"', "'")


def usable_note(note: Optional[str], keep=None) -> str:
    body = (note or "").strip()
    if not body or (keep is not None and not keep(body)):
        return ""
    return body


def is_abstention(note: Optional[str]) -> bool:
    if note is None:
        return False
    s = note.strip()
    if _ABSTAIN_RE.match(s):
        return True
    low, ab = s.lower(), ABSTAIN_REPLY.lower()
    if not low.startswith(ab):
        return False
    return len(s) == len(ab) or s[len(ab)] in ".!?" or s[len(ab)].isspace()


def contentful_terms(text: Optional[str]) -> Set[str]:
    if not text or not text.strip():
        return set()
    return {t for t in _TERM.findall(text.lower()) if len(t) >= CONTENTFUL_MIN_LEN}


def is_grounded(note: str, context_terms: Set[str]) -> bool:
    if not context_terms:
        return False
    terms = contentful_terms(note)
    if not terms:
        return False
    hit = sum(1 for t in terms if t in context_terms)
    need = max(1, -(-len(terms) * 6 // 10))  # ceil(0.6 * n) in integers
    return hit >= need


def select_notes(model_user_text: str, notes: Sequence[Optional[str]]) -> List[str]:
    """Distinct usable notes; with passages in the turn, only notes grounded in them."""
    grounded_turn = has_facts(model_user_text)
    ctx = contentful_terms(facts(model_user_text)) if grounded_turn else set()
    out: List[str] = []
    for n in notes:
        body = usable_note(n)
        if not body or (grounded_turn and not is_grounded(body, ctx)) or body in out:
            continue
        out.append(body)
    return out


def with_notes(model_user_text: str, notes: Iterable[str]) -> str:
    base = model_user_text.strip()
    if not base:
        raise ValueError("model user text must not be blank")
    notes = list(notes)
    if not notes:
        return base
    f, q = facts(base), question(base)
    had_passages = bool(f.strip())
    if not q:
        q, f, had_passages = base, "", False
    block = "\n".join(line for line in (note_line(n) for n in notes) if line not in f)
    if not block:
        return base
    merged = block if not f.strip() else f + "\n" + block
    return with_context(q, merged) if had_passages else f"{merged}\n\n{q}"


def mix(model_user_text: str, answers: Sequence[Optional[str]]) -> str:
    base = model_user_text.strip()
    if not base:
        raise ValueError("model user text must not be blank")
    notes: List[str] = []
    for a in answers:
        body = usable_note(a)
        if body and body not in notes:
            notes.append(body)
    return with_notes(base, notes) if notes else base


def advisor_user(q: str, context: str) -> str:
    q = q.strip()
    if not q:
        raise ValueError("question must not be blank")
    return with_context(q, context) if context and context.strip() else q


def advisor_facing_user_text(model_user_text: str) -> str:
    """What an advisor sees: the question, plus the passages when the turn is grounded (no earlier notes)."""
    base = model_user_text.strip()
    if not base:
        return ""
    if has_facts(base):
        q, ctx = question(base), facts(base)
        if q and ctx:
            return advisor_user(q, ctx)
    return question(base)
