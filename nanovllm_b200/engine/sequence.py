"""Per-request state of the continuous-batching engine.

Behavior follows nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/engine/Sequence.java:
a process-wide monotonically increasing ``seq_id`` (Sequence.java:28-86), the token list with the prompt
length, the page table (``block_table``), cached / scheduled token counters, per-request sampling knobs, and a
WAITING -> RUNNING -> FINISHED status.  Block math (Sequence.java:323-350): ``num_blocks`` is
ceil(len / block_size) and ``block(i)`` is the i-th page's token slice.

The degenerate-repetition stop (Sequence.java:379-449) is reproduced: after >= 32 completion tokens the
sequence stops on a >= 32 same-token streak, on two identical trailing halves with period 16..64 (step 8),
or, after >= 48 completion tokens, on any 12-gram seen 3 times in the last 128 completion tokens.

New: per-request timestamps (arrival, first token, finish) so the engine reports TTFT / TPOT.
"""
from __future__ import annotations

import enum
import itertools
import time
from typing import List, Optional

from ..sampling_params import SamplingParams


class SequenceStatus(enum.Enum):
    WAITING = 0
    RUNNING = 1
    FINISHED = 2


_SEQ_COUNTER = itertools.count()


class Sequence:
    __slots__ = ("seq_id", "token_ids", "num_tokens", "num_prompt_tokens", "last_token", "block_size",
                 "block_table", "num_cached_tokens", "num_scheduled_tokens", "status", "is_prefill",
                 "temperature", "top_k", "top_p", "max_tokens", "ignore_eos", "seed", "t_arrival",
                 "t_first_token", "t_finish", "user_tag", "bt_gen", "_ngrams")

    def __init__(self, token_ids: List[int], sampling: Optional[SamplingParams] = None, block_size: int = 256,
                 user_tag=None):
        if not token_ids:
            raise ValueError("prompt must contain at least one token")
        sp = sampling or SamplingParams()
        self.seq_id = next(_SEQ_COUNTER)
        self.token_ids = list(token_ids)
        self.num_tokens = len(self.token_ids)
        self.num_prompt_tokens = self.num_tokens
        self.last_token = self.token_ids[-1]
        self.block_size = block_size
        self.block_table: List[int] = []
        self.bt_gen = 0  # bumped whenever the block table is released (preemption, finish)
        self.num_cached_tokens = 0
        self.num_scheduled_tokens = 0
        self.status = SequenceStatus.WAITING
        self.is_prefill = True
        self.temperature = sp.temperature
        self.top_k = sp.top_k
        self.top_p = sp.top_p
        self.max_tokens = sp.max_tokens
        self.ignore_eos = sp.ignore_eos
        self.seed = sp.seed
        self.t_arrival = time.perf_counter()
        self.t_first_token: Optional[float] = None
        self.t_finish: Optional[float] = None
        self.user_tag = user_tag
        self._ngrams: Optional[_NgramWindow] = None  # created by the first n-gram check

    @classmethod
    def mirror(cls, seq_id: int, token_ids: List[int], num_prompt_tokens: int, block_size: int) -> "Sequence":
        """A copy of another rank's sequence, kept up to date from step plans (no id drawn, no validation)."""
        s = cls.__new__(cls)
        s.seq_id = seq_id
        s.token_ids = list(token_ids)
        s.num_tokens = len(s.token_ids)
        s.num_prompt_tokens = num_prompt_tokens
        s.last_token = s.token_ids[-1]
        s.block_size = block_size
        s.block_table = []
        s.bt_gen = 0
        s.num_cached_tokens = 0
        s.num_scheduled_tokens = 0
        s.status = SequenceStatus.RUNNING
        s.is_prefill = True
        s.temperature, s.top_k, s.top_p, s.max_tokens, s.ignore_eos, s.seed = 1.0, 0, 1.0, 0, True, None
        s.t_arrival, s.t_first_token, s.t_finish = time.perf_counter(), None, None
        s.user_tag = None
        s._ngrams = None
        return s

    def __len__(self):
        return self.num_tokens

    @property
    def is_finished(self) -> bool:
        return self.status == SequenceStatus.FINISHED

    @property
    def num_completion_tokens(self) -> int:
        return self.num_tokens - self.num_prompt_tokens

    @property
    def prompt_token_ids(self) -> List[int]:
        return self.token_ids[:self.num_prompt_tokens]

    @property
    def completion_token_ids(self) -> List[int]:
        return self.token_ids[self.num_prompt_tokens:]

    @property
    def num_cached_blocks(self) -> int:
        return self.num_cached_tokens // self.block_size

    @property
    def num_blocks(self) -> int:
        return (self.num_tokens + self.block_size - 1) // self.block_size

    @property
    def last_block_num_tokens(self) -> int:
        return self.num_tokens - (self.num_blocks - 1) * self.block_size

    def block(self, i: int) -> List[int]:
        if not (0 <= i < self.num_blocks):
            raise IndexError(i)
        return self.token_ids[i * self.block_size:(i + 1) * self.block_size]

    def append_token(self, token_id: int) -> None:
        self.token_ids.append(int(token_id))
        self.last_token = int(token_id)
        self.num_tokens += 1
        if self.t_first_token is None:
            self.t_first_token = time.perf_counter()

    # ----------------------------------------------------------- degenerate-repetition stop
    def has_degenerate_repetition(self) -> bool:
        completion = self.num_completion_tokens
        if completion < 32:
            return False
        if self._same_token_streak() >= 32:
            return True
        ids = self.token_ids
        last = self.num_tokens - 1
        max_period = min(64, completion // 2)
        for period in range(16, max_period + 1, 8):
            # two equal trailing halves must at least end in equal tokens: one compare rejects almost every period
            if ids[last] == ids[last - period] and self._ends_with_two_identical_blocks(period):
                return True
        return completion >= 48 and self._has_overused_ngram()

    def _same_token_streak(self) -> int:
        streak = 0
        ids = self.token_ids
        for i in range(self.num_tokens - 1, self.num_prompt_tokens - 1, -1):
            if ids[i] != self.last_token:
                break
            streak += 1
        return streak

    def _ends_with_two_identical_blocks(self, period: int) -> bool:
        start = self.num_tokens - 2 * period
        if start < self.num_prompt_tokens:
            return False
        ids = self.token_ids
        return ids[start:start + period] == ids[start + period:start + 2 * period]

    def _has_overused_ngram(self, ngram: int = 12, min_hits: int = 3) -> bool:
        """True when some ``ngram``-gram lying inside the last min(completion, 128) tokens occurs ``min_hits``
        times there.  The counts are kept across calls and slid by the tokens appended since the previous call
        (one n-gram added at the front, one dropped at the back per token) instead of recounting the window."""
        window = min(self.num_completion_tokens, 128)
        if window < ngram * min_hits:
            return False
        start0 = self.num_tokens - window
        w = self._ngrams
        if w is None or w.ngram != ngram or w.min_hits != min_hits:
            w = self._ngrams = _NgramWindow(start0, ngram, min_hits)
        return w.advance(self.token_ids, self.num_tokens, start0)


class _NgramWindow:
    """Occurrence counts of the n-grams whose starts lie in [lo, hi), with the number of n-grams counted at least
    ``min_hits`` times; ``advance`` moves both ends forward over a token list that only grows at its end."""
    __slots__ = ("ngram", "min_hits", "counts", "over", "lo", "hi")

    def __init__(self, start: int, ngram: int, min_hits: int):
        self.ngram = ngram
        self.min_hits = min_hits
        self.counts = {}
        self.over = 0
        self.lo = start
        self.hi = start

    def advance(self, ids: List[int], num_tokens: int, start0: int) -> bool:
        n, hits, counts = self.ngram, self.min_hits, self.counts
        end = num_tokens - n + 1
        hi = self.hi
        while hi < end:
            key = tuple(ids[hi:hi + n])
            c = counts.get(key, 0) + 1
            counts[key] = c
            if c == hits:
                self.over += 1
            hi += 1
        self.hi = hi
        lo = self.lo
        while lo < start0:
            key = tuple(ids[lo:lo + n])
            c = counts[key]
            if c == hits:
                self.over -= 1
            if c == 1:
                del counts[key]
            else:
                counts[key] = c - 1
            lo += 1
        self.lo = lo
        return self.over > 0
