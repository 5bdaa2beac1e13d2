"""Continuous-batching scheduler: prefill first, chunked prefill under a token budget, LIFO preemption.

Policy follows nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/engine/Scheduler.java:178-412:

* ``schedule`` returns a prefill batch whenever the waiting head can be admitted, else a decode batch;
* prefill admission is capped by ``max_num_seqs`` and ``max_num_batched_tokens``; the FIRST sequence of a
  batch may be chunked to the remaining budget, and a partially prefilled sequence stays at the waiting head
  until its prompt is fully cached (Scheduler.java:191-256);
* decode takes running sequences from the head; when a page cannot be appended it preempts the running
  TAIL (or the sequence itself when it is alone): status back to WAITING, pages freed, pushed to the waiting
  HEAD and recomputed from scratch (Scheduler.java:262-327); an empty decode batch is an error;
* postprocess hashes the finished pages, advances the cached counter, returns early for mid-prompt chunks
  (their sampled token is discarded) and otherwise appends the token and checks the stop rules: stop id
  (unless ignore_eos), ``max_tokens``, ``max_model_len`` and the degenerate-repetition detector
  (Scheduler.java:370-403).

``on_release`` is called whenever a sequence gives up its pages (finish, preempt, clear) so the model runner
can free per-sequence recurrent state (LFM2 conv state), as Scheduler.java:92-103 does.
"""
from __future__ import annotations

import itertools
from collections import deque
from typing import Callable, List, Optional, Sequence as Seq, Tuple

from ..config import EngineConfig
from .block_manager import BlockManager
from .sequence import Sequence, SequenceStatus


class Scheduler:
    def __init__(self, cfg: EngineConfig, num_blocks: int, stop_token_ids: Seq[int] = (),
                 on_release: Optional[Callable[[Sequence], None]] = None, max_live_seqs: Optional[int] = None):
        self.max_num_seqs = cfg.max_num_seqs
        # models with per-sequence recurrent state (LFM2) hold one state row per live sequence: no new sequence
        # is admitted while ``max_live_seqs`` are running or part-way through prefill
        self.max_live_seqs = max_live_seqs
        self.max_num_batched_tokens = cfg.max_num_batched_tokens
        self.max_model_len = cfg.max_model_len
        self.block_size = cfg.kvcache_block_size
        self.stop_on_degenerate = cfg.stop_on_degenerate
        ids = list(stop_token_ids) if stop_token_ids else ([cfg.eos] if cfg.eos >= 0 else [])
        self.stop_token_ids = frozenset(int(x) for x in ids)
        self.block_manager = BlockManager(num_blocks, cfg.kvcache_block_size, cfg.enable_prefix_caching)
        self.waiting: deque = deque()
        self.running: deque = deque()
        self.on_release = on_release
        self.num_preemptions = 0
        self.decode_fast_path = True  # one-pass decode batch when no page is short (tests compare both forms)

    def is_finished(self) -> bool:
        return not self.waiting and not self.running

    def add(self, seq: Sequence) -> None:
        if len(seq) >= self.max_model_len:
            raise ValueError(f"prompt of {len(seq)} tokens does not fit max_model_len={self.max_model_len}")
        self.waiting.append(seq)

    def abort(self, seq_id: int) -> bool:
        for q in (self.waiting, self.running):
            for s in list(q):
                if s.seq_id == seq_id:
                    q.remove(s)
                    s.status = SequenceStatus.FINISHED
                    self._release(s)
                    return True
        return False

    def clear(self) -> None:
        for q in (self.running, self.waiting):
            while q:
                s = q.popleft()
                s.status = SequenceStatus.FINISHED
                self._release(s)

    def _release(self, seq: Sequence) -> None:
        if seq.block_table:
            self.block_manager.deallocate(seq)
        seq.num_scheduled_tokens = 0
        if self.on_release is not None:
            self.on_release(seq)

    def _live(self) -> int:
        return len(self.running) + sum(1 for s in self.waiting if s.block_table)

    # ------------------------------------------------------------------ scheduling
    def schedule(self) -> Tuple[List[Sequence], bool]:
        batch = self._try_schedule_prefill()
        if batch:
            return batch, True
        return self._schedule_decode(), False

    def _try_schedule_prefill(self) -> List[Sequence]:
        scheduled: List[Sequence] = []
        batched = 0
        bm = self.block_manager
        while self.waiting and len(scheduled) < self.max_num_seqs:
            seq = self.waiting[0]
            remaining = self.max_num_batched_tokens - batched
            if remaining == 0:
                break
            if not seq.block_table:
                if self.max_live_seqs is not None and self._live() >= self.max_live_seqs:
                    break
                cached_blocks = bm.can_allocate(seq)
                if cached_blocks == -1:
                    break
                tokens = len(seq) - cached_blocks * self.block_size
                needs_alloc = True
            else:
                cached_blocks = 0
                tokens = len(seq) - seq.num_cached_tokens
                needs_alloc = False
            if remaining < tokens and scheduled:
                break
            if needs_alloc:
                bm.allocate(seq, cached_blocks)
            seq.num_scheduled_tokens = min(tokens, remaining)
            seq.is_prefill = True
            batched += seq.num_scheduled_tokens
            if seq.num_cached_tokens + seq.num_scheduled_tokens == len(seq):
                seq.status = SequenceStatus.RUNNING
                self.waiting.popleft()
                self.running.append(seq)
            scheduled.append(seq)
        return scheduled

    def _schedule_decode(self) -> List[Sequence]:
        scheduled: List[Sequence] = []
        bm = self.block_manager
        # common case: the free pages cover every sequence that opens a new page this step, so nobody is
        # preempted and the batch is the running head in order (what the loop below produces, without the churn)
        head = list(itertools.islice(self.running, self.max_num_seqs)) if self.decode_fast_path else []
        bs = self.block_size
        opening = sum(1 for s in head if s.num_tokens % bs == 1)
        if head and opening <= bm.num_free_blocks:
            for s in head:
                s.num_scheduled_tokens = 1
                s.is_prefill = False
                bm.may_append(s)
            return head
        while self.running and len(scheduled) < self.max_num_seqs:
            seq = self.running.popleft()
            ok = True
            while not bm.can_append(seq):
                if not self.running:
                    self.preempt(seq)
                    ok = False
                    break
                self.preempt(self.running.pop())
            if not ok:
                break
            seq.num_scheduled_tokens = 1
            seq.is_prefill = False
            bm.may_append(seq)
            scheduled.append(seq)
        if not scheduled:
            raise RuntimeError("scheduler produced an empty decode batch")
        for s in reversed(scheduled):
            self.running.appendleft(s)
        return scheduled

    def preempt(self, seq: Sequence) -> None:
        seq.status = SequenceStatus.WAITING
        seq.is_prefill = True
        self._release(seq)
        self.waiting.appendleft(seq)
        self.num_preemptions += 1

    # ------------------------------------------------------------------ postprocess
    def postprocess(self, seqs: List[Sequence], token_ids: List[int], is_prefill: bool,
                    appended_out: Optional[list] = None) -> List[Sequence]:
        finished = []
        bm = self.block_manager
        for seq, tok in zip(seqs, token_ids):
            bm.hash_blocks(seq)
            seq.num_cached_tokens += seq.num_scheduled_tokens
            seq.num_scheduled_tokens = 0
            if is_prefill and seq.num_cached_tokens < len(seq):
                continue
            seq.append_token(tok)
            if appended_out is not None:
                appended_out.append((seq.seq_id, int(tok)))
            if self._should_finish(seq, tok):
                seq.status = SequenceStatus.FINISHED
                self._release(seq)
                try:
                    self.running.remove(seq)
                except ValueError:
                    pass
                finished.append(seq)
        return finished

    def _should_finish(self, seq: Sequence, tok: int) -> bool:
        return ((not seq.ignore_eos and tok in self.stop_token_ids)
                or seq.num_completion_tokens == seq.max_tokens
                or len(seq) >= self.max_model_len
                or (self.stop_on_degenerate and seq.has_degenerate_repetition()))
