"""Step-plan broadcast: tensor-parallel serving with a single front door on rank 0.

The reference runs one engine in one JVM (nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/llm/LLM.java:
774-928, the generate loop around ``Transformer.step``), so it has no cross-process plan.  Under TP this engine
offers two ways to keep the ranks in lock-step:

* SPMD (default): every rank receives the same requests in the same order and runs its own scheduler; the
  sampler is deterministic, so the schedulers agree without any per-step message;
* front door (``EngineConfig.front_door = "rank0"``): only rank 0 takes requests and schedules.  Before each
  step it broadcasts the step plan over a Gloo control group; the other ranks (``LLM.serve_worker``) keep a
  mirror of every scheduled sequence, apply the plan to it and run the same forward, collectives and sampler.

A plan carries only what changed since the previous one: per scheduled sequence its counters, the tokens
appended since the last plan that named it (the whole prompt the first time, then one sampled token per decode
step), the block-table entries appended (or the whole table after the table was released and reallocated) and
its sampling knobs; plus the sequences released since the last plan (finished ones are dropped, preempted ones
keep their tokens and lose their pages).  Each worker compares the token it sampled in a step with the token
rank 0 appended for it, so a rank that diverged is reported instead of silently generating other text.

Wire format: one int64 array, ``[kind, is_prefill, n_seqs, n_released, n_tok, n_blk] + released (seq id, drop)
pairs + per sequence REC ints + per sequence (temperature, top_p) as float64 bits + appended tokens + appended
blocks``; it is sent as a length broadcast followed by the array.  Workers wait with ``async_op`` and poll the
abort flag, so a failed rank 0 (which publishes its abort reason) ends an idle worker at once instead of after
the control group's timeout.
"""
from __future__ import annotations

import time
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch
import torch.distributed as dist

from ..exceptions import TensorParallelAbort
from ..parallel import state as ps
from .sequence import Sequence, SequenceStatus

KIND_STEP, KIND_SHUTDOWN = 1, 2
HEADER = 6
# per-sequence record: seq id, tokens after the plan, prompt length, cached tokens, scheduled tokens, index of
# the first appended token, index of the first appended block, blocks after the plan, block-table generation,
# top_k, seed (-1: none)
REC = 11


def _poll(work, what: str) -> None:
    """Wait for an async collective while watching the TP abort flag (an idle server waits indefinitely)."""
    spins = 0
    while not work.is_completed():
        if ps.abort_requested():
            raise TensorParallelAbort(ps.abort_reason() or f"a peer rank aborted while this rank waited for {what}")
        spins += 1
        if spins > 2000:
            time.sleep(0.0002)
    work.wait()


class PlanSender:
    """Rank 0 side: encodes each step's plan from the scheduler's batch and broadcasts it."""

    def __init__(self, group):
        self.group = group
        self.synced: Dict[int, List[int]] = {}   # seq id -> [tokens sent, block-table generation, blocks sent]
        self.released: List[Tuple[int, int]] = []

    def note_release(self, seq: Sequence) -> None:
        """Called whenever the scheduler releases a sequence's pages (finish, abort, clear, preemption)."""
        drop = 1 if seq.status == SequenceStatus.FINISHED else 0
        self.released.append((seq.seq_id, drop))
        if drop:
            self.synced.pop(seq.seq_id, None)

    def encode(self, seqs: List[Sequence], is_prefill: bool) -> np.ndarray:
        ints: List[int] = []
        floats: List[float] = []
        toks: List[int] = []
        blks: List[int] = []
        for s in seqs:
            st = self.synced.get(s.seq_id)
            if st is None:
                st = self.synced[s.seq_id] = [0, -1, 0]
            t0 = st[0]
            toks.extend(s.token_ids[t0:s.num_tokens])
            nb = len(s.block_table)
            b0 = st[2] if (st[1] == s.bt_gen and st[2] <= nb) else 0
            blks.extend(s.block_table[b0:])
            ints += [s.seq_id, s.num_tokens, s.num_prompt_tokens, s.num_cached_tokens, s.num_scheduled_tokens, t0, b0,
                     nb, s.bt_gen, s.top_k, -1 if s.seed is None else int(s.seed) & 0x7FFFFFFFFFFFFFFF]
            floats += [s.temperature, s.top_p]
            st[0], st[1], st[2] = s.num_tokens, s.bt_gen, nb
        rel = [x for pair in self.released for x in pair]
        head = [KIND_STEP, int(is_prefill), len(seqs), len(self.released), len(toks), len(blks)]
        self.released = []
        return np.concatenate([np.asarray(head + rel + ints, dtype=np.int64),
                               np.asarray(floats, dtype=np.float64).view(np.int64),
                               np.asarray(toks, dtype=np.int64), np.asarray(blks, dtype=np.int64)])

    def send(self, plan: np.ndarray) -> None:
        n = torch.tensor([plan.size], dtype=torch.int64)
        dist.broadcast(n, src=0, group=self.group)
        dist.broadcast(torch.from_numpy(plan), src=0, group=self.group)

    def send_step(self, seqs: List[Sequence], is_prefill: bool) -> None:
        self.send(self.encode(seqs, is_prefill))

    def send_shutdown(self) -> None:
        rel = [x for pair in self.released for x in pair]
        self.released = []
        self.send(np.asarray([KIND_SHUTDOWN, 0, 0, len(rel) // 2, 0, 0] + rel, dtype=np.int64))


class PlanReceiver:
    """Worker side: receives plans and keeps the mirrored sequences they describe."""

    def __init__(self, group, block_size: int, release=None):
        self.group = group
        self.block_size = block_size
        self.release = release                # runner hook: free per-sequence state of a released sequence
        self.mirrors: Dict[int, Sequence] = {}
        self.expect: Dict[int, int] = {}      # seq id -> token this rank sampled in the last step that produced one

    def recv(self) -> np.ndarray:
        n = torch.zeros(1, dtype=torch.int64)
        _poll(dist.broadcast(n, src=0, group=self.group, async_op=True), "the next step plan")
        buf = torch.empty(int(n[0]), dtype=torch.int64)
        _poll(dist.broadcast(buf, src=0, group=self.group, async_op=True), "the next step plan")
        return buf.numpy()

    def apply(self, plan: np.ndarray) -> Tuple[int, bool, List[Sequence]]:
        """Apply a plan to the mirrors; returns (kind, is_prefill, scheduled mirrors in batch order)."""
        kind, is_prefill, n, n_rel, n_tok, n_blk = (int(x) for x in plan[:HEADER])
        o = HEADER
        for i in range(n_rel):
            sid, drop = int(plan[o + 2 * i]), int(plan[o + 2 * i + 1])
            m = self.mirrors.get(sid)
            if m is None:
                continue
            if self.release is not None:
                self.release(m)
            m.block_table = []
            m.num_cached_tokens = 0
            if drop:
                del self.mirrors[sid]
                self.expect.pop(sid, None)
        o += 2 * n_rel
        recs = plan[o:o + REC * n].reshape(n, REC).tolist()
        o += REC * n
        fl = plan[o:o + 2 * n].view(np.float64).reshape(n, 2).tolist()
        o += 2 * n
        toks = plan[o:o + n_tok].tolist()
        o += n_tok
        blks = plan[o:o + n_blk].tolist()
        seqs: List[Sequence] = []
        tp = bp = 0
        for (sid, ntok, nprompt, ncached, nsched, t0, b0, nb, gen, top_k, seed), (temp, top_p) in zip(recs, fl):
            new_toks = toks[tp:tp + ntok - t0]
            tp += ntok - t0
            m = self.mirrors.get(sid)
            if m is None:
                if t0 != 0:
                    raise TensorParallelAbort(f"step plan names sequence {sid} that this rank never saw")
                m = self.mirrors[sid] = Sequence.mirror(sid, new_toks, nprompt, self.block_size)
            else:
                if t0 != m.num_tokens:
                    raise TensorParallelAbort(f"step plan for sequence {sid} starts at token {t0}, this rank holds "
                                              f"{m.num_tokens}")
                if new_toks:
                    want = self.expect.pop(sid, None)
                    if want is not None and want != new_toks[0]:
                        raise TensorParallelAbort(f"ranks diverged: sequence {sid} sampled {want} here, "
                                                  f"{new_toks[0]} on rank 0")
                    m.token_ids.extend(new_toks)
                    m.num_tokens = len(m.token_ids)
                    m.last_token = m.token_ids[-1]
            new_blks = blks[bp:bp + nb - b0]
            bp += nb - b0
            if b0 == 0:
                m.block_table = new_blks
            else:
                m.block_table.extend(new_blks)
            m.bt_gen = gen
            m.num_cached_tokens = ncached
            m.num_scheduled_tokens = nsched
            m.is_prefill = bool(is_prefill)
            m.top_k, m.seed = top_k, (None if seed < 0 else seed)
            m.temperature, m.top_p = temp, top_p
            seqs.append(m)
        return kind, bool(is_prefill), seqs

    def note_sampled(self, seqs: List[Sequence], toks: List[int]) -> None:
        """Remember the tokens of this step that rank 0 will append (the others are mid-prompt chunks)."""
        for s, t in zip(seqs, toks):
            if s.num_cached_tokens + s.num_scheduled_tokens >= s.num_tokens:
                self.expect[s.seq_id] = int(t)
