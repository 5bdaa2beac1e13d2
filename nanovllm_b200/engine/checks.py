"""Debug-mode checks of a step's kernel inputs (``EngineConfig.check_inputs`` or ``NVB_CHECK_INPUTS=1``).

Every address a kernel forms from host data comes from the step staging: token ids index the embedding,
positions the RoPE table, slots the KV arena, block-table entries the KV pages the attention kernels read,
state rows the recurrent-state arena.  ``compute-sanitizer`` is not available on this GPU pool, so instead of a
bounds-checked device build the engine can check these arrays on the host, where they are built, before the
kernels see them:

* ranges: ids in [0, vocab), positions in [0, max_model_len], slots -1 or inside the arena, block-table entries
  (up to each row's context) inside the pool, context lengths covered by the row's pages, state rows inside the
  arena;
* consistency: a token's slot lies in the page its block table names for its position;
* races: no slot is written twice in one step, and no page written in this step appears in another sequence's
  block table (a shared prefix page must never be written -- copy-on-write is violated otherwise).

A violation raises ``StepInputError`` naming the row and the value.  The reference is a single JVM process
whose arrays are bounds-checked by the runtime (nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/engine/
Transformer.java:342-457 builds the same step arrays); this module stands in for that safety net.
"""
from __future__ import annotations

from typing import Optional, Sequence

import numpy as np

from ..exceptions import StepInputError


def _bad(name: str, arr: np.ndarray, mask: np.ndarray) -> None:
    if mask.any():
        i = int(np.flatnonzero(mask)[0])
        raise StepInputError(f"{name}[{i}] = {int(arr.reshape(-1)[i])} is out of range")


def check_step(*, ids: np.ndarray, pos: np.ndarray, slots: np.ndarray, block_tables: np.ndarray,
               context_lens: np.ndarray, seq_of_token: np.ndarray, vocab: int, max_pos: int, num_blocks: int,
               block_size: int, state_rows: Optional[np.ndarray] = None, state_capacity: int = 0) -> None:
    """``block_tables`` [S, W] with the rows of the step's sequences, ``context_lens`` [S] (tokens cached after
    this step), ``seq_of_token`` [T] the batch row of every token of ``ids`` / ``pos`` / ``slots``."""
    _bad("token id", ids, (ids < 0) | (ids >= vocab))
    _bad("position", pos, (pos < 0) | (pos > max_pos))
    _bad("slot", slots, (slots < -1) | (slots >= num_blocks * block_size))
    S = context_lens.shape[0]
    need = (context_lens + block_size - 1) // block_size
    if need.size and int(need.max()) > block_tables.shape[1]:
        r = int(np.argmax(need))
        raise StepInputError(f"sequence row {r}: context {int(context_lens[r])} needs {int(need[r])} pages, the block "
                             f"table has {block_tables.shape[1]}")
    cols = np.arange(block_tables.shape[1])[None, :]
    used = cols < need[:, None]
    _bad("block-table entry", block_tables, used & ((block_tables < 0) | (block_tables >= num_blocks)))
    live = slots >= 0
    if live.any():
        t = np.flatnonzero(live)
        rows, p, sl = seq_of_token[t], pos[t], slots[t]
        want = block_tables[rows, p // block_size] * block_size + p % block_size
        wrong = want != sl
        if wrong.any():
            k = int(np.flatnonzero(wrong)[0])
            raise StepInputError(f"token {int(t[k])} (row {int(rows[k])}, position {int(p[k])}): slot {int(sl[k])} is "
                                 f"not the block table's slot {int(want[k])}")
        uniq, counts = np.unique(sl, return_counts=True)
        if (counts > 1).any():
            raise StepInputError(f"slot {int(uniq[np.argmax(counts > 1)])} is written by more than one token in one step")
        # pages written this step must not be readable through another sequence's table
        written = np.unique(sl // block_size)
        for r in range(S):
            mine = set(block_tables[r, :need[r]].tolist())
            own = set(np.unique(sl[rows == r] // block_size).tolist())
            shared = (set(written.tolist()) - own) & mine
            if shared:
                raise StepInputError(f"sequence row {r} reads page {min(shared)} that another sequence writes in this "
                                     f"step (shared page written: copy-on-write violated)")
    if state_rows is not None:
        _bad("state row", state_rows, (state_rows < 0) | (state_rows >= state_capacity))
