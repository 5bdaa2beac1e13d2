"""Paged KV block allocator with hash-chained prefix reuse.

Semantics match nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/engine/BlockManager.java:147-266:

* a fixed pool of ``num_blocks`` pages with reference counts, a FIFO free list and a used set;
* prefix reuse only for FULL pages, chained by hash over (previous page hash, page tokens) and confirmed by
  token equality; the last page of a prompt is never taken from the cache (the probe loops to
  ``num_blocks - 1``);
* a cached page that is still in use is shared (refcount + 1) and costs no free page;
* ``may_append`` adds a page when the sequence length modulo the page size is 1 (the newest token opened a
  new page); ``hash_blocks`` publishes pages that the last step completed.

The hash function itself is our own (64-bit BLAKE2b of the previous hash and the little-endian int32
tokens); only its role -- a chain key confirmed by token equality -- has to match the reference.
"""
from __future__ import annotations

import hashlib
from array import array
from collections import OrderedDict
from typing import Dict, List

from .sequence import Sequence


def compute_hash(token_ids: List[int], prefix: int = -1) -> int:
    h = hashlib.blake2b(digest_size=8)
    h.update(int(prefix).to_bytes(8, "little", signed=True))
    h.update(array("i", token_ids).tobytes())
    return int.from_bytes(h.digest(), "little", signed=True)


class Block:
    __slots__ = ("block_id", "ref_count", "hash", "token_ids")

    def __init__(self, block_id: int):
        self.block_id = block_id
        self.ref_count = 0
        self.hash = -1
        self.token_ids: List[int] = []

    def update(self, h: int, token_ids: List[int]) -> None:
        self.hash = h
        self.token_ids = list(token_ids)

    def reset(self) -> None:
        self.ref_count = 1
        self.hash = -1
        self.token_ids = []


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int, prefix_caching: bool = True):
        if num_blocks <= 0:
            raise ValueError("num_blocks must be > 0")
        self.block_size = block_size
        # models with recurrent per-sequence state (LFM2 conv) cannot skip a cached prefix
        self.prefix_caching = prefix_caching
        self.blocks = [Block(i) for i in range(num_blocks)]
        self.hash_to_block_id: Dict[int, int] = {}
        # FIFO free list as an ordered set: pop the oldest, append freed pages, and take a cached page out of
        # the middle in O(1) (a prefix-cache hit on a free page)
        self.free_block_ids: "OrderedDict[int, None]" = OrderedDict.fromkeys(range(num_blocks))
        self.used_block_ids = set()
        # counters for observability
        self.prefix_hit_blocks = 0
        self.prefix_probe_blocks = 0

    @property
    def num_blocks(self) -> int:
        return len(self.blocks)

    @property
    def num_free_blocks(self) -> int:
        return len(self.free_block_ids)

    def utilization(self) -> float:
        return 1.0 - len(self.free_block_ids) / len(self.blocks)

    # ------------------------------------------------------------------ internals
    def _allocate_block(self) -> int:
        if not self.free_block_ids:
            raise RuntimeError("no free KV blocks")
        bid, _ = self.free_block_ids.popitem(last=False)
        block = self.blocks[bid]
        if block.ref_count != 0:
            raise RuntimeError("free block has ref_count != 0")
        if block.hash != -1 and self.hash_to_block_id.get(block.hash) == bid:
            del self.hash_to_block_id[block.hash]
        block.reset()
        self.used_block_ids.add(bid)
        return bid

    def _deallocate_block(self, bid: int) -> None:
        if self.blocks[bid].ref_count != 0:
            raise RuntimeError("cannot free block with refs")
        self.used_block_ids.discard(bid)
        self.free_block_ids[bid] = None

    # ------------------------------------------------------------------ prefill admission
    def can_allocate(self, seq: Sequence) -> int:
        """Cached full-page count, or -1 when the free list cannot cover the remaining pages."""
        h = -1
        cached = 0
        new_blocks = seq.num_blocks
        for i in range(seq.num_blocks - 1 if self.prefix_caching else 0):
            toks = seq.block(i)
            h = compute_hash(toks, h)
            bid = self.hash_to_block_id.get(h, -1)
            if bid == -1 or self.blocks[bid].token_ids != toks:
                break
            cached += 1
            if bid in self.used_block_ids:
                new_blocks -= 1
        if len(self.free_block_ids) < new_blocks:
            return -1
        return cached

    def allocate(self, seq: Sequence, num_cached_blocks: int) -> None:
        if seq.block_table:
            raise RuntimeError("sequence already has a block table")
        h = -1
        for i in range(num_cached_blocks):
            toks = seq.block(i)
            h = compute_hash(toks, h)
            bid = self.hash_to_block_id[h]
            block = self.blocks[bid]
            if bid in self.used_block_ids:
                block.ref_count += 1
            else:
                block.ref_count = 1
                del self.free_block_ids[bid]
                self.used_block_ids.add(bid)
            seq.block_table.append(bid)
        for _ in range(num_cached_blocks, seq.num_blocks):
            seq.block_table.append(self._allocate_block())
        seq.num_cached_tokens = num_cached_blocks * self.block_size
        self.prefix_hit_blocks += num_cached_blocks
        self.prefix_probe_blocks += max(0, seq.num_blocks - 1)

    def deallocate(self, seq: Sequence) -> None:
        for bid in reversed(seq.block_table):
            block = self.blocks[bid]
            block.ref_count -= 1
            if block.ref_count == 0:
                self._deallocate_block(bid)
        seq.num_cached_tokens = 0
        seq.block_table.clear()
        seq.bt_gen += 1

    # ------------------------------------------------------------------ decode growth
    def can_append(self, seq: Sequence) -> bool:
        need = 1 if (len(seq) % self.block_size == 1) else 0
        return len(self.free_block_ids) >= need

    def may_append(self, seq: Sequence) -> None:
        if len(seq) % self.block_size == 1:
            seq.block_table.append(self._allocate_block())

    def hash_blocks(self, seq: Sequence) -> None:
        start = seq.num_cached_tokens // self.block_size
        end = (seq.num_cached_tokens + seq.num_scheduled_tokens) // self.block_size
        if start == end:
            return
        h = self.blocks[seq.block_table[start - 1]].hash if start > 0 else -1
        for i in range(start, end):
            block = self.blocks[seq.block_table[i]]
            toks = seq.block(i)
            h = compute_hash(toks, h)
            block.update(h, toks)
            self.hash_to_block_id[h] = block.block_id

    def clear_prefix_cache(self) -> None:
        self.hash_to_block_id.clear()
        for b in self.blocks:
            if b.ref_count == 0:
                b.hash = -1
                b.token_ids = []
