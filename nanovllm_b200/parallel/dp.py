"""Data-parallel sentence embeddings: one BERT replica per GPU (process), the batch split across ranks.

The reference encodes one text at a time on a sequential matmul runtime and shares one ``LlmModel`` between
engines as its only form of data parallelism (nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/
internal/LlmModelImpl.java:292-351, BertForEmbedding.java:127-157).  Here every rank holds a full replica of the
(small) encoder; ``DataParallelEmbedder.embed_ids`` deals the sequences out by length so every rank gets about the
same number of tokens, each rank encodes its share as packed varlen batches, and one all-gather of the [n, H]
results (padded to the largest share) returns every embedding, in input order, on every rank.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

import torch
import torch.distributed as dist

from . import state as ps


def deal_by_tokens(lengths: Sequence[int], ranks: int) -> List[List[int]]:
    """Indices per rank: longest sequences first, each to the rank with the fewest tokens so far (ties: lower
    rank), so token counts differ by at most one sequence length; every rank's list is in input order."""
    load = [0] * ranks
    out: List[List[int]] = [[] for _ in range(ranks)]
    for i in sorted(range(len(lengths)), key=lambda k: (-lengths[k], k)):
        r = min(range(ranks), key=lambda q: (load[q], q))
        out[r].append(i)
        load[r] += lengths[i]
    return [sorted(o) for o in out]


class DataParallelEmbedder:
    """``encoder``: this rank's replica (``BertEncoder`` or anything with ``embed_ids(batch, keep_device=True)``)."""

    def __init__(self, encoder, max_tokens: int = 65536):
        self.encoder = encoder
        self.max_tokens = int(max_tokens)

    def shard(self, batch: Sequence[Sequence[int]]) -> Tuple[List[int], List[List[int]]]:
        """(this rank's input indices, the per-rank index lists)."""
        plan = deal_by_tokens([len(s) for s in batch], ps.tp_size())
        return plan[ps.tp_rank()], plan

    @torch.inference_mode()
    def embed_ids(self, batch: Sequence[Sequence[int]]) -> torch.Tensor:
        """[N, H] fp32 embeddings of ``batch`` on every rank (on the encoder's device), in input order."""
        R = ps.tp_size()
        mine, plan = self.shard(batch)
        local = self.encoder.embed_ids([list(batch[i]) for i in mine], max_tokens=self.max_tokens, keep_device=True) \
            if mine else None
        if R == 1:
            return local
        dev = local.device if local is not None else getattr(self.encoder, "device", torch.device("cpu"))
        H = self.encoder.hf.hidden_size
        width = max(len(p) for p in plan)
        buf = torch.zeros(width, H, dtype=torch.float32, device=dev)
        if local is not None:
            buf[:local.shape[0]] = local
        parts = [torch.empty_like(buf) for _ in range(R)]
        dist.all_gather(parts, buf, group=ps.tp_group())
        out = torch.empty(len(batch), H, dtype=torch.float32, device=dev)
        for r in range(R):
            if plan[r]:
                out[torch.tensor(plan[r], device=dev)] = parts[r][:len(plan[r])]
        return out
