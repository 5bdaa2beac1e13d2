"""Vocab-parallel embedding and LM head.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/layers/VocabParallelEmbedding.java:32-253.
The embedding gathers rows (optionally scaled, Gemma's sqrt(H)); the LM head scores only the LAST token of each
prefill sequence (cu_seqlens_q[i+1] - 1, VocabParallelEmbedding.java:227-252) and every row in decode.
With TP each rank owns V/TP vocabulary rows: the embedding zeroes ids outside its range and all-reduces (or, on
the sequence-parallel decode path, pushes its rows to their owners: the gather is fused with the reduce-scatter,
``sp_push``); the head computes its logit slice -- with the final all-gather + RMSNorm fused into its GEMM on the
SP path -- and all-gathers the logits so every rank samples the same token.
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import ops
from ..engine.context import get_context
from ..parallel import state as ps


class VocabParallelEmbedding:
    def __init__(self, weight: torch.Tensor, scale: float = 1.0):
        r, s = ps.tp_rank(), ps.tp_size()
        self.vocab = weight.shape[0]
        if s > 1:
            per = (self.vocab + s - 1) // s
            self.vstart = r * per
            self.vend = min(self.vocab, (r + 1) * per)
            self.weight = weight[self.vstart:self.vend].clone()  # a copy: the full table can be freed
        else:
            self.vstart, self.vend, self.weight = 0, self.vocab, weight
        self.scale = scale

    def __call__(self, ids: torch.Tensor) -> torch.Tensor:
        w = self.weight
        if hasattr(w, "embedding"):
            y = w.embedding(ids, self.scale, self.vstart, self.vend)
        else:
            y = ops.embedding(w, ids, self.scale, self.vstart, self.vend)
        return ps.all_reduce(y)

    def sp_push(self, ids: torch.Tensor, ws):
        """Vocab-parallel gather fused with the reduce-scatter into the SP row owners (csrc/tp_sp.cu)."""
        from ..parallel.sp import SPPartial
        w = self.weight
        if not isinstance(w, torch.Tensor):  # packed embedding table: gather, then push
            y = w.embedding(ids, self.scale, self.vstart, self.vend)
            return ws.rs_push(y)
        slot, plan = ws.producer_plan()
        n = ops._cuda_ext().sp_embed_rs(w, ids.long(), float(self.scale), int(self.vstart), int(self.vend), plan)
        ops.add_launches(1)
        return SPPartial(ws, slot, int(n), ws.T)


class ParallelLMHead:
    def __init__(self, weight: torch.Tensor, vocab: Optional[int] = None):
        r, s = ps.tp_rank(), ps.tp_size()
        self.vocab = vocab or weight.shape[0]
        self.sharded = s > 1 and weight.shape[0] == self.vocab
        if self.sharded:
            per = (self.vocab + s - 1) // s
            self.vstart, self.ncols = r * per, max(0, min(self.vocab, (r + 1) * per) - r * per)
            w = weight[r * per:min(self.vocab, (r + 1) * per)]
            if w.shape[0] < per:  # pad the last shard so all_gather sees equal shapes (torch.cat copies)
                w = torch.cat([w, torch.zeros(per - w.shape[0], w.shape[1], dtype=w.dtype, device=w.device)])
            else:
                w = w.clone()  # a row slice is a view of the full head: copy it so the full tensor can be freed
            self.weight = w
        else:
            self.vstart, self.ncols = 0, self.vocab
            self.weight = weight

    def __call__(self, hidden: torch.Tensor, gather_last: bool = True) -> torch.Tensor:
        w = self.weight
        if isinstance(hidden, ops.SPHidden):
            ctx = get_context()
            if gather_last and ctx.is_prefill:
                hidden = hidden.materialize()  # all-gather + final norm, then score only the last tokens
            else:
                # decode: every row is scored; the final all-gather + RMSNorm runs in the LM-head GEMM prologue
                return ops.linear_sp_consume(hidden.part, hidden.norm_w, hidden.eps, hidden.norm_mode, True, w)
        if gather_last:
            ctx = get_context()
            if ctx.is_prefill:
                hidden = ops.gather_rows(hidden, ctx.last_token_idx)
        return w.linear(hidden) if hasattr(w, "linear") else ops.linear(hidden, w)

    # Under TP the head returns this rank's vocabulary slice [T, ceil(V/TP)] (columns past ``ncols`` are padding);
    # the sampler either takes the distributed argmax (greedy rows) or gathers the full logits.
    def gather_full(self, logits: torch.Tensor) -> torch.Tensor:
        """[T, V] logits on every rank from the per-rank slices (NCCL / gloo all-gather)."""
        if not self.sharded:
            return logits
        return ps.all_gather_last(ops.materialize(logits))[:, :self.vocab]

    def argmax(self, logits: torch.Tensor, softcap: float = 0.0) -> torch.Tensor:
        """Greedy tokens [T] (ties to the lowest id) without gathering the logits: each rank reduces its slice and
        only (value, id) pairs are exchanged -- over peer memory with the SP workspace, else an all-gather."""
        logits = ops.materialize(logits)
        from ..parallel import sp
        ws = sp.workspace()
        T = logits.shape[0]
        if self.sharded and logits.is_cuda and ws is not None and T <= sp.MAX_ROWS:
            return ws.argmax(logits, self.ncols, self.vstart, softcap)
        x = logits[:, :self.ncols].float()
        if softcap > 0:
            x = softcap * torch.tanh(x / softcap)
        val, idx = x.max(dim=1)  # first maximum: lowest id on ties
        if not self.sharded:
            return idx
        pair = torch.stack([val.double(), (idx + self.vstart).double()], 1)
        allp = ps.all_gather_last(pair.unsqueeze(1)).view(T, -1, 2)  # [T, R, 2]
        best_v = allp[:, :, 0].max(dim=1, keepdim=True).values
        ids = torch.where(allp[:, :, 0] == best_v, allp[:, :, 1], torch.full_like(allp[:, :, 1], float("inf")))
        return ids.min(dim=1).values.long()
