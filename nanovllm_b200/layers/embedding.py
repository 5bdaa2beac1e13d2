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

    # rows whose top_k is at most this sample from exchanged candidates instead of gathered logits
    CANDIDATE_K = 64

    def sample_candidates(self, logits: torch.Tensor, temps, top_ks, top_ps, seeds, seq_ids, steps, kmax: int,
                          softcap: float = 0.0) -> torch.Tensor:
        """Seeded sampling of rows with 1 <= top_k <= kmax <= CANDIDATE_K without gathering the logits.  The
        global top-k set lies inside the union of the ranks' own top-k (value descending, id ascending), and the
        sampler's masses, cut-offs and Philox draws depend only on the kept tokens' values and ids, so each rank
        exchanges kmax (value, id) pairs per row and every rank runs the same sampler over the id-sorted union:
        the tokens equal the single-GPU sampler's (Sampler.java:69-134 semantics)."""
        logits = ops.materialize(logits)
        x = logits[:, :self.ncols]
        K = max(1, min(int(kmax), self.ncols))
        # exact order: 64-bit keys from the order-preserving float bits, then the inverted local index
        b = x.float().contiguous().view(torch.int32)
        okey = torch.where(b < 0, b ^ 0x7FFFFFFF, b).to(torch.int64)
        idx = torch.arange(x.shape[1], device=x.device, dtype=torch.int64)
        key = (okey << 32) | (0xFFFFFFFF - idx)
        top = torch.topk(key, K, dim=1, sorted=False).indices
        vals = x.gather(1, top).float()
        gids = (top + self.vstart).to(torch.int32)
        allv = ps.all_gather_last(vals)
        allg = ps.all_gather_last(gids)
        order = torch.argsort(allg, dim=1)
        allg = allg.gather(1, order)
        allv = allv.gather(1, order)
        C = allg.shape[1]
        Cp = (C + 7) // 8 * 8  # the sampler streams 8 bf16 per load
        if Cp != C:
            allv = torch.cat([allv, torch.full((allv.shape[0], Cp - C), float("-inf"), device=allv.device)], 1)
            allg = torch.cat([allg, torch.full((allg.shape[0], Cp - C), self.vocab, dtype=torch.int32,
                                               device=allg.device)], 1)
        return ops.sample(allv.to(torch.bfloat16).contiguous(), temps, top_ks, top_ps, seeds, seq_ids, steps,
                          softcap=softcap, ids=allg.contiguous())

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
