"""Linear layers with real tensor-parallel sharding.

The reference's Linear family (nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/layers/Linear.java:26-405)
binds a kernel per weight type, applies bias and (Gemma4 QAT) input/output SRQ fake-quant; its Column / Row /
Merged / Qkv subclasses are TP names that never shard.  Here:

* ``ColumnParallelLinear`` keeps rows [r*N/TP, (r+1)*N/TP) of W (output features);
* ``MergedColumnParallelLinear`` (gate_up) keeps each rank's gate and up slice and stores them interleaved in
  128-row blocks so the GEMM epilogue computes act(gate) * up on one tile;
* ``QKVParallelLinear`` keeps each rank's q heads and kv heads (kv heads are replicated when nkv < TP);
* ``RowParallelLinear`` keeps columns [r*K/TP, (r+1)*K/TP) of W and all-reduces the partial outputs -- or, on
  the sequence-parallel decode path (``sp_produce``), pushes them to the token-row owners from the GEMM epilogue
  (reduce-scatter); the column-parallel classes' ``sp_consume`` fuses the matching all-gather + RMSNorm into
  their GEMM prologue.

Weights may also be packed (GGUF blocks kept in block format, ``ops.quant.GgufPacked``): they expose
``linear(x, out, partial_ok)`` and the same row / K sharding, concatenation and row permutation as a dense
tensor, so every class here takes either.
"""
from __future__ import annotations

import os
from typing import Optional

import torch

from .. import ops
from ..parallel import state as ps
from ..parallel import symm


from ..ops.quant import cat_rows, is_packed, shard_cols, shard_rows  # dense tensors and GgufPacked alike


class LinearBase:
    weight: torch.Tensor
    bias: Optional[torch.Tensor]

    def __init__(self):
        self.bias = None
        self.act = ops.ACT_NONE

    def _mm(self, x: torch.Tensor, act: int = ops.ACT_NONE) -> torch.Tensor:
        w = self.weight
        if hasattr(w, "linear"):  # packed weight (GGUF blocks): fused dequant path
            y = w.linear(x)
            if act != ops.ACT_NONE:
                y = ops.act_mul(y, act, interleaved=True)
        else:
            y = ops.linear(x, w, act)
        if self.bias is not None:
            ops.bias_act_(y, self.bias, ops.BIAS_ACT_NONE)
        return y


class ColumnSPMixin:
    """Column-parallel projection of an SP forward: all-gather + RMSNorm of the producer's partial rows fused
    into the GEMM prologue (``ops.linear_sp_consume``)."""

    def sp_consume(self, part, norm, has_res: bool, partial_ok: bool = False):
        w = self.weight
        act = self.act if getattr(self, "interleaved", True) else ops.ACT_NONE
        if self.bias is not None or (self.act != ops.ACT_NONE and not getattr(self, "interleaved", True)):
            x = part.ws.ag_norm(part, norm.weight, norm.eps, norm.mode, has_res)
            return self(x)
        return ops.linear_sp_consume(part, norm.weight, norm.eps, norm.mode, has_res, w, act, partial_ok)


class ReplicatedLinear(LinearBase):
    def __init__(self, weight: torch.Tensor, bias: Optional[torch.Tensor] = None):
        super().__init__()
        self.weight, self.bias = weight, bias

    def __call__(self, x):
        return self._mm(x)


class ColumnParallelLinear(ColumnSPMixin, LinearBase):
    def __init__(self, weight: torch.Tensor, bias: Optional[torch.Tensor] = None, shard: bool = True):
        super().__init__()
        r, s = ps.tp_rank(), ps.tp_size()
        self.weight = shard_rows(weight, r, s) if (shard and s > 1) else weight
        self.bias = shard_rows(bias, r, s) if (bias is not None and shard and s > 1) else bias

    def __call__(self, x):
        return self._mm(x)


class MergedColumnParallelLinear(ColumnSPMixin, LinearBase):
    """gate_up: per-rank [gate_r; up_r] interleaved in 128-row blocks; __call__ returns act(gate) * up."""

    def __init__(self, gate: torch.Tensor, up: torch.Tensor, act: int, interleave_block: int = 128):
        super().__init__()
        r, s = ps.tp_rank(), ps.tp_size()
        g = shard_rows(gate, r, s) if s > 1 else gate
        u = shard_rows(up, r, s) if s > 1 else up
        self.act = act
        self.intermediate = g.shape[0]
        gu = cat_rows([g, u])
        if self.intermediate % interleave_block == 0:
            if is_packed(gu):
                order = ops.ref.interleave_gate_up(torch.arange(gu.shape[0]).unsqueeze(1), interleave_block)
                self.weight = gu.permute_rows(order.squeeze(1))
            else:
                self.weight = ops.ref.interleave_gate_up(gu, interleave_block).contiguous()
            self.interleaved = True
        else:
            self.weight = gu.contiguous()
            self.interleaved = False

    def __call__(self, x):
        if self.interleaved and not hasattr(self.weight, "linear"):
            return ops.linear(x, self.weight, self.act)
        y = self._mm(x) if hasattr(self.weight, "linear") else ops.linear(x, self.weight)
        return ops.act_mul(y, self.act, interleaved=self.interleaved)


class QKVParallelLinear(ColumnSPMixin, LinearBase):
    """q/k/v merged; without a bias the decode output may stay split-K (the RoPE kernel sums it)."""
    def __init__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, num_heads: int, num_kv_heads: int,
                 head_dim: int, bq=None, bk=None, bv=None):
        super().__init__()
        r, s = ps.tp_rank(), ps.tp_size()
        assert num_heads % s == 0, "num_heads must be divisible by TP"
        self.nq = num_heads // s
        if num_kv_heads >= s:
            assert num_kv_heads % s == 0
            self.nkv = num_kv_heads // s
            kv_rank = r
            kv_parts = s
        else:  # replicate kv heads: rank r uses kv head r * nkv / s
            self.nkv = 1
            kv_parts = num_kv_heads
            kv_rank = r * num_kv_heads // s
        self.head_dim = head_dim
        qs = shard_rows(q, r, s) if s > 1 else q
        ks = shard_rows(k, kv_rank, kv_parts) if s > 1 else k
        vs = shard_rows(v, kv_rank, kv_parts) if s > 1 else v
        self.weight = cat_rows([qs, ks, vs]).contiguous()
        if bq is not None:
            bqs = shard_rows(bq, r, s) if s > 1 else bq
            bks = shard_rows(bk, kv_rank, kv_parts) if s > 1 else bk
            bvs = shard_rows(bv, kv_rank, kv_parts) if s > 1 else bv
            self.bias = torch.cat([bqs, bks, bvs], 0).contiguous()

    def __call__(self, x):
        if self.bias is None:
            if is_packed(self.weight):
                return self.weight.linear(x, partial_ok=True)
            return ops.linear(x, self.weight, partial_ok=True)
        return self._mm(x)

    def sp_consume(self, part, norm, has_res: bool, partial_ok: bool = True):
        return super().sp_consume(part, norm, has_res, partial_ok=partial_ok and self.bias is None)


class RowParallelLinear(LinearBase):
    def __init__(self, weight: torch.Tensor, bias: Optional[torch.Tensor] = None, reduce: bool = True):
        super().__init__()
        r, s = ps.tp_rank(), ps.tp_size()
        self.weight = shard_cols(weight, r, s).contiguous() if s > 1 else weight
        self.bias = bias  # added once, after the reduction
        self.reduce = reduce

    def __call__(self, x):
        w = self.weight
        packed = is_packed(w)

        def mm(out=None, partial_ok=False):
            if packed:
                return w.linear(x, out=out, partial_ok=partial_ok)
            return ops.linear(x, w, out=out, partial_ok=partial_ok)

        if ps.tp_size() == 1 and self.bias is None:
            return mm(partial_ok=True)  # the following add+RMSNorm sums the split partials
        if self.reduce and self.bias is None and getattr(x, "is_cuda", False):
            ws = symm.workspace()
            T = x.shape[0]
            if ws is not None and ws.fits(T, w.shape[0]):
                # partial sum straight into the symmetric buffer; the consumer fuses all-reduce + norm
                mm(out=ws.in_view(T))
                return ops.TPPartial(ws, T)
        y = ops.materialize(mm())
        if self.reduce:
            ps.all_reduce(y)
        if self.bias is not None:
            ops.bias_act_(y, self.bias, ops.BIAS_ACT_NONE)
        return y

    def sp_produce(self, x, ws):
        """GEMM + reduce-scatter of an SP forward: the partial rows go to their owners (``ops.linear_sp_produce``)."""
        assert self.reduce and self.bias is None, "SP producers are bias-free reducing projections"
        return ops.linear_sp_produce(ws, x, self.weight)
