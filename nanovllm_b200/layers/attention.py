"""Causal paged attention layer (and the bidirectional variant for BERT).

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/layers/Attention.java:49-411 (storeKvCache, dense
vs cached prefill, decode, shared-KV read path) and BidirectionalAttention.java:22-145.  Here one fused kernel
does q/k RMSNorm + RoPE + the KV store, and the attention itself is the paged prefill kernel (which covers both
the dense and the prefix-cached prefill) or the split-KV decode kernel.
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import ops
from ..engine.context import get_context


class Attention:
    def __init__(self, num_heads: int, num_kv_heads: int, head_dim: int, scale: float, rope: torch.Tensor,
                 q_norm: Optional[torch.Tensor] = None, k_norm: Optional[torch.Tensor] = None, norm_mode: int = -1,
                 eps: float = 1e-6, v_norm: bool = False, window: int = 0, softcap: float = 0.0,
                 apply_rope: bool = True, write_kv: bool = True, q_only: bool = False):
        """``q_only``: the input holds only the q heads (a KV-shared layer reading another layer's cache)."""
        self.nq, self.nkv, self.hd = num_heads, num_kv_heads, head_dim
        self.scale = scale
        self.rope = rope
        self.q_norm, self.k_norm, self.norm_mode = q_norm, k_norm, norm_mode
        self.eps = eps
        self.v_norm = v_norm
        self.window = window
        self.softcap = softcap
        self.apply_rope = apply_rope
        self.write_kv = write_kv
        self.q_only = q_only
        self.k_cache: Optional[torch.Tensor] = None
        self.v_cache: Optional[torch.Tensor] = None

    def bind_cache(self, k_cache: torch.Tensor, v_cache: torch.Tensor) -> None:
        self.k_cache, self.v_cache = k_cache, v_cache

    def __call__(self, qkv: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        ctx = get_context()
        T = qkv.shape[0]
        kc = self.k_cache if self.write_kv else None
        vc = self.v_cache if self.write_kv else None
        q = ops.qk_norm_rope_store(qkv, positions, self.rope, self.q_norm, self.k_norm, self.norm_mode, self.v_norm,
                                   self.eps, kc, vc, ctx.slot_mapping if kc is not None else None, self.nq,
                                   0 if self.q_only else self.nkv, self.hd, self.apply_rope)
        if ctx.is_prefill:
            o = ops.prefill_attention(q, ctx.cu_seqlens_q, ctx.cu_seqlens_k, ctx.max_seqlen_q, self.nq, self.nkv,
                                      self.hd, self.scale, self.softcap, self.window, True, self.k_cache,
                                      self.v_cache, ctx.block_tables)
        else:
            o = ops.paged_decode(q, self.k_cache, self.v_cache, ctx.block_tables, ctx.context_lens, self.scale,
                                 self.softcap, self.window, max_len=ctx.max_context_len, scratch=ctx.attn_scratch)
        return o.reshape(T, self.nq * self.hd)


class BidirectionalAttention:
    """Full (non-causal) attention over packed variable-length sequences; K/V read from the qkv tensor."""

    def __init__(self, num_heads: int, head_dim: int, scale: float):
        self.nh, self.hd, self.scale = num_heads, head_dim, scale

    def __call__(self, qkv: torch.Tensor, cu_seqlens: torch.Tensor, max_len: int) -> torch.Tensor:
        H = self.nh * self.hd
        q = qkv[:, :H]
        o = ops.prefill_attention(q, cu_seqlens, cu_seqlens, max_len, self.nh, self.nh, self.hd, self.scale, 0.0, 0,
                                  False, kv_src=qkv)
        return o.reshape(qkv.shape[0], H)
