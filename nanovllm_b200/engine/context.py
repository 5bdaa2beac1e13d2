"""Per-step metadata handed to the model (flash-attn varlen style).

Same fields as the reference's step Context (nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/internal/
Context.java:12-122): prefill flag, cu_seqlens_q/k, max seqlens, slot mapping, context lengths, block tables and
sequence ids -- here as device tensors, plus the index of each sequence's last token for the LM head and the
rows of the recurrent-state arena (LFM2).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import torch


@dataclass
class StepContext:
    is_prefill: bool
    num_seqs: int
    num_tokens: int
    slot_mapping: Optional[torch.Tensor] = None      # int32 [T]
    block_tables: Optional[torch.Tensor] = None      # int32 [S, max_blocks]
    cu_seqlens_q: Optional[torch.Tensor] = None      # int32 [S+1] (prefill)
    cu_seqlens_k: Optional[torch.Tensor] = None      # int32 [S+1] (prefill)
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    context_lens: Optional[torch.Tensor] = None      # int32 [S] (decode)
    max_context_len: int = 0                          # decode grid sizing (static under CUDA graphs)
    last_token_idx: Optional[torch.Tensor] = None    # int64 [S]
    state_rows: Optional[torch.Tensor] = None        # int64 [S] rows of the conv-state arena
    state_fresh: Optional[torch.Tensor] = None       # bool [S]: sequence starts from an empty recurrent state
    seq_token_counts: List[int] = field(default_factory=list)  # prefill: scheduled tokens per sequence (host)
    attn_scratch: Optional[torch.Tensor] = None      # fp32 split-KV partials


_CTX: Optional[StepContext] = None


def set_context(ctx: Optional[StepContext]) -> None:
    global _CTX
    _CTX = ctx


def get_context() -> StepContext:
    if _CTX is None:
        raise RuntimeError("no step context set")
    return _CTX
