"""RMSNorm / LayerNorm / rotary tables.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/layers/Norms.java:32-148 (RMSNorm with the
(1+w) Gemma and weightless variants, fused residual add; LayerNorm with bias) and 158-387 (NeoX rotary tables,
the proportional partial-rotary variant, per-model table cache).
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch

from .. import ops

MODE_W, MODE_ONE_PLUS_W, MODE_WEIGHTLESS = 0, 1, 2


class RMSNorm:
    def __init__(self, weight: Optional[torch.Tensor], eps: float, one_plus: bool = False):
        self.weight = weight
        self.eps = eps
        self.mode = MODE_WEIGHTLESS if weight is None else (MODE_ONE_PLUS_W if one_plus else MODE_W)

    def __call__(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None
                 ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        return ops.rms_norm(x, self.weight, self.eps, self.mode, residual)


class LayerNorm:
    def __init__(self, weight: torch.Tensor, bias: torch.Tensor, eps: float):
        self.weight, self.bias, self.eps = weight, bias, eps

    def __call__(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        return ops.layer_norm(x, self.weight, self.bias, self.eps, residual)


class RotaryTables:
    """Per-model cache of cos/sin tables keyed by (head_dim, base, partial factor)."""

    def __init__(self, max_pos: int, device):
        self.max_pos = max_pos
        self.device = device
        self._tables: Dict[tuple, torch.Tensor] = {}

    def get(self, head_dim: int, base: float, partial_factor: float = 1.0) -> torch.Tensor:
        key = (head_dim, float(base), float(partial_factor))
        t = self._tables.get(key)
        if t is None:
            t = ops.ref.rope_cos_sin(head_dim, self.max_pos, base, partial_factor, device=self.device)
            self._tables[key] = t
        return t
