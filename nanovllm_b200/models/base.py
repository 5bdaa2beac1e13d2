"""Shared pieces of the model graphs: the causal-LM interface, weight access helpers and random init.

Interface mirrors nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/internal/CausalLM.java:12-21
(``forward(ids, positions)`` -> hidden states, ``compute_logits(hidden)``) and EmbeddingEncoder.java:10-17.
``kv_specs`` tells the model runner which layers own a paged KV cache and with which (kv heads, head dim);
``bind_kv`` hands each attention layer its cache views.
"""
from __future__ import annotations

import contextlib
import contextvars
import math
from typing import Callable, Dict, Iterable, List, Optional, Tuple

import torch

from ..config import HfConfig
from ..exceptions import ModelLoadException

# set while an engine that unpacks its parameters builds its model graph: packed sources (GGUF blocks, QAT
# integer weights) are expanded to dense bf16 instead of taking the dequant-fused GEMM
_UNPACK = contextvars.ContextVar("nvb_unpack_parameters", default=False)


@contextlib.contextmanager
def unpacked_parameters(on: bool = True):
    token = _UNPACK.set(bool(on))
    try:
        yield
    finally:
        _UNPACK.reset(token)


def unpacking() -> bool:
    return _UNPACK.get()


class WeightBag:
    """Name -> tensor (or packed weight) map with required / optional access (WeightBag.java:15-179)."""

    def __init__(self, tensors: Dict[str, object], device, dtype=torch.bfloat16):
        self.tensors = tensors
        self.device = device
        self.dtype = dtype
        self.used = set()

    def _prep(self, t):
        if isinstance(t, torch.Tensor):
            if t.is_floating_point():
                t = t.to(device=self.device, dtype=self.dtype)
            else:
                t = t.to(self.device)
            return t.contiguous()
        if hasattr(t, "to_device"):
            return t.to_device(self.device)
        return t

    def has(self, name: str) -> bool:
        return name in self.tensors

    def require(self, name: str):
        if name not in self.tensors:
            raise ModelLoadException(f"missing weight: {name}")
        self.used.add(name)
        return self._prep(self.tensors[name])

    def find(self, name: str):
        if name not in self.tensors:
            return None
        return self.require(name)

    def dense(self, name: str) -> torch.Tensor:
        """Dense bf16 tensor even when the source is packed (for norms, embeddings on CPU, tests)."""
        t = self.require(name)
        if not isinstance(t, torch.Tensor) and hasattr(t, "dequantize"):
            return t.dequantize(self.dtype)
        return t

    def release(self, name: str) -> None:
        self.tensors.pop(name, None)


class CausalLMBase:
    hf: HfConfig
    final_softcap: float = 0.0

    def kv_specs(self) -> List[Tuple[int, int, int]]:
        """[(layer_idx, kv_heads_local, head_dim)] for layers that own a KV cache."""
        raise NotImplementedError

    def bind_kv(self, caches: Dict[int, Tuple[torch.Tensor, torch.Tensor]]) -> None:
        raise NotImplementedError

    def forward(self, ids: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    def compute_logits(self, hidden: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    # recurrent state (LFM2) hooks
    def state_specs(self) -> List[Tuple[int, int]]:
        return []

    def bind_state(self, arena: Optional[torch.Tensor]) -> None:
        pass


def _normal(shape, gen: torch.Generator, std: float, device) -> torch.Tensor:
    t = torch.empty(shape, dtype=torch.float32, device=device)
    t.normal_(0.0, std, generator=gen)
    return t.to(torch.bfloat16)


def random_weights(names_shapes: Iterable[Tuple[str, tuple]], seed: int, device="cpu", std: float = 0.02,
                   ones_for: Callable[[str], bool] = None, zeros_for: Callable[[str], bool] = None
                   ) -> Dict[str, torch.Tensor]:
    """Seeded N(0, std) weights; norm weights set to 1 (or 0 for (1+w) norms via ``zeros_for``)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    out = {}
    for name, shape in names_shapes:
        if zeros_for is not None and zeros_for(name):
            out[name] = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        elif ones_for is not None and ones_for(name):
            out[name] = torch.ones(shape, dtype=torch.bfloat16, device=device)
        else:
            out[name] = _normal(shape, gen, std, device)
    return out


def is_norm_name(name: str) -> bool:
    return "norm" in name.split(".")[-2] if name.count(".") >= 1 else False
