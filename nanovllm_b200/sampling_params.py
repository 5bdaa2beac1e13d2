"""Per-request sampling parameters.

Semantics follow nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/llm/SamplingParams.java:45-110:
temperature must be > 1e-10 ("greedy sampling is not permitted" -- greedy is spelled ``deterministic()``,
which sets top_k=1 and top_p=1 so the sampler takes the argmax), ``max_tokens >= 1``, ``top_k >= 0``
(0 = off) and ``top_p`` in (0, 1].  Defaults are T=0.6, top_p=0.95, top_k=0, max_tokens=256.

New here: ``seed``.  The reference draws from ``ThreadLocalRandom`` (Sampler.java:118); this engine draws
from a counter-based Philox stream keyed by (seed, sequence id, step), so reruns with the same seed and the
same batch composition give bit-identical tokens.
"""
from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Optional

DEFAULT_TEMPERATURE = 0.6
DEFAULT_TOP_P = 0.95
DEFAULT_TOP_K = 0
DEFAULT_MAX_TOKENS = 256


@dataclass(frozen=True)
class SamplingParams:
    temperature: float = DEFAULT_TEMPERATURE
    top_p: float = DEFAULT_TOP_P
    top_k: int = DEFAULT_TOP_K
    max_tokens: int = DEFAULT_MAX_TOKENS
    ignore_eos: bool = False
    seed: Optional[int] = None

    def __post_init__(self):
        if not (self.temperature > 1e-10):
            raise ValueError("temperature must be > 1e-10 (greedy sampling is not permitted; use deterministic())")
        if self.max_tokens < 1:
            raise ValueError("max_tokens must be >= 1")
        if self.top_k < 0:
            raise ValueError("top_k must be >= 0 (0 disables top-k)")
        if not (0.0 < self.top_p <= 1.0):
            raise ValueError("top_p must be in (0, 1]")

    @property
    def is_greedy(self) -> bool:
        return self.top_k == 1

    def deterministic(self) -> "SamplingParams":
        """Argmax decoding: top_k=1, top_p=1 (SamplingParams.java ``deterministic()``)."""
        return replace(self, top_k=1, top_p=1.0)

    def with_(self, **kw) -> "SamplingParams":
        return replace(self, **kw)

    # Builder-style API mirroring the reference's fluent builder.
    class Builder:
        def __init__(self):
            self._kw = {}

        def temperature(self, v: float):
            self._kw["temperature"] = float(v)
            return self

        def top_p(self, v: float):
            self._kw["top_p"] = float(v)
            return self

        def top_k(self, v: int):
            self._kw["top_k"] = int(v)
            return self

        def max_tokens(self, v: int):
            self._kw["max_tokens"] = int(v)
            return self

        def ignore_eos(self, v: bool = True):
            self._kw["ignore_eos"] = bool(v)
            return self

        def seed(self, v: int):
            self._kw["seed"] = int(v)
            return self

        def deterministic(self):
            self._kw["top_k"] = 1
            self._kw["top_p"] = 1.0
            return self

        def build(self) -> "SamplingParams":
            return SamplingParams(**self._kw)

    @staticmethod
    def builder() -> "SamplingParams.Builder":
        return SamplingParams.Builder()

    @staticmethod
    def defaults() -> "SamplingParams":
        return SamplingParams()
