"""Architecture dispatch: config -> model class, random-init schema and the embedding/causal split.

Mirrors the reference's processors (nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/llmarch/
ArchitectureProcessors.java:31-42 and CausalLMFactory.java:17-31): the model family is chosen from
``model_type`` / ``architectures`` after ModelSupport has accepted the checkpoint.
"""
from __future__ import annotations

from typing import Callable, Dict, Tuple

import torch

from ..config import HfConfig
from ..exceptions import UnsupportedModelException


def causal_model_class(hf: HfConfig):
    mt = (hf.model_type or "").lower()
    if mt == "qwen3":
        from .qwen3 import Qwen3ForCausalLM
        return Qwen3ForCausalLM
    if mt == "llama":
        from .qwen3 import LlamaForCausalLM
        return LlamaForCausalLM
    if mt in ("gemma3", "gemma3_text"):
        from .gemma3 import Gemma3ForCausalLM
        return Gemma3ForCausalLM
    if mt in ("gemma4", "gemma4_text"):
        from .gemma4 import Gemma4ForCausalLM
        return Gemma4ForCausalLM
    if mt in ("lfm2",):
        from .lfm2 import Lfm2ForCausalLM
        return Lfm2ForCausalLM
    raise UnsupportedModelException(f"no causal model for model_type={hf.model_type!r}")


def init_random_weights(hf: HfConfig, seed: int, device="cpu") -> Dict[str, torch.Tensor]:
    mt = (hf.model_type or "").lower()
    if mt == "qwen3":
        from .qwen3 import init_random
        return init_random(hf, seed, device, qk_norm=True)
    if mt == "llama":
        from .qwen3 import init_random
        return init_random(hf, seed, device, qk_norm=False)
    if mt in ("gemma3", "gemma3_text"):
        from .gemma3 import init_random
        return init_random(hf, seed, device)
    if mt in ("gemma4", "gemma4_text"):
        from .gemma4 import init_random
        return init_random(hf, seed, device)
    if mt == "lfm2":
        from .lfm2 import init_random
        return init_random(hf, seed, device)
    if mt == "bert":
        from .bert import init_random
        return init_random(hf, seed, device)
    raise UnsupportedModelException(f"no random init for model_type={hf.model_type!r}")
