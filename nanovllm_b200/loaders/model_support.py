"""Which checkpoints this library accepts (exact architecture detection + container rules).

Behaviour follows nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/ModelSupport.java:34-566:
chat models from a Hugging Face folder are qwen3, gemma3 / gemma3_text, gemma4 (text / QAT) and llama; chat
from GGUF is qwen3 and lfm2; embeddings (bert) come from GGUF or ONNX.  Look-alike families are rejected with
the catalogue in the message (Qwen2 / 2.5, Qwen3.5 / Next, VL models, Gemma 1 / 2, Mistral / Mixtral, Phi, MoE),
and so are the wrong containers (Gemma4 not from safetensors, LFM2 not from GGUF, BERT from HF safetensors,
GGUF Llama / Gemma).  ``NANOVLLM_ARCH`` may confirm the detected family but never override it.
"""
from __future__ import annotations

import os
import re
from dataclasses import dataclass
from typing import List, Optional

from ..exceptions import UnsupportedModelException

CATALOG = (
    "Supported by this library:\n"
    "  Chat from a Hugging Face folder (config.json + *.safetensors or *.onnx): qwen3, gemma3 / gemma3_text, "
    "gemma4 (text / QAT mobile), llama\n"
    "  Chat from a GGUF file: qwen3, lfm2\n"
    "  Embeddings from GGUF or ONNX: bert\n"
    "Not supported: Qwen2 / Qwen2.5, Qwen3.5 / Qwen3-Next, vision-language models, Gemma 1 / 2, Gemma 4 "
    "vision/audio towers, Mistral / Mixtral, Phi, MoE, GGUF Llama / Gemma, Hugging Face BERT safetensors.")

SRC_HF_SAFETENSORS, SRC_ONNX, SRC_GGUF = "hf-safetensors", "onnx", "gguf"
QWEN3, GEMMA3, GEMMA4, LLAMA, LFM2, BERT = "qwen3", "gemma3", "gemma4", "llama", "lfm2", "bert"

_SUFFIX = re.compile(r"(ForCausalLM|ForConditionalGeneration|ForSequenceClassification|ForMaskedLM|"
                     r"ForQuestionAnswering|ForTokenClassification|ForImageTextToText|ForVision2Seq|Model)$")


@dataclass(frozen=True)
class Selection:
    architecture: str
    embedding: bool


def _norm(s: Optional[str]) -> str:
    s = (s or "").strip()
    s = _SUFFIX.sub("", s)
    return re.sub(r"[^a-z0-9]", "", s.lower())


def _classify(token: str):
    """-> (architecture or None, supported, detail)"""
    if not token:
        return None
    rejects = [
        (("qwen35", "qwen3next", "qwen3moe", "qwen3vl", "fara"), "Qwen3.5 / Qwen3-Next / MoE / VL variants"),
        (("qwen2", "qwen25", "qwen"), "Qwen2 / Qwen2.5 (only Qwen3 text models are supported)"),
        (("gemma3n",), "Gemma 3n"),
        (("gemma2", "gemma1"), "Gemma 1 / 2"),
        (("mixtral", "mistral"), "Mistral / Mixtral"),
        (("phi",), "Phi"),
        (("llava", "paligemma", "idefics", "vision", "vl"), "vision-language models"),
    ]
    if token in ("qwen3", "qwen3forcausallm") or token == "qwen3":
        return QWEN3, True, ""
    if token.startswith("qwen3") and token not in ("qwen3",):
        for keys, what in rejects[:1]:
            if any(token.startswith(k) for k in keys):
                return None, False, f"{what} are not supported."
    if token in ("gemma3", "gemma3text"):
        return GEMMA3, True, ""
    if token in ("gemma4", "gemma4text"):
        return GEMMA4, True, ""
    if token == "llama":
        return LLAMA, True, ""
    if token in ("lfm2",):
        return LFM2, True, ""
    if token in ("bert", "nomicbert", "jinabert"):
        return BERT, True, ""
    for keys, what in rejects:
        if any(token.startswith(k) for k in keys):
            return None, False, f"{what} are not supported."
    if "moe" in token:
        return None, False, "mixture-of-experts models are not supported."
    return None


def _unsupported(detail: str, model_type, archs) -> UnsupportedModelException:
    return UnsupportedModelException(f"{detail} (model_type={model_type!r}, architectures={archs!r})\n\n{CATALOG}")


def resolve(hf) -> Selection:
    """HfConfig -> Selection, rejecting look-alikes, MoE flags and multimodal-only checkpoints."""
    candidates = [hf.model_type] + list(hf.architectures or [])
    verdict = None
    for c in candidates:
        v = _classify(_norm(c))
        if v is not None:
            verdict = v
            if not v[1]:
                break
            if v[0] is not None:
                break
    if verdict is None:
        raise _unsupported("Architecture is not recognized.", hf.model_type, hf.architectures)
    arch, ok, detail = verdict
    if not ok:
        raise _unsupported(detail, hf.model_type, hf.architectures)
    raw = hf.raw or {}
    if raw.get("num_experts") or raw.get("num_local_experts") or (hf.gemma4 and hf.gemma4.enable_moe_block):
        raise _unsupported("mixture-of-experts models are not supported.", hf.model_type, hf.architectures)
    forced = os.environ.get("NANOVLLM_ARCH")
    if forced and _norm(forced) != arch:
        raise _unsupported(f"NANOVLLM_ARCH={forced!r} does not match the detected architecture {arch!r}",
                           hf.model_type, hf.architectures)
    return Selection(arch, arch == BERT)


def resolve_gguf(general_architecture: Optional[str]) -> Selection:
    v = _classify(_norm(general_architecture))
    if v is None:
        raise _unsupported(f"GGUF architecture {general_architecture!r} is not recognized.", general_architecture, [])
    arch, ok, detail = v
    if not ok:
        raise _unsupported(detail, general_architecture, [])
    return Selection(arch, arch == BERT)


def require(hf, source: str) -> Selection:
    sel = resolve(hf)
    check_source(sel, source, hf.model_type, hf.architectures)
    return sel


def check_source(sel: Selection, source: str, model_type=None, archs=None) -> None:
    a = sel.architecture
    if a == GEMMA4 and source != SRC_HF_SAFETENSORS:
        raise _unsupported("gemma4 loads from a Hugging Face folder (config.json + *.safetensors QAT), not from "
                           "GGUF or ONNX; vision and audio towers are skipped.", model_type, archs)
    if a in (GEMMA3, LLAMA) and source == SRC_GGUF:
        raise _unsupported(f"{a} loads from a Hugging Face folder, not from GGUF. GGUF chat is qwen3 and lfm2.",
                           model_type, archs)
    if a == LFM2 and source != SRC_GGUF:
        raise _unsupported("LFM2 loads from a .gguf file only.", model_type, archs)
    if a == BERT and source == SRC_HF_SAFETENSORS:
        raise _unsupported("BERT embeddings load from GGUF or ONNX, not from Hugging Face safetensors.",
                           model_type, archs)


def chat_misuse_message(arch: str) -> str:
    return f"This checkpoint is a {arch} embedding encoder, not a chat model; call LlmModel.embed().\n\n{CATALOG}"


def embed_misuse_message(arch: str) -> str:
    return f"This checkpoint is a {arch} chat model, not an embedding encoder; use LLM.builder(model).\n\n{CATALOG}"
