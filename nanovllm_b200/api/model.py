"""``LlmModel``: the loaded-model handle shared by engines.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/LlmModel.java:68-218 and
models/internal/LlmModelImpl.java:29-456 -- tokenizer, config, options, think tags / chat specials, architecture
name, declared vs usable modalities, causal / embedding flag, packed-weight flag, ``embed`` (text, list or ids;
[CLS]..[SEP] or <s>..</s> wrapping, mean pool + L2) and ``close``.  Several ``LLM`` engines may share one model;
the handle counts engines so ``close`` can refuse while engines are alive.
"""
from __future__ import annotations

import threading
from typing import Dict, List, Optional, Sequence, Union

import torch

from ..config import HfConfig


class LlmModel:
    def __init__(self, hf_config: HfConfig, weights: Dict[str, object], tokenizer=None, options: Optional[dict] = None,
                 source: str = "", container: str = "", packed: bool = False):
        self.hf_config = hf_config
        self.weights = weights
        self.tokenizer = tokenizer
        self.options = dict(options or {})
        self.source = source
        self.container = container
        self.packed = packed
        self._engines = 0
        self._lock = threading.Lock()
        self._closed = False
        self._encoder = None

    # ------------------------------------------------------------------ descriptors
    @property
    def architecture_name(self) -> str:
        a = self.hf_config.architectures
        return a[0] if a else (self.hf_config.model_type or "unknown")

    def is_embedding(self) -> bool:
        return (self.hf_config.model_type or "").lower() == "bert"

    def is_causal(self) -> bool:
        return not self.is_embedding()

    def has_packed_weights(self) -> bool:
        return self.packed

    def modalities(self) -> List[str]:
        hf = self.hf_config
        out = ["text"]
        if hf.image:
            out.append("image")
        if hf.audio:
            out.append("audio")
        if hf.video:
            out.append("video")
        return out

    def usable_modalities(self) -> List[str]:
        return ["text->embedding"] if self.is_embedding() else ["text->text"]

    def input_modalities(self) -> List[str]:
        """Inputs the checkpoint declares (text, plus image / audio / video towers it carries)."""
        return self.modalities()

    def output_modalities(self) -> List[str]:
        return ["embedding"] if self.is_embedding() else ["text"]

    @property
    def path(self) -> str:
        """Where the model was loaded from (folder or .gguf file)."""
        return self.source

    def think_tags(self):
        from ..chat.markup import ThinkTags
        return self.options.get("think_tags") or ThinkTags.default()

    def chat_specials(self):
        """Chat-markup markers that end a visible answer (checkpoint option ``chat_specials``, else the default
        ChatML / Gemma / Llama set)."""
        from ..chat.markup import ChatSpecials
        sp = self.options.get("chat_specials")
        if sp is None:
            return ChatSpecials.default()
        return sp if isinstance(sp, ChatSpecials) else ChatSpecials(tuple(sp))

    def __repr__(self) -> str:
        hf = self.hf_config
        return (f"LlmModel(arch={self.architecture_name}, layers={hf.num_hidden_layers}, hidden={hf.hidden_size}, "
                f"heads={hf.num_attention_heads}/{hf.num_key_value_heads}, vocab={hf.vocab_size}, "
                f"container={self.container}, packed={self.packed})")

    # ------------------------------------------------------------------ engines
    def acquire_engine(self) -> None:
        with self._lock:
            if self._closed:
                raise RuntimeError("model is closed")
            self._engines += 1

    def release_engine(self) -> None:
        with self._lock:
            self._engines = max(0, self._engines - 1)

    def close(self) -> None:
        with self._lock:
            if self._engines > 0:
                raise RuntimeError("close the engines that use this model first")
            self._closed = True
            self.weights = {}
            self._encoder = None

    # ------------------------------------------------------------------ embeddings
    def _get_encoder(self, device=None):
        if self._encoder is None:
            from ..models.bert import BertEncoder
            if device is None:
                device = torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
            self._encoder = BertEncoder(self.hf_config, self.weights, torch.device(device))
        return self._encoder

    def embed(self, text: Union[str, Sequence[str], Sequence[int]], device=None) -> torch.Tensor:
        """Mean-pooled, L2-normalised embedding(s): one string -> [H]; a list of strings -> [N, H]; ids -> [H]."""
        if not self.is_embedding():
            raise ValueError("embed() needs an embedding model")
        enc = self._get_encoder(device)
        if isinstance(text, str):
            return enc.embed_ids([self._wrap(self.tokenizer.encode(text))])[0]
        if len(text) > 0 and isinstance(text[0], int):
            return enc.embed_ids([self._wrap(list(text))])[0]
        return enc.embed_ids([self._wrap(self.tokenizer.encode(t)) for t in text])

    def embed_ids(self, batches: List[List[int]], device=None, keep_device: bool = False) -> torch.Tensor:
        return self._get_encoder(device).embed_ids(batches, keep_device=keep_device)

    def embed_batch(self, texts: Sequence[str], device=None) -> torch.Tensor:
        """[N, H] embeddings left on the encoder's device (one packed encoder pass per 64k tokens)."""
        if not self.is_embedding():
            raise ValueError("embed_batch() needs an embedding model")
        ids = [self._wrap(self.tokenizer.encode(t)) for t in texts]
        return self._get_encoder(device).embed_ids(ids, keep_device=True)

    def is_closed(self) -> bool:
        return self._closed

    def _wrap(self, ids: List[int]) -> List[int]:
        tok = self.tokenizer
        cls_id, sep_id = tok.cls_sep_ids()
        limit = self.hf_config.max_position_embeddings
        body = ids[:max(0, limit - 2)]
        out = ([cls_id] if cls_id is not None else []) + body + ([sep_id] if sep_id is not None else [])
        return out[:limit]
