"""Model blueprint (``HfConfig``) and engine knobs (``EngineConfig``).

``HfConfig`` parses a Hugging Face ``config.json`` (or the JSON-shaped dict that the GGUF binder produces)
with the same defaults and per-layer helpers as the reference record
(nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/llm/Config.java:587-907):
``attention_scale`` (Config.java:728-733), ``is_sliding_layer`` (every layer except each 6th when only
``sliding_window`` is given, Config.java:898-907), ``is_conv_layer``, ``layer_head_dim``,
``is_kv_shared_layer`` / ``kv_producer_layer`` (Gemma4 shared KV) and the Gemma4 ``text_config`` flattener.

``EngineConfig`` carries the engine defaults of Config.java:278-286 (max_num_batched_tokens=16384,
max_num_seqs=512, max_model_len=4096 clamped to max_position_embeddings, block size 256 and a multiple of
256).  The JVM-heap fraction that sized the KV pool in the reference becomes ``gpu_memory_utilization``:
KV blocks are sized from free device memory after weights and activation workspaces are resident.
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import dataclass, field
from typing import Any, Optional


@dataclass
class Gemma4Text:
    hidden_size_per_layer_input: int = 256
    num_kv_shared_layers: int = 0
    use_double_wide_mlp: bool = False
    global_head_dim: int = 512
    full_partial_rotary_factor: float = 0.25
    final_logit_softcapping: float = 0.0
    enable_moe_block: bool = False


def _is_gemma4_family(model_type: Optional[str]) -> bool:
    return model_type in ("gemma4", "gemma4_text")


@dataclass
class HfConfig:
    vocab_size: int = 0
    hidden_size: int = 0
    intermediate_size: int = 0
    num_hidden_layers: int = 0
    num_attention_heads: int = 0
    num_key_value_heads: int = 0
    head_dim: int = 0
    max_position_embeddings: int = 32768
    rms_norm_eps: float = 1e-6
    hidden_act: str = "silu"
    tie_word_embeddings: bool = False
    attention_bias: bool = False
    rope_theta: float = 1_000_000.0
    rope_scaling: Optional[dict] = None
    torch_dtype: str = "float16"
    model_type: Optional[str] = None
    architectures: Optional[list] = None
    hidden_activation: Optional[str] = None
    sliding_window: int = 0
    layer_types: Optional[list] = None
    rope_local_base_freq: float = 10_000.0
    query_pre_attn_scalar: float = 0.0
    conv_l_cache: int = 0
    vision: bool = False
    image: bool = False
    audio: bool = False
    video: bool = False
    nested_text: bool = False
    gemma4: Optional[Gemma4Text] = None
    # Fields that are not part of the reference record but that some families need.
    layer_norm_eps: float = 1e-12
    type_vocab_size: int = 2
    final_logit_softcapping: float = 0.0
    attn_logit_softcapping: float = 0.0
    bos_token_id: Optional[int] = None
    eos_token_id: Any = None
    pad_token_id: Optional[int] = None
    layer_kv_heads: Optional[list] = None  # LFM2: per-layer KV head count, 0 = conv layer
    raw: dict = field(default_factory=dict, repr=False)

    # ------------------------------------------------------------------ parsing
    @staticmethod
    def load(path: str) -> "HfConfig":
        with open(path, "r", encoding="utf-8") as f:
            return HfConfig.parse(f.read())

    @staticmethod
    def parse(text_or_dict) -> "HfConfig":
        if isinstance(text_or_dict, (str, bytes)):
            from .utils.json_limits import loads
            root = loads(text_or_dict, "config.json")
        else:
            root = dict(text_or_dict)
        model_type = root.get("model_type")
        nested = isinstance(root.get("text_config"), dict)
        image = "vision_config" in root or "image_token_id" in root
        audio = "audio_config" in root or "audio_token_id" in root
        video = "video_config" in root or "video_token_id" in root
        if _is_gemma4_family(model_type) and nested:
            m = dict(root["text_config"])
            m["model_type"] = model_type
        else:
            m = root
            model_type = m.get("model_type")
        hidden = int(m.get("hidden_size", 0) or 0)
        heads = int(m.get("num_attention_heads", 0) or m.get("num_heads", 0) or 0)
        head_dim = int(m["head_dim"]) if m.get("head_dim") else (hidden // heads if heads else 0)
        archs = root.get("architectures", m.get("architectures"))
        if "rms_norm_eps" in m:
            eps = float(m["rms_norm_eps"])
        else:
            eps = float(m.get("norm_eps", 1e-6))
        theta = float(m.get("rope_theta", 1_000_000.0))
        local = float(m.get("rope_local_base_freq", 10_000.0))
        partial = 0.25
        rp = m.get("rope_parameters")
        if isinstance(rp, dict):
            theta = float(rp.get("rope_theta", theta))
            if isinstance(rp.get("sliding_attention"), dict):
                local = float(rp["sliding_attention"].get("rope_theta", local))
            if isinstance(rp.get("full_attention"), dict):
                theta = float(rp["full_attention"].get("rope_theta", theta))
                partial = float(rp["full_attention"].get("partial_rotary_factor", partial))
        g4 = None
        if _is_gemma4_family(model_type):
            g4 = Gemma4Text(
                hidden_size_per_layer_input=int(m.get("hidden_size_per_layer_input", 256)),
                num_kv_shared_layers=int(m.get("num_kv_shared_layers", 0)),
                use_double_wide_mlp=bool(m.get("use_double_wide_mlp", False)),
                global_head_dim=int(m.get("global_head_dim", 512)),
                full_partial_rotary_factor=partial,
                final_logit_softcapping=float(m.get("final_logit_softcapping", 0.0) or 0.0),
                enable_moe_block=bool(m.get("enable_moe_block", False)),
            )
        qpre = float(m["query_pre_attn_scalar"]) if m.get("query_pre_attn_scalar") is not None else 0.0
        eos = m.get("eos_token_id", root.get("eos_token_id"))
        return HfConfig(
            vocab_size=int(m.get("vocab_size", 0) or 0),
            hidden_size=hidden,
            intermediate_size=int(m.get("intermediate_size", 0) or 0),
            num_hidden_layers=int(m.get("num_hidden_layers", 0) or 0),
            num_attention_heads=heads,
            num_key_value_heads=int(m.get("num_key_value_heads", heads) or heads),
            head_dim=head_dim,
            max_position_embeddings=int(m.get("max_position_embeddings", 32768) or 32768),
            rms_norm_eps=eps,
            hidden_act=str(m.get("hidden_act", "silu") or "silu"),
            tie_word_embeddings=bool(m.get("tie_word_embeddings", root.get("tie_word_embeddings", False))),
            attention_bias=bool(m.get("attention_bias", False)),
            rope_theta=theta,
            rope_scaling=m.get("rope_scaling") if isinstance(m.get("rope_scaling"), dict) else None,
            torch_dtype=str(m.get("torch_dtype", m.get("dtype", "float16")) or "float16"),
            model_type=model_type,
            architectures=list(archs) if isinstance(archs, list) else None,
            hidden_activation=m.get("hidden_activation"),
            sliding_window=int(m.get("sliding_window", 0) or 0),
            layer_types=list(m["layer_types"]) if isinstance(m.get("layer_types"), list) else None,
            rope_local_base_freq=local,
            query_pre_attn_scalar=qpre,
            conv_l_cache=int(m.get("conv_L_cache", 0) or 0),
            vision=image or video,
            image=image,
            audio=audio,
            video=video,
            nested_text=nested,
            gemma4=g4,
            layer_norm_eps=float(m.get("layer_norm_eps", 1e-12) or 1e-12),
            type_vocab_size=int(m.get("type_vocab_size", 2) or 2),
            final_logit_softcapping=float(m.get("final_logit_softcapping", 0.0) or 0.0),
            attn_logit_softcapping=float(m.get("attn_logit_softcapping", 0.0) or 0.0),
            bos_token_id=m.get("bos_token_id", root.get("bos_token_id")),
            eos_token_id=eos,
            pad_token_id=m.get("pad_token_id", root.get("pad_token_id")),
            layer_kv_heads=m.get("layer_kv_heads"),
            raw=root,
        )

    def to_dict(self) -> dict:
        """JSON-shaped dict (``config.json`` style) that ``parse`` reads back."""
        d = {
            "vocab_size": self.vocab_size,
            "hidden_size": self.hidden_size,
            "intermediate_size": self.intermediate_size,
            "num_hidden_layers": self.num_hidden_layers,
            "num_attention_heads": self.num_attention_heads,
            "num_key_value_heads": self.num_key_value_heads,
            "head_dim": self.head_dim,
            "max_position_embeddings": self.max_position_embeddings,
            "rms_norm_eps": self.rms_norm_eps,
            "hidden_act": self.hidden_act,
            "tie_word_embeddings": self.tie_word_embeddings,
            "attention_bias": self.attention_bias,
            "rope_theta": self.rope_theta,
            "torch_dtype": self.torch_dtype,
            "model_type": self.model_type,
            "architectures": self.architectures,
        }
        if self.rope_scaling:
            d["rope_scaling"] = self.rope_scaling
        if self.hidden_activation:
            d["hidden_activation"] = self.hidden_activation
        if self.sliding_window:
            d["sliding_window"] = self.sliding_window
        if self.layer_types:
            d["layer_types"] = self.layer_types
        if self.query_pre_attn_scalar:
            d["query_pre_attn_scalar"] = self.query_pre_attn_scalar
        if self.model_type and self.model_type.startswith("gemma"):
            d["rope_local_base_freq"] = self.rope_local_base_freq
        if self.conv_l_cache:
            d["conv_L_cache"] = self.conv_l_cache
        if self.final_logit_softcapping:
            d["final_logit_softcapping"] = self.final_logit_softcapping
        if self.eos_token_id is not None:
            d["eos_token_id"] = self.eos_token_id
        if self.bos_token_id is not None:
            d["bos_token_id"] = self.bos_token_id
        if self.layer_kv_heads is not None:
            d["layer_kv_heads"] = self.layer_kv_heads
        if self.model_type == "bert":
            d["layer_norm_eps"] = self.layer_norm_eps
            d["type_vocab_size"] = self.type_vocab_size
        if self.gemma4 is not None:
            g = self.gemma4
            d.update({
                "hidden_size_per_layer_input": g.hidden_size_per_layer_input,
                "num_kv_shared_layers": g.num_kv_shared_layers,
                "use_double_wide_mlp": g.use_double_wide_mlp,
                "global_head_dim": g.global_head_dim,
                "final_logit_softcapping": g.final_logit_softcapping,
                "enable_moe_block": g.enable_moe_block,
                "rope_parameters": {
                    "sliding_attention": {"rope_theta": self.rope_local_base_freq},
                    "full_attention": {"rope_theta": self.rope_theta,
                                       "partial_rotary_factor": g.full_partial_rotary_factor},
                },
            })
        return {k: v for k, v in d.items() if v is not None}

    # ------------------------------------------------------------------ helpers
    def attention_scale(self) -> float:
        if self.gemma4 is not None:
            return 1.0
        denom = self.query_pre_attn_scalar if self.query_pre_attn_scalar > 0 else self.head_dim
        return float(denom) ** -0.5

    def effective_activation(self) -> str:
        if self.hidden_activation:
            return self.hidden_activation
        return self.hidden_act or "silu"

    def is_sliding_layer(self, i: int) -> bool:
        if self.layer_types is not None and 0 <= i < len(self.layer_types):
            t = self.layer_types[i]
            return t is not None and "sliding" in t.lower()
        if self.sliding_window > 0:
            return (i + 1) % 6 != 0
        return False

    def is_conv_layer(self, i: int) -> bool:
        if self.layer_types is not None and 0 <= i < len(self.layer_types):
            t = (self.layer_types[i] or "").lower()
            return "conv" in t and "attention" not in t
        return False

    def is_gemma4(self) -> bool:
        return self.gemma4 is not None

    def layer_head_dim(self, i: int) -> int:
        if self.gemma4 is None:
            return self.head_dim
        return self.head_dim if self.is_sliding_layer(i) else self.gemma4.global_head_dim

    def mlp_intermediate_size(self, i: int) -> int:
        if self.gemma4 is None:
            return self.intermediate_size
        if self.gemma4.use_double_wide_mlp and self.is_kv_shared_layer(i):
            return self.intermediate_size * 2
        return self.intermediate_size

    def first_kv_shared_layer(self) -> int:
        if self.gemma4 is None or self.gemma4.num_kv_shared_layers <= 0:
            return self.num_hidden_layers
        return self.num_hidden_layers - self.gemma4.num_kv_shared_layers

    def is_kv_shared_layer(self, i: int) -> bool:
        first = self.first_kv_shared_layer()
        return first > 0 and i >= first

    def kv_producer_layer(self, i: int) -> int:
        if not self.is_kv_shared_layer(i):
            return i
        sliding = self.is_sliding_layer(i)
        for j in range(self.first_kv_shared_layer() - 1, -1, -1):
            if self.is_sliding_layer(j) == sliding:
                return j
        raise RuntimeError(f"no KV producer layer of matching type for shared layer {i}")

    def layer_rope_base(self, i: int) -> float:
        if self.model_type and self.model_type.startswith("gemma") and self.is_sliding_layer(i):
            return self.rope_local_base_freq
        theta = self.rope_theta
        if self.rope_scaling and "rope_theta" in self.rope_scaling:
            theta = float(self.rope_scaling["rope_theta"])
        return theta

    def layer_window(self, i: int) -> int:
        return self.sliding_window if (self.sliding_window > 0 and self.is_sliding_layer(i)) else 0

    def kv_layers(self) -> list:
        """Indices of layers that own a KV cache (attention layers that are not KV-shared)."""
        return [i for i in range(self.num_hidden_layers)
                if not self.is_conv_layer(i) and not self.is_kv_shared_layer(i)]


@dataclass
class EngineConfig:
    """Engine knobs (Config.java:278-286 defaults) plus the device-side additions."""
    max_num_batched_tokens: int = 16384
    max_num_seqs: int = 512
    max_model_len: int = 4096
    kvcache_block_size: int = 256
    num_kvcache_blocks: int = -1
    gpu_memory_utilization: float = 0.90
    tensor_parallel_size: int = 1
    enforce_eager: bool = False
    cuda_graph_max_bs: int = 512
    kv_cache_dtype: str = "bf16"
    eos: int = -1
    stop_token_ids: tuple = ()
    stop_on_degenerate: bool = True
    enable_prefix_caching: bool = True
    fused_comm: bool = True
    seed: int = 0
    # TP request intake: "spmd" = every rank receives the same requests and schedules them itself; "rank0" = only
    # rank 0 takes requests and broadcasts each step's plan, the other ranks run ``LLM.serve_worker``
    front_door: str = "spmd"
    # debug: check every step's ids / positions / slots / block tables / state rows on the host before the kernels
    # use them as addresses, and that no KV slot or shared page is written twice (engine/checks.py)
    check_inputs: bool = False

    def __post_init__(self):
        if self.kvcache_block_size % 256 != 0:
            raise ValueError("kvcache_block_size must be a multiple of 256")
        if not (0.0 < self.gpu_memory_utilization <= 1.0):
            raise ValueError("gpu_memory_utilization must be in (0, 1]")
        if self.max_num_seqs < 1 or self.max_num_batched_tokens < 1:
            raise ValueError("max_num_seqs and max_num_batched_tokens must be >= 1")
        if os.environ.get("NVB_CHECK_INPUTS") not in (None, "", "0"):
            self.check_inputs = True
        self.front_door = os.environ.get("NVB_TP_FRONT_DOOR", self.front_door)
        if self.front_door not in ("spmd", "rank0"):
            raise ValueError("front_door must be 'spmd' or 'rank0'")
        env = os.environ.get("NANOVLLM_ENFORCE_EAGER")
        if env is not None:
            self.enforce_eager = env not in ("0", "false", "False")

    def clamp_to_model(self, hf: HfConfig) -> None:
        self.max_model_len = min(self.max_model_len, hf.max_position_embeddings)


def kv_bytes_per_block(hf: HfConfig, block_size: int, elem_bytes: int, tp: int = 1) -> int:
    """Bytes of K+V cache per block summed over KV-owning layers (Config.java:93-125, shared layers skipped)."""
    total = 0
    for i in hf.kv_layers():
        kvh = max(1, hf.num_key_value_heads // tp) if hf.num_key_value_heads >= tp else 1
        total += 2 * block_size * kvh * hf.layer_head_dim(i) * elem_bytes
    return total


def resolve_num_kv_blocks(cfg: EngineConfig, hf: HfConfig, free_bytes: int, elem_bytes: int = 2,
                          tp: int = 1) -> int:
    """KV block count: explicit if configured, else min(estimate, budget / bytes_per_block), at least 32."""
    if cfg.num_kvcache_blocks > 0:
        return cfg.num_kvcache_blocks
    per_seq = math.ceil(cfg.max_model_len / cfg.kvcache_block_size)
    estimated = max(cfg.max_num_seqs * per_seq, 128)
    bpb = max(1, kv_bytes_per_block(hf, cfg.kvcache_block_size, elem_bytes, tp))
    cap = max(32, int(free_bytes) // bpb)
    return int(min(estimated, cap))
