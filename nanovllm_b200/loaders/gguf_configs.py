"""GGUF metadata -> HfConfig, and GGUF tensor names -> the names each model graph consumes.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/llmarch/GgufConfigs.java:30-271 (qwen3 with
``head_dim`` from ``attention.key_length``, lfm2 with the per-layer kv-head array deciding conv vs attention layers
and ``shortconv.l_cache``, bert with its layer-norm epsilon) and WeightSchema.forGguf.  Qwen3 GGUF tensors are
renamed to Hugging Face names (one model graph for both containers); LFM2 and BERT graphs consume GGUF names.
"""
from __future__ import annotations

import re
from typing import Dict, Optional

from ..config import HfConfig
from ..exceptions import ModelLoadException


def _g(meta: dict, arch: str, key: str, default=None):
    return meta.get(f"{arch}.{key}", default)


def hf_config_from_gguf(meta: dict, arch: str) -> HfConfig:
    tokens = meta.get("tokenizer.ggml.tokens") or []
    vocab = int(_g(meta, arch, "vocab_size", len(tokens)) or len(tokens))
    hidden = int(_g(meta, arch, "embedding_length", 0))
    heads = int(_g(meta, arch, "attention.head_count", 0) or 0)
    kv = _g(meta, arch, "attention.head_count_kv", heads)
    layers = int(_g(meta, arch, "block_count", 0))
    ctx = int(_g(meta, arch, "context_length", 2048))
    ffn = _g(meta, arch, "feed_forward_length", 0)
    if isinstance(ffn, list):
        ffn = max(ffn)
    d = dict(vocab_size=vocab, hidden_size=hidden, intermediate_size=int(ffn or 0), num_hidden_layers=layers,
             num_attention_heads=heads, max_position_embeddings=ctx, model_type=arch,
             architectures=[{"qwen3": "Qwen3ForCausalLM", "lfm2": "Lfm2ForCausalLM", "bert": "BertModel",
                             "llama": "LlamaForCausalLM"}.get(arch, arch)])
    eos = meta.get("tokenizer.ggml.eos_token_id")
    bos = meta.get("tokenizer.ggml.bos_token_id")
    if arch == "bert":
        d.update(num_key_value_heads=heads, head_dim=hidden // max(1, heads),
                 layer_norm_eps=float(_g(meta, arch, "attention.layer_norm_epsilon", 1e-12)), hidden_act="gelu")
        hf = HfConfig(**d)
    else:
        if isinstance(kv, list):
            kv_list = [int(x) for x in kv]
            kv_heads = max(kv_list) if kv_list else heads
        else:
            kv_list = None
            kv_heads = int(kv)
        head_dim = int(_g(meta, arch, "attention.key_length", 0) or (hidden // max(1, heads)))
        d.update(num_key_value_heads=kv_heads, head_dim=head_dim,
                 rms_norm_eps=float(_g(meta, arch, "attention.layer_norm_rms_epsilon", 1e-6)),
                 rope_theta=float(_g(meta, arch, "rope.freq_base", 1_000_000.0)))
        if arch == "lfm2":
            if kv_list is None:
                raise ModelLoadException("lfm2 GGUF needs a per-layer attention.head_count_kv array")
            d["layer_types"] = ["full_attention" if k > 0 else "conv" for k in kv_list]
            d["layer_kv_heads"] = kv_list
            d["conv_l_cache"] = int(_g(meta, arch, "shortconv.l_cache", 3))
        hf = HfConfig(**d)
        hf.tie_word_embeddings = False
    hf.eos_token_id = eos
    hf.bos_token_id = bos
    hf.raw = {"gguf": True, "general.architecture": arch}
    return hf


_QWEN_MAP = {
    "attn_norm.weight": "input_layernorm.weight", "attn_q.weight": "self_attn.q_proj.weight",
    "attn_k.weight": "self_attn.k_proj.weight", "attn_v.weight": "self_attn.v_proj.weight",
    "attn_output.weight": "self_attn.o_proj.weight", "attn_q_norm.weight": "self_attn.q_norm.weight",
    "attn_k_norm.weight": "self_attn.k_norm.weight", "ffn_norm.weight": "post_attention_layernorm.weight",
    "ffn_gate.weight": "mlp.gate_proj.weight", "ffn_up.weight": "mlp.up_proj.weight",
    "ffn_down.weight": "mlp.down_proj.weight", "attn_q.bias": "self_attn.q_proj.bias",
    "attn_k.bias": "self_attn.k_proj.bias", "attn_v.bias": "self_attn.v_proj.bias",
}
_BLK = re.compile(r"^blk\.(\d+)\.(.+)$")


def hf_name_for_qwen3(gguf_name: str) -> Optional[str]:
    if gguf_name == "token_embd.weight":
        return "model.embed_tokens.weight"
    if gguf_name == "output_norm.weight":
        return "model.norm.weight"
    if gguf_name == "output.weight":
        return "lm_head.weight"
    m = _BLK.match(gguf_name)
    if m and m.group(2) in _QWEN_MAP:
        return f"model.layers.{int(m.group(1))}.{_QWEN_MAP[m.group(2)]}"
    return None


# ----------------------------------------------------------------------------------------------- writers
def gguf_metadata_for(hf: HfConfig, tokenizer_meta: Optional[dict] = None) -> Dict:
    """Inverse of hf_config_from_gguf for the random-init GGUF writers."""
    arch = hf.model_type
    meta = {"general.architecture": arch, "general.name": f"random-{arch}",
            f"{arch}.block_count": hf.num_hidden_layers, f"{arch}.embedding_length": hf.hidden_size,
            f"{arch}.context_length": hf.max_position_embeddings, f"{arch}.attention.head_count": hf.num_attention_heads}
    if arch == "bert":
        meta[f"{arch}.feed_forward_length"] = hf.intermediate_size
        meta[f"{arch}.attention.layer_norm_epsilon"] = float(hf.layer_norm_eps)
    else:
        meta[f"{arch}.feed_forward_length"] = hf.intermediate_size
        meta[f"{arch}.attention.key_length"] = hf.head_dim
        meta[f"{arch}.attention.value_length"] = hf.head_dim
        meta[f"{arch}.attention.layer_norm_rms_epsilon"] = float(hf.rms_norm_eps)
        meta[f"{arch}.rope.freq_base"] = float(hf.rope_theta)
        if arch == "lfm2":
            meta[f"{arch}.attention.head_count_kv"] = list(hf.layer_kv_heads)
            meta[f"{arch}.shortconv.l_cache"] = hf.conv_l_cache
        else:
            meta[f"{arch}.attention.head_count_kv"] = hf.num_key_value_heads
    meta[f"{arch}.vocab_size"] = hf.vocab_size
    if tokenizer_meta:
        meta.update(tokenizer_meta)
    return meta
