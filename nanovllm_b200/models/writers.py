"""Random-init checkpoint writers: Hugging Face folders (config.json + safetensors + tokenizer.json), GGUF files
and ONNX initializer files, so every loader path can be exercised and benchmarked without downloads.

The checkpoints hold seeded N(0, 0.02) weights (norms 1, or 0 for the (1 + w) Gemma norms); GGUF tensors can be
packed as Q8_0 / F16 or as random K-quant blocks with the same spread.
"""
from __future__ import annotations

import json
import os
from typing import Dict, Optional

import torch

from ..config import HfConfig
from ..loaders.dequant import TYPE_BY_NAME
from ..loaders.gguf import f16_bytes, f32_bytes, pack_random_blocks, quantize_q8_0, write_gguf
from ..loaders.gguf_configs import gguf_metadata_for
from ..loaders.safetensors import save_file


def byte_level_tokenizer_json(vocab_size: int, specials=("<|endoftext|>", "<|im_start|>", "<|im_end|>",
                                                         "<think>", "</think>")) -> dict:
    """A byte-level BPE tokenizer.json over the 256 byte symbols (+ a few merges) padded to ``vocab_size``."""
    from ..tokenizer.codecs import BYTE_ENCODER
    if vocab_size < 256 + len(specials):
        raise ValueError(f"a byte-level vocabulary needs at least {256 + len(specials)} ids")
    vocab = {BYTE_ENCODER[b]: b for b in range(256)}
    merges = []
    nxt = 256
    for a, b in (("t", "h"), ("th", "e"), ("Ġ", "t"), ("i", "n"), ("e", "r"), ("a", "n"), ("o", "n")):
        if nxt >= vocab_size - len(specials):
            break
        vocab[a + b] = nxt
        merges.append(f"{a} {b}")
        nxt += 1
    while nxt < vocab_size - len(specials):
        vocab[f"<filler{nxt}>"] = nxt
        nxt += 1
    # think tags are plain added tokens (special=False) as in Qwen3's tokenizer.json: they survive skip-special decode
    added = [{"id": nxt + i, "content": s, "special": s not in ("<think>", "</think>")} for i, s in enumerate(specials)]
    return {"version": "1.0", "added_tokens": added, "normalizer": None,
            "pre_tokenizer": {"type": "ByteLevel", "add_prefix_space": False, "use_regex": True},
            "decoder": {"type": "ByteLevel"},
            "model": {"type": "BPE", "vocab": vocab, "merges": merges}}


def write_hf_folder(path: str, hf: HfConfig, weights: Dict[str, torch.Tensor], tokenizer_json: Optional[dict] = None,
                    tokenizer_config: Optional[dict] = None, shards: int = 1) -> str:
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(hf.to_dict(), f)
    names = sorted(weights)
    if shards <= 1:
        save_file({k: weights[k] for k in names}, os.path.join(path, "model.safetensors"))
    else:
        wm = {}
        per = (len(names) + shards - 1) // shards
        for s in range(shards):
            part = names[s * per:(s + 1) * per]
            fn = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
            save_file({k: weights[k] for k in part}, os.path.join(path, fn))
            wm.update({k: fn for k in part})
        with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
            json.dump({"weight_map": wm}, f)
    tj = tokenizer_json or byte_level_tokenizer_json(hf.vocab_size)
    with open(os.path.join(path, "tokenizer.json"), "w") as f:
        json.dump(tj, f)
    with open(os.path.join(path, "tokenizer_config.json"), "w") as f:
        json.dump(tokenizer_config or {"eos_token": "<|endoftext|>"}, f)
    return path


def gguf_tokenizer_meta(vocab_size: int, model: str = "gpt2") -> dict:
    tj = byte_level_tokenizer_json(vocab_size) if model == "gpt2" else None
    if model == "gpt2":
        tokens = [None] * vocab_size
        for k, v in tj["model"]["vocab"].items():
            tokens[v] = k
        types = [1] * vocab_size
        for a in tj["added_tokens"]:
            tokens[a["id"]] = a["content"]
            types[a["id"]] = 3
        return {"tokenizer.ggml.model": "gpt2", "tokenizer.ggml.pre": "qwen2", "tokenizer.ggml.tokens": tokens,
                "tokenizer.ggml.token_type": types, "tokenizer.ggml.merges": tj["model"]["merges"],
                "tokenizer.ggml.eos_token_id": vocab_size - 5}
    # WordPiece vocabulary for BERT
    tokens = ["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]"] + [chr(c) for c in range(97, 123)] + \
        [f"##{chr(c)}" for c in range(97, 123)]
    tokens += [f"w{i}" for i in range(vocab_size - len(tokens))]
    return {"tokenizer.ggml.model": "bert", "tokenizer.ggml.tokens": tokens,
            "tokenizer.ggml.token_type": [3] * 5 + [1] * (len(tokens) - 5), "tokenizer.ggml.unknown_token_id": 1,
            "tokenizer.ggml.cls_token_id": 2, "tokenizer.ggml.seperator_token_id": 3,
            "tokenizer.ggml.padding_token_id": 0}


_HF_TO_GGUF_QWEN = {
    "input_layernorm.weight": "attn_norm.weight", "self_attn.q_proj.weight": "attn_q.weight",
    "self_attn.k_proj.weight": "attn_k.weight", "self_attn.v_proj.weight": "attn_v.weight",
    "self_attn.o_proj.weight": "attn_output.weight", "self_attn.q_norm.weight": "attn_q_norm.weight",
    "self_attn.k_norm.weight": "attn_k_norm.weight", "post_attention_layernorm.weight": "ffn_norm.weight",
    "mlp.gate_proj.weight": "ffn_gate.weight", "mlp.up_proj.weight": "ffn_up.weight",
    "mlp.down_proj.weight": "ffn_down.weight",
}


def to_gguf_names(hf: HfConfig, weights: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    if hf.model_type != "qwen3":
        return dict(weights)
    out = {}
    for k, v in weights.items():
        if k == "model.embed_tokens.weight":
            out["token_embd.weight"] = v
        elif k == "model.norm.weight":
            out["output_norm.weight"] = v
        elif k == "lm_head.weight":
            out["output.weight"] = v
        else:
            parts = k.split(".")
            i = int(parts[2])
            rest = ".".join(parts[3:])
            out[f"blk.{i}.{_HF_TO_GGUF_QWEN[rest]}"] = v
    return out


def write_gguf_model(path: str, hf: HfConfig, weights: Dict[str, torch.Tensor], matrix_type: str = "Q8_0",
                     big_type: Optional[str] = None, random_packed: bool = False, seed: int = 0,
                     tokenizer_model: str = "gpt2") -> str:
    """Pack 2-D weights as ``matrix_type`` (``big_type`` for output / ffn_down, as in Q4_K_M), vectors as F32."""
    named = to_gguf_names(hf, weights)
    tensors = {}
    for i, (name, t) in enumerate(sorted(named.items())):
        if t.dim() == 2 and t.shape[1] % 32 == 0:
            tname = big_type if (big_type and (name == "output.weight" or "ffn_down" in name)) else matrix_type
            if tname == "F16":
                tensors[name] = (1, tuple(t.shape), f16_bytes(t))
            elif tname == "Q8_0" and not random_packed:
                tensors[name] = (8, tuple(t.shape), quantize_q8_0(t))
            else:
                tid = TYPE_BY_NAME[tname]
                tensors[name] = (tid, tuple(t.shape), pack_random_blocks(tid, tuple(t.shape), seed + i))
        elif t.dim() == 2:
            tensors[name] = (1, tuple(t.shape), f16_bytes(t))
        else:
            tensors[name] = (0, tuple(t.shape), f32_bytes(t))
    meta = gguf_metadata_for(hf, gguf_tokenizer_meta(hf.vocab_size, tokenizer_model))
    write_gguf(path, meta, tensors)
    return path
