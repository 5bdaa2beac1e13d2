"""Gemma3 text causal LM.

Reference graph: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/internal/Gemma3ForCausalLM.java:41-297
-- embeddings scaled by sqrt(H); sandwich norms (x + post_attn_norm(attn(input_norm(x))),
x + post_ffw_norm(mlp(pre_ffw_norm(x)))), every RMSNorm and the q/k norms use (1 + w); sliding layers use
``rope_local_base_freq`` and the ``sliding_window``, global layers ``rope_theta`` (layer type from ``layer_types``,
else every 6th layer is global); attention scale ``query_pre_attn_scalar^-0.5``; GELU-tanh(gate) * up MLP; the LM
head reuses the embeddings when ``lm_head`` is absent.  The post-attention norm and the residual add + pre-FFW
norm are two fused RMSNorm launches.
"""
from __future__ import annotations

import math
from typing import Dict

import torch

from .. import ops
from ..config import HfConfig
from ..layers.attention import Attention
from ..layers.embedding import ParallelLMHead, VocabParallelEmbedding
from ..layers.linear import MergedColumnParallelLinear, QKVParallelLinear, RowParallelLinear
from ..layers.norms import RMSNorm, RotaryTables
from .base import CausalLMBase, WeightBag, random_weights


def param_shapes(hf: HfConfig):
    H, I, hd = hf.hidden_size, hf.intermediate_size, hf.head_dim
    nq, nkv = hf.num_attention_heads, hf.num_key_value_heads
    out = [("model.embed_tokens.weight", (hf.vocab_size, H))]
    for i in range(hf.num_hidden_layers):
        p = f"model.layers.{i}."
        out += [(p + n, (H,)) for n in ("input_layernorm.weight", "post_attention_layernorm.weight",
                                         "pre_feedforward_layernorm.weight", "post_feedforward_layernorm.weight")]
        out += [(p + "self_attn.q_proj.weight", (nq * hd, H)), (p + "self_attn.k_proj.weight", (nkv * hd, H)),
                (p + "self_attn.v_proj.weight", (nkv * hd, H)), (p + "self_attn.o_proj.weight", (H, nq * hd)),
                (p + "self_attn.q_norm.weight", (hd,)), (p + "self_attn.k_norm.weight", (hd,)),
                (p + "mlp.gate_proj.weight", (I, H)), (p + "mlp.up_proj.weight", (I, H)),
                (p + "mlp.down_proj.weight", (H, I))]
    out.append(("model.norm.weight", (H,)))
    return out


def init_random(hf: HfConfig, seed: int, device="cpu") -> Dict[str, torch.Tensor]:
    # (1 + w) norms: w = 0 gives the unit scale
    return random_weights(param_shapes(hf), seed, device, zeros_for=lambda n: n.endswith("norm.weight"))


class _L:
    pass


class Gemma3ForCausalLM(CausalLMBase):
    def __init__(self, hf: HfConfig, weights, device, dtype=torch.bfloat16, max_pos: int = None):
        self.hf = hf
        bag = WeightBag(weights, device, dtype)
        H, hd, eps = hf.hidden_size, hf.head_dim, hf.rms_norm_eps
        self.rope = RotaryTables(max_pos or hf.max_position_embeddings, device)
        emb = bag.require("model.embed_tokens.weight")
        self.embed = VocabParallelEmbedding(emb, scale=math.sqrt(H))
        self.layers = []
        act = ops.ACT_GELU_MUL
        for i in range(hf.num_hidden_layers):
            p = f"model.layers.{i}."
            L = _L()
            L.input_norm = RMSNorm(bag.require(p + "input_layernorm.weight"), eps, one_plus=True)
            L.post_attn_norm = RMSNorm(bag.require(p + "post_attention_layernorm.weight"), eps, one_plus=True)
            L.pre_ffw_norm = RMSNorm(bag.require(p + "pre_feedforward_layernorm.weight"), eps, one_plus=True)
            L.post_ffw_norm = RMSNorm(bag.require(p + "post_feedforward_layernorm.weight"), eps, one_plus=True)
            L.qkv = QKVParallelLinear(bag.require(p + "self_attn.q_proj.weight"), bag.require(p + "self_attn.k_proj.weight"),
                                      bag.require(p + "self_attn.v_proj.weight"), hf.num_attention_heads,
                                      hf.num_key_value_heads, hd)
            L.attn = Attention(L.qkv.nq, L.qkv.nkv, hd, hf.attention_scale(), self.rope.get(hd, hf.layer_rope_base(i)),
                               bag.require(p + "self_attn.q_norm.weight"), bag.require(p + "self_attn.k_norm.weight"),
                               1, eps, window=hf.layer_window(i), softcap=hf.attn_logit_softcapping)
            L.o_proj = RowParallelLinear(bag.require(p + "self_attn.o_proj.weight"))
            L.gate_up = MergedColumnParallelLinear(bag.require(p + "mlp.gate_proj.weight"),
                                                   bag.require(p + "mlp.up_proj.weight"), act)
            L.down = RowParallelLinear(bag.require(p + "mlp.down_proj.weight"))
            self.layers.append(L)
        self.norm = RMSNorm(bag.require("model.norm.weight"), eps, one_plus=True)
        head = bag.find("lm_head.weight")
        self.lm_head = ParallelLMHead(head if head is not None else emb, hf.vocab_size)
        self.final_softcap = hf.final_logit_softcapping

    def kv_specs(self):
        return [(i, L.attn.nkv, L.attn.hd) for i, L in enumerate(self.layers)]

    def bind_kv(self, caches):
        for i, L in enumerate(self.layers):
            L.attn.bind_cache(*caches[i])

    def forward(self, ids, positions):
        h = self.embed(ids)
        residual = None
        for L in self.layers:
            if residual is None:
                residual = h
                x, _ = L.input_norm(h)
            else:
                x, residual = L.input_norm(h, residual)
            a = L.o_proj(L.attn(L.qkv(x), positions))
            a, _ = L.post_attn_norm(a)
            x, residual = L.pre_ffw_norm(a, residual)
            m = L.down(L.gate_up(x))
            h, _ = L.post_ffw_norm(m)
        out, _ = self.norm(h, residual)
        return out

    def compute_logits(self, hidden):
        return self.lm_head(hidden)
