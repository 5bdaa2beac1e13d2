"""Qwen3 (and Llama) decoder-only causal LM.

Reference graph: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/internal/Qwen3ForCausalLM.java
(embed -> N x [RMSNorm(+residual) -> qkv -> per-head q_norm / k_norm (skipped with attention_bias) -> RoPE ->
paged attention -> o_proj -> add+RMSNorm -> gate_up -> SiLU*up -> down] -> final norm; LM head = lm_head or
the tied embedding; rope_scaling.rope_theta overrides the base) and LlamaForCausalLM.java (the same without
q/k norms).  Per layer this runs six kernels: fused add+RMSNorm, qkv GEMM, q/k-norm + RoPE + KV store, paged
attention, o_proj GEMM, add+RMSNorm, gate_up GEMM with the SiLU*up epilogue, down GEMM.
"""
from __future__ import annotations

from typing import Dict, List, Tuple

import torch

from .. import ops
from ..config import HfConfig
from ..layers.attention import Attention
from ..layers.embedding import ParallelLMHead, VocabParallelEmbedding
from ..layers.linear import MergedColumnParallelLinear, QKVParallelLinear, RowParallelLinear
from ..layers.norms import RMSNorm, RotaryTables
from ..parallel import sp
from ..parallel import state as ps
from .base import CausalLMBase, WeightBag, random_weights


def param_shapes(hf: HfConfig, qk_norm: bool = True) -> List[Tuple[str, tuple]]:
    H, I, hd = hf.hidden_size, hf.intermediate_size, hf.head_dim
    nq, nkv = hf.num_attention_heads, hf.num_key_value_heads
    out = [("model.embed_tokens.weight", (hf.vocab_size, H))]
    for i in range(hf.num_hidden_layers):
        p = f"model.layers.{i}."
        out += [
            (p + "input_layernorm.weight", (H,)),
            (p + "self_attn.q_proj.weight", (nq * hd, H)),
            (p + "self_attn.k_proj.weight", (nkv * hd, H)),
            (p + "self_attn.v_proj.weight", (nkv * hd, H)),
            (p + "self_attn.o_proj.weight", (H, nq * hd)),
            (p + "post_attention_layernorm.weight", (H,)),
            (p + "mlp.gate_proj.weight", (I, H)),
            (p + "mlp.up_proj.weight", (I, H)),
            (p + "mlp.down_proj.weight", (H, I)),
        ]
        if qk_norm and not hf.attention_bias:
            out += [(p + "self_attn.q_norm.weight", (hd,)), (p + "self_attn.k_norm.weight", (hd,))]
        if hf.attention_bias:
            out += [(p + "self_attn.q_proj.bias", (nq * hd,)), (p + "self_attn.k_proj.bias", (nkv * hd,)),
                    (p + "self_attn.v_proj.bias", (nkv * hd,))]
    out.append(("model.norm.weight", (H,)))
    if not hf.tie_word_embeddings:
        out.append(("lm_head.weight", (hf.vocab_size, H)))
    return out


def init_random(hf: HfConfig, seed: int, device="cpu", qk_norm: bool = True) -> Dict[str, torch.Tensor]:
    return random_weights(param_shapes(hf, qk_norm), seed, device,
                          ones_for=lambda n: n.endswith("norm.weight"))


class _Layer:
    pass


class Qwen3ForCausalLM(CausalLMBase):
    QK_NORM = True

    def __init__(self, hf: HfConfig, weights: Dict[str, object], device, dtype=torch.bfloat16, max_pos: int = None):
        self.hf = hf
        self.device = device
        bag = WeightBag(weights, device, dtype)
        tp = ps.tp_size()
        H, hd = hf.hidden_size, hf.head_dim
        self.rope = RotaryTables(max_pos or hf.max_position_embeddings, device)
        self.embed = VocabParallelEmbedding(bag.require("model.embed_tokens.weight"))
        self.layers = []
        qk_norm = self.QK_NORM and not hf.attention_bias
        eps = hf.rms_norm_eps
        for i in range(hf.num_hidden_layers):
            p = f"model.layers.{i}."
            L = _Layer()
            L.input_norm = RMSNorm(bag.require(p + "input_layernorm.weight"), eps)
            L.qkv = QKVParallelLinear(bag.require(p + "self_attn.q_proj.weight"), bag.require(p + "self_attn.k_proj.weight"),
                                      bag.require(p + "self_attn.v_proj.weight"), hf.num_attention_heads,
                                      hf.num_key_value_heads, hd, bag.find(p + "self_attn.q_proj.bias"),
                                      bag.find(p + "self_attn.k_proj.bias"), bag.find(p + "self_attn.v_proj.bias"))
            qn = bag.require(p + "self_attn.q_norm.weight") if qk_norm else None
            kn = bag.require(p + "self_attn.k_norm.weight") if qk_norm else None
            L.attn = Attention(L.qkv.nq, L.qkv.nkv, hd, hf.attention_scale(), self.rope.get(hd, hf.layer_rope_base(i)),
                               qn, kn, 0 if qk_norm else -1, eps, window=hf.layer_window(i))
            L.o_proj = RowParallelLinear(bag.require(p + "self_attn.o_proj.weight"))
            L.post_norm = RMSNorm(bag.require(p + "post_attention_layernorm.weight"), eps)
            L.gate_up = MergedColumnParallelLinear(bag.require(p + "mlp.gate_proj.weight"),
                                                   bag.require(p + "mlp.up_proj.weight"), ops.ACT_SILU_MUL)
            L.down = RowParallelLinear(bag.require(p + "mlp.down_proj.weight"))
            self.layers.append(L)
        self.norm = RMSNorm(bag.require("model.norm.weight"), eps)
        head = bag.find("lm_head.weight")
        if head is None:
            head = bag.require("model.embed_tokens.weight")
        self.lm_head = ParallelLMHead(head, hf.vocab_size)

    def kv_specs(self):
        return [(i, L.attn.nkv, L.attn.hd) for i, L in enumerate(self.layers)]

    def bind_kv(self, caches):
        for i, L in enumerate(self.layers):
            k, v = caches[i]
            L.attn.bind_cache(k, v)

    def forward(self, ids: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        ws = sp.active_for(ids.shape[0], self.hf.hidden_size, ids.is_cuda)
        if ws is not None:
            return self._forward_sp(ids, positions, ws)
        h = self.embed(ids)
        residual = None
        for L in self.layers:
            if residual is None:
                residual = h
                x, _ = L.input_norm(h)
            else:
                x, residual = L.input_norm(h, residual)
            a = L.attn(L.qkv(x), positions)
            h = L.o_proj(a)
            x, residual = L.post_norm(h, residual)
            h = L.down(L.gate_up(x))
        out, _ = self.norm(h, residual)
        return out

    def _forward_sp(self, ids: torch.Tensor, positions: torch.Tensor, ws):
        """Tensor-parallel forward with the sequence-parallel residual: per layer
        [AG + RMSNorm + qkv GEMM] -> [q/k-norm + RoPE + KV store] -> [paged attention] -> [o_proj GEMM + RS]
        -> [AG + RMSNorm + gate_up GEMM + SiLU*up] -> [down GEMM + RS]; the residual stream never leaves its
        owner rank and no NCCL call remains inside the layers."""
        ws.begin(ids.shape[0])
        part = self.embed.sp_push(ids, ws)
        for i, L in enumerate(self.layers):
            qkv = L.qkv.sp_consume(part, L.input_norm, has_res=i > 0)
            a = L.attn(qkv, positions)
            part = L.o_proj.sp_produce(a, ws)
            x = L.gate_up.sp_consume(part, L.post_norm, has_res=True)
            part = L.down.sp_produce(x, ws)
        return ops.SPHidden(part, self.norm.weight, self.norm.eps, self.norm.mode)

    def compute_logits(self, hidden: torch.Tensor) -> torch.Tensor:
        return self.lm_head(hidden)


class LlamaForCausalLM(Qwen3ForCausalLM):
    QK_NORM = False
