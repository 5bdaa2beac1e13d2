"""Gemma4 text causal LM (the QAT "mobile" family: E2B / E4B).

Reference graph: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/internal/Gemma4ForCausalLM.java
:39-399 with Config.java:810-934:
* embeddings x sqrt(H); per-layer inputs (PLE) = (rmsnorm(proj(embeds) / sqrt(H)) + embed_per_layer(ids) *
  sqrt(P)) / sqrt(2), one P-wide slice per layer;
* layer: h += post_attn_norm(attn(input_norm(h))); h += post_ffw_norm(mlp(pre_ffw_norm(h)));
  h += post_ple_norm(ple_proj(gelu(ple_gate(h)) * ple_i)); h *= layer_scalar.  Norms use the stored weight;
* attention: q_norm; k_norm and a weightless v_norm on KV-owning layers; scale 1.0; sliding layers use
  ``head_dim``, the local RoPE base and the window, global layers use ``global_head_dim`` and proportional
  partial RoPE; the last ``num_kv_shared_layers`` layers project only q and read the KV cache of the last
  earlier layer of the same type;
* GELU-tanh(gate) * up MLP (double width on KV-shared layers with ``use_double_wide_mlp``);
* every linear (and the embeddings) comes packed (int2 / int4 / int8 + per-block scales) with optional
  static-range activation quantisation (SRQ) of its input and output; final-logit tanh softcap.

B200 layout: packed weights are expanded to bf16 once on the device (the tcgen05 GEMMs run bf16); q/k/v and
gate/up run as single GEMMs when their SRQ input scales agree (gate/up with the GELU fused into the epilogue when
no output SRQ is present); "norm then add into the residual" (+ layer_scalar) is one kernel; the PLE combine is
one kernel.  Tensor parallelism is not offered for this family (mobile-sized models).
"""
from __future__ import annotations

import math
import os
from typing import Dict, List, Optional, Sequence

import torch

from .. import ops
from ..config import HfConfig
from ..layers.attention import Attention
from ..layers.embedding import ParallelLMHead, VocabParallelEmbedding
from ..layers.norms import RMSNorm, RotaryTables
from ..ops.quant import cat_rows
from ..parallel import state as tp
from .base import CausalLMBase, WeightBag, random_weights, unpacking


def _dims(hf: HfConfig, i: int):
    return hf.layer_head_dim(i), hf.mlp_intermediate_size(i)


def param_shapes(hf: HfConfig):
    H, V, L = hf.hidden_size, hf.vocab_size, hf.num_hidden_layers
    P = hf.gemma4.hidden_size_per_layer_input
    nq, nkv = hf.num_attention_heads, hf.num_key_value_heads
    out = [("model.embed_tokens.weight", (V, H)), ("model.embed_tokens_per_layer.weight", (V, L * P)),
           ("model.per_layer_model_projection.weight", (L * P, H)), ("model.per_layer_projection_norm.weight", (P,))]
    for i in range(L):
        hd, I = _dims(hf, i)
        p = f"model.layers.{i}."
        out += [(p + n, (H,)) for n in ("input_layernorm.weight", "post_attention_layernorm.weight",
                                         "pre_feedforward_layernorm.weight", "post_feedforward_layernorm.weight",
                                         "post_per_layer_input_norm.weight")]
        out += [(p + "self_attn.q_proj.weight", (nq * hd, H)), (p + "self_attn.o_proj.weight", (H, nq * hd)),
                (p + "self_attn.q_norm.weight", (hd,))]
        if not hf.is_kv_shared_layer(i):
            out += [(p + "self_attn.k_proj.weight", (nkv * hd, H)), (p + "self_attn.v_proj.weight", (nkv * hd, H)),
                    (p + "self_attn.k_norm.weight", (hd,))]
        out += [(p + "mlp.gate_proj.weight", (I, H)), (p + "mlp.up_proj.weight", (I, H)),
                (p + "mlp.down_proj.weight", (H, I)), (p + "per_layer_input_gate.weight", (P, H)),
                (p + "per_layer_projection.weight", (H, P)), (p + "layer_scalar", (1,))]
    out.append(("model.norm.weight", (H,)))
    return out


def init_random(hf: HfConfig, seed: int, device="cpu") -> Dict[str, torch.Tensor]:
    w = random_weights(param_shapes(hf), seed, device, ones_for=lambda n: n.endswith("norm.weight"))
    for i in range(hf.num_hidden_layers):
        p = f"model.layers.{i}."
        w[p + "layer_scalar"] = torch.full((1,), 0.875, dtype=torch.bfloat16, device=device)
        # attention scale is 1.0 on unit-RMS q/k: q.k has std sqrt(head_dim), which makes random-init attention
        # near-argmax and numerically chaotic; 0.3 norm gains give O(1) logits like trained checkpoints
        for n in ("self_attn.q_norm.weight", "self_attn.k_norm.weight"):
            if p + n in w:
                w[p + n].fill_(0.3)
    return w


def _srq_scales(t) -> tuple:
    return (float(getattr(t, "in_scale", 0.0)), float(getattr(t, "out_scale", 0.0)))


def _packed(w) -> bool:
    return not isinstance(w, torch.Tensor) and hasattr(w, "linear")


def qat_group_weights(bag, names: Sequence[str], device) -> list:
    """The group's weights as GGUF blocks for the dequant-fused GEMM (QatWeight.to_gguf_blocks) when every
    member converts and packed execution is on (a CUDA device unless NVB_GGUF_PACKED=0; "force" also on the
    CPU), else dense bf16 for all members -- one GEMM never mixes the two."""
    mode = os.environ.get("NVB_GGUF_PACKED", "1")
    on = mode == "force" or (torch.device(device).type == "cuda" and mode not in ("0", "false", "no"))
    if on and not unpacking():
        raws = [bag.tensors.get(n) for n in names]
        blocks = [r.to_gguf_blocks() if hasattr(r, "to_gguf_blocks") else None for r in raws]
        if all(b is not None for b in blocks):
            for n in names:
                bag.used.add(n)
            return [b.to_device(device) for b in blocks]
    return [bag.dense(n) for n in names]


class QatLinearGroup:
    """One GEMM over several packed projections that read the same input (q/k/v or gate/up).

    SRQ: the input is fake-quantised once when every member shares its input scale (else each member runs its
    own GEMM on its own quantised copy); output SRQ is applied per member column range.  ``gelu_mul`` (members
    = [gate, up]) fuses GELU-tanh(gate) * up into the GEMM epilogue when no member has an output scale.
    Members are dense bf16 tensors or GGUF blocks (``qat_group_weights``): packed members are multiplied by the
    dequant-fused GEMM without ever being expanded in memory (the QAT integers stay 4 / 8-bit on the device)."""

    def __init__(self, weights: Sequence, srq: Sequence[tuple], gelu_mul: bool = False):
        self.widths = [int(w.shape[0]) for w in weights]
        self.in_scales = [s[0] for s in srq]
        self.out_scales = [s[1] for s in srq]
        self.gelu_mul = gelu_mul
        self.shared_in = len(set(self.in_scales)) == 1
        self.fused_act = gelu_mul and not any(self.out_scales) and self.widths[0] % 128 == 0
        if self.fused_act:
            if _packed(weights[0]):
                gu = cat_rows([weights[0], weights[1]])
                order = ops.ref.interleave_gate_up(torch.arange(gu.shape[0]).unsqueeze(1), 128).squeeze(1)
                self.w = gu.permute_rows(order)
            else:
                self.w = ops.ref.interleave_gate_up(torch.cat([weights[0], weights[1]], 0)).contiguous()
        elif self.shared_in:
            if len(weights) > 1:
                self.w = cat_rows(list(weights))
                self.w = self.w if _packed(self.w) else self.w.contiguous()
            else:
                self.w = weights[0] if _packed(weights[0]) else weights[0].contiguous()
        else:
            self.ws = [w if _packed(w) else w.contiguous() for w in weights]

    @staticmethod
    def _quant_in(x, s):
        return ops.srq_(ops.materialize(x).clone(), s) if s else x

    @staticmethod
    def _mm(x, w, act: int = ops.ACT_NONE):
        if _packed(w):
            y = w.linear(ops.materialize(x))
            return ops.act_mul(y, act, interleaved=True) if act != ops.ACT_NONE else y
        return ops.linear(x, w, act)

    def __call__(self, x):
        if self.fused_act:
            return self._mm(self._quant_in(x, self.in_scales[0]), self.w, ops.ACT_GELU_MUL)
        if self.shared_in:
            y = ops.materialize(self._mm(self._quant_in(x, self.in_scales[0]), self.w))
        else:
            y = torch.cat([ops.materialize(self._mm(self._quant_in(x, s), w))
                           for w, s in zip(self.ws, self.in_scales)], 1)
        off = 0
        for width, s in zip(self.widths, self.out_scales):
            if s:
                ops.srq_(y[:, off:off + width], s)
            off += width
        if self.gelu_mul:
            return ops.act_mul(y, ops.ACT_GELU_MUL, interleaved=False)
        return y


class _L:
    pass


class Gemma4ForCausalLM(CausalLMBase):
    def __init__(self, hf: HfConfig, weights, device, dtype=torch.bfloat16, max_pos: int = None):
        if hf.gemma4 is None:
            raise ValueError("Gemma4ForCausalLM needs a gemma4 config")
        if tp.tp_size() > 1:
            raise ValueError("the gemma4 family runs on one GPU (tensor parallelism is not offered for it)")
        self.hf = hf
        g4 = hf.gemma4
        bag = WeightBag(weights, device, dtype)
        H, eps, L = hf.hidden_size, hf.rms_norm_eps, hf.num_hidden_layers
        self.P = P = g4.hidden_size_per_layer_input
        self.rope = RotaryTables(max_pos or hf.max_position_embeddings, device)
        emb = bag.dense("model.embed_tokens.weight")
        self.embed = VocabParallelEmbedding(emb, scale=math.sqrt(H))
        self.embed_ple = bag.dense("model.embed_tokens_per_layer.weight")
        self.ple_tok_scale = math.sqrt(P)
        self.ple_proj_w = bag.dense("model.per_layer_model_projection.weight")
        self.ple_norm_w = bag.require("model.per_layer_projection_norm.weight")
        self.ple_proj_scale = 1.0 / math.sqrt(H)
        self.layers: List[_L] = []
        for i in range(L):
            p = f"model.layers.{i}."
            hd, I = _dims(hf, i)
            shared = hf.is_kv_shared_layer(i)
            sliding = hf.is_sliding_layer(i)
            Ly = _L()
            Ly.idx, Ly.shared = i, shared
            Ly.input_norm = RMSNorm(bag.require(p + "input_layernorm.weight"), eps)
            Ly.pre_ffw_norm = RMSNorm(bag.require(p + "pre_feedforward_layernorm.weight"), eps)
            Ly.post_attn_w = bag.require(p + "post_attention_layernorm.weight")
            Ly.post_ffw_w = bag.require(p + "post_feedforward_layernorm.weight")
            Ly.post_ple_w = bag.require(p + "post_per_layer_input_norm.weight")
            Ly.scalar = float(bag.require(p + "layer_scalar").float().reshape(-1)[0])
            names = ["q_proj"] if shared else ["q_proj", "k_proj", "v_proj"]
            raw = [bag.require(p + f"self_attn.{n}.weight") for n in names]
            Ly.qkv = QatLinearGroup(qat_group_weights(bag, [p + f"self_attn.{n}.weight" for n in names], device),
                                    [_srq_scales(r) for r in raw])
            o_raw = bag.require(p + "self_attn.o_proj.weight")
            Ly.o_proj = QatLinearGroup(qat_group_weights(bag, [p + "self_attn.o_proj.weight"], device),
                                       [_srq_scales(o_raw)])
            rope = (self.rope.get(hd, hf.rope_local_base_freq) if sliding
                    else self.rope.get(hd, hf.rope_theta, g4.full_partial_rotary_factor))
            q_norm = bag.require(p + "self_attn.q_norm.weight")
            k_norm = q_norm if shared else bag.require(p + "self_attn.k_norm.weight")
            Ly.attn = Attention(hf.num_attention_heads, hf.num_key_value_heads, hd, hf.attention_scale(), rope, q_norm,
                                k_norm, 0, eps, v_norm=not shared, window=hf.layer_window(i),
                                softcap=hf.attn_logit_softcapping, write_kv=not shared, q_only=shared)
            g_raw, u_raw = bag.require(p + "mlp.gate_proj.weight"), bag.require(p + "mlp.up_proj.weight")
            Ly.gate_up = QatLinearGroup(qat_group_weights(bag, [p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight"],
                                                          device), [_srq_scales(g_raw), _srq_scales(u_raw)], gelu_mul=True)
            d_raw = bag.require(p + "mlp.down_proj.weight")
            Ly.down = QatLinearGroup(qat_group_weights(bag, [p + "mlp.down_proj.weight"], device), [_srq_scales(d_raw)])
            pg_raw = bag.require(p + "per_layer_input_gate.weight")
            Ly.ple_gate = QatLinearGroup(qat_group_weights(bag, [p + "per_layer_input_gate.weight"], device),
                                         [_srq_scales(pg_raw)])
            pp_raw = bag.require(p + "per_layer_projection.weight")
            Ly.ple_proj = QatLinearGroup(qat_group_weights(bag, [p + "per_layer_projection.weight"], device),
                                         [_srq_scales(pp_raw)])
            self.layers.append(Ly)
        self.norm = RMSNorm(bag.require("model.norm.weight"), eps)
        head = bag.dense("lm_head.weight") if bag.has("lm_head.weight") else emb
        self.lm_head = ParallelLMHead(head, hf.vocab_size)
        self.final_softcap = g4.final_logit_softcapping
        self.eps = eps

    # ------------------------------------------------------------------ KV cache
    def kv_specs(self):
        return [(i, L.attn.nkv, L.attn.hd) for i, L in enumerate(self.layers) if not L.shared]

    def bind_kv(self, caches):
        for i, L in enumerate(self.layers):
            L.attn.bind_cache(*caches[self.hf.kv_producer_layer(i)])

    # ------------------------------------------------------------------ forward
    def per_layer_inputs(self, ids: torch.Tensor, h: torch.Tensor) -> torch.Tensor:
        tok = ops.embedding(self.embed_ple, ids, self.ple_tok_scale)
        proj = ops.linear(h, self.ple_proj_w)
        return ops.ple_combine(proj, tok, self.ple_norm_w, self.eps, self.ple_proj_scale, 1.0 / math.sqrt(2.0))

    def forward(self, ids, positions):
        h = self.embed(ids)
        ple = self.per_layer_inputs(ids, h)
        P = self.P
        for L in self.layers:
            x, _ = L.input_norm(h)
            a = L.o_proj(L.attn(L.qkv(x), positions))
            ops.rms_norm_post_add_(a, h, L.post_attn_w, self.eps)
            x, _ = L.pre_ffw_norm(h)
            m = L.down(L.gate_up(x))
            ops.rms_norm_post_add_(m, h, L.post_ffw_w, self.eps)
            g = ops.gate_act_mul(L.ple_gate(h), ple[:, L.idx * P:(L.idx + 1) * P])
            ops.rms_norm_post_add_(L.ple_proj(g), h, L.post_ple_w, self.eps, 0, L.scalar)
        out, _ = self.norm(h)
        return out

    def compute_logits(self, hidden):
        return self.lm_head(hidden)
