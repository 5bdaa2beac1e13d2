"""LFM2 hybrid causal LM (gated short-conv layers + GQA attention layers), GGUF tensor names.

Reference graph: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/internal/Lfm2ForCausalLM.java:31-304
-- per layer: operator norm -> (attention with q/k norms, or ShortConv) -> residual -> ffn norm -> SwiGLU (separate
gate / up / down) -> residual; the token-embedding norm (``token_embd_norm``) is applied at the END as the output
norm; head_dim = hidden / heads; a layer is a conv layer when its per-layer KV-head count is 0.  Conv layers keep a
per-sequence recurrent state (the last L-1 gated inputs) in the model runner's state arena; attention layers use
the paged KV cache.
"""
from __future__ import annotations

from typing import Dict, List, Tuple

import torch

from .. import ops
from ..config import HfConfig
from ..engine.context import get_context
from ..layers.attention import Attention
from ..layers.embedding import ParallelLMHead, VocabParallelEmbedding
from ..layers.linear import ColumnParallelLinear, MergedColumnParallelLinear, QKVParallelLinear, ReplicatedLinear, \
    RowParallelLinear
from ..layers.norms import RMSNorm, RotaryTables
from ..ops.quant import cat_rows, is_packed
from ..parallel import state as ps
from .base import CausalLMBase, WeightBag, random_weights


def param_shapes(hf: HfConfig) -> List[Tuple[str, tuple]]:
    H, I = hf.hidden_size, hf.intermediate_size
    hd = hf.head_dim
    L = hf.conv_l_cache or 3
    out = [("token_embd.weight", (hf.vocab_size, H)), ("token_embd_norm.weight", (H,))]
    for i in range(hf.num_hidden_layers):
        p = f"blk.{i}."
        out += [(p + "attn_norm.weight", (H,)), (p + "ffn_norm.weight", (H,)), (p + "ffn_gate.weight", (I, H)),
                (p + "ffn_up.weight", (I, H)), (p + "ffn_down.weight", (H, I))]
        if hf.is_conv_layer(i):
            out += [(p + "shortconv.in_proj.weight", (3 * H, H)), (p + "shortconv.conv.weight", (H, L)),
                    (p + "shortconv.out_proj.weight", (H, H))]
        else:
            nkv = hf.layer_kv_heads[i]
            out += [(p + "attn_q.weight", (hf.num_attention_heads * hd, H)), (p + "attn_k.weight", (nkv * hd, H)),
                    (p + "attn_v.weight", (nkv * hd, H)), (p + "attn_output.weight", (H, hf.num_attention_heads * hd)),
                    (p + "attn_q_norm.weight", (hd,)), (p + "attn_k_norm.weight", (hd,))]
    return out


def init_random(hf: HfConfig, seed: int, device="cpu") -> Dict[str, torch.Tensor]:
    return random_weights(param_shapes(hf), seed, device, ones_for=lambda n: n.endswith("norm.weight"))


class ShortConv:
    """in_proj -> fused gated conv kernel (state in the arena) -> out_proj.

    Under TP the conv is channel-parallel (the depthwise conv and the gating never mix channels): rank r keeps
    channels [r*H/TP, (r+1)*H/TP) of each of the B, C and x thirds of in_proj (column-parallel), the same rows of
    the conv weight and a recurrent state of H/TP channels per sequence, and out_proj is row-parallel (its partial
    output is all-reduced, fused with the next add + RMSNorm like o_proj)."""

    def __init__(self, in_proj, conv_w: torch.Tensor, out_proj, hidden: int, layer: int):
        r, s = ps.tp_rank(), ps.tp_size()
        if s > 1:
            if hidden % s != 0:
                raise ValueError(f"hidden size {hidden} is not divisible by TP={s}")
            hl = hidden // s

            def rows(w, a, b):
                return w.rows(a, b) if is_packed(w) else w[a:b]

            in_proj = cat_rows([rows(in_proj, j * hidden + r * hl, j * hidden + (r + 1) * hl) for j in range(3)])
            conv_w = conv_w[r * hl:(r + 1) * hl]
        else:
            hl = hidden
        self.in_proj = ReplicatedLinear(in_proj)   # this rank's [B | C | x] channels (packed weights stay packed)
        self.conv_w = conv_w.float().contiguous()
        self.out_proj = RowParallelLinear(out_proj)
        self.H = hl
        self.L = conv_w.shape[1]
        self.layer = layer
        self.state = None
        self.state_off = 0
        self.decode_cu = None

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        ctx = get_context()
        proj = self.in_proj(x)
        if ctx.is_prefill:
            cu = ctx.cu_seqlens_q
        else:
            n = ctx.num_seqs
            if self.decode_cu is None or self.decode_cu.numel() < n + 1 or self.decode_cu.device != proj.device:
                self.decode_cu = torch.arange(0, 1024 + 1, dtype=torch.int32, device=proj.device)
            cu = self.decode_cu[:n + 1]
        y = ops.shortconv(proj, self.conv_w, cu, ctx.state_rows, ctx.state_fresh, self.state, self.state_off)
        return self.out_proj(y)


class _L:
    pass


class Lfm2ForCausalLM(CausalLMBase):
    def __init__(self, hf: HfConfig, weights, device, dtype=torch.bfloat16, max_pos: int = None):
        self.hf = hf
        bag = WeightBag(weights, device, dtype)
        H, hd, eps = hf.hidden_size, hf.head_dim, hf.rms_norm_eps
        self.rope = RotaryTables(max_pos or hf.max_position_embeddings, device)
        emb = bag.require("token_embd.weight")
        self.embed = VocabParallelEmbedding(emb)
        self.layers = []
        self.conv_layers = []
        for i in range(hf.num_hidden_layers):
            p = f"blk.{i}."
            L = _L()
            L.op_norm = RMSNorm(bag.require(p + "attn_norm.weight"), eps)
            L.ffn_norm = RMSNorm(bag.require(p + "ffn_norm.weight"), eps)
            L.gate_up = MergedColumnParallelLinear(bag.require(p + "ffn_gate.weight"), bag.require(p + "ffn_up.weight"),
                                                   ops.ACT_SILU_MUL)
            L.down = RowParallelLinear(bag.require(p + "ffn_down.weight"))
            L.is_conv = hf.is_conv_layer(i)
            if L.is_conv:
                L.conv = ShortConv(bag.require(p + "shortconv.in_proj.weight"),
                                   bag.require(p + "shortconv.conv.weight"),
                                   bag.require(p + "shortconv.out_proj.weight"), H, i)
                self.conv_layers.append(L.conv)
            else:
                nkv = hf.layer_kv_heads[i] if hf.layer_kv_heads else hf.num_key_value_heads
                L.qkv = QKVParallelLinear(bag.require(p + "attn_q.weight"), bag.require(p + "attn_k.weight"),
                                          bag.require(p + "attn_v.weight"), hf.num_attention_heads, nkv, hd)
                L.attn = Attention(L.qkv.nq, L.qkv.nkv, hd, hf.attention_scale(), self.rope.get(hd, hf.rope_theta),
                                   bag.require(p + "attn_q_norm.weight"), bag.require(p + "attn_k_norm.weight"), 0, eps)
                L.o_proj = RowParallelLinear(bag.require(p + "attn_output.weight"))
            self.layers.append(L)
        self.out_norm = RMSNorm(bag.require("token_embd_norm.weight"), eps)
        head = bag.find("output.weight")
        self.lm_head = ParallelLMHead(head if head is not None else emb, hf.vocab_size)

    def kv_specs(self):
        return [(i, L.attn.nkv, L.attn.hd) for i, L in enumerate(self.layers) if not L.is_conv]

    def bind_kv(self, caches):
        for i, L in enumerate(self.layers):
            if not L.is_conv:
                L.attn.bind_cache(*caches[i])

    def state_specs(self):
        return [(L.layer, (L.L - 1) * L.H) for L in self.conv_layers]

    def bind_state(self, arena):
        off = 0
        for c in self.conv_layers:
            c.state = arena
            c.state_off = off
            off += (c.L - 1) * c.H

    def forward(self, ids, positions):
        h = self.embed(ids)
        residual = None
        for L in self.layers:
            if residual is None:
                residual = h
                x, _ = L.op_norm(h)
            else:
                x, residual = L.op_norm(h, residual)
            if L.is_conv:
                y = L.conv(x)
            else:
                y = L.o_proj(L.attn(L.qkv(x), positions))
            x, residual = L.ffn_norm(y, residual)
            h = L.down(L.gate_up(x))
        out, _ = self.out_norm(h, residual)
        return out

    def compute_logits(self, hidden):
        return self.lm_head(hidden)
