"""BERT sentence-embedding encoder (GGUF tensor names; ONNX names are mapped onto them at load).

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/internal/BertForEmbedding.java:31-214 --
token + position + token-type(0) embeddings -> LayerNorm -> N post-LN blocks [biased q/k/v -> bidirectional MHA
-> o -> LN(x + attn) -> GELU(tanh) FFN -> LN(x + ffn)] -> masked mean pool -> L2 normalise.  The reference
encodes one text at a time; here a whole batch of variable-length sequences is packed into one [T, H] tensor
(cu_seqlens) and run through the varlen bidirectional attention kernel; ``parallel/dp.py`` spreads a batch
data-parallel over GPUs (one replica per rank, token-balanced shares, one all-gather of the embeddings).
"""
from __future__ import annotations

import itertools
from typing import Dict, List, Tuple

import numpy as np
import torch

from .. import ops
from ..config import HfConfig
from ..layers.attention import BidirectionalAttention
from .base import WeightBag, random_weights


def param_shapes(hf: HfConfig) -> List[Tuple[str, tuple]]:
    H, I = hf.hidden_size, hf.intermediate_size
    out = [("token_embd.weight", (hf.vocab_size, H)), ("position_embd.weight", (hf.max_position_embeddings, H)),
           ("token_types.weight", (hf.type_vocab_size, H)), ("token_embd_norm.weight", (H,)),
           ("token_embd_norm.bias", (H,))]
    for i in range(hf.num_hidden_layers):
        p = f"blk.{i}."
        for n in ("attn_q", "attn_k", "attn_v", "attn_output"):
            out += [(p + n + ".weight", (H, H)), (p + n + ".bias", (H,))]
        out += [(p + "attn_output_norm.weight", (H,)), (p + "attn_output_norm.bias", (H,)),
                (p + "ffn_up.weight", (I, H)), (p + "ffn_up.bias", (I,)), (p + "ffn_down.weight", (H, I)),
                (p + "ffn_down.bias", (H,)), (p + "layer_output_norm.weight", (H,)),
                (p + "layer_output_norm.bias", (H,))]
    return out


def init_random(hf: HfConfig, seed: int, device="cpu") -> Dict[str, torch.Tensor]:
    w = random_weights(param_shapes(hf), seed, device, ones_for=lambda n: n.endswith("norm.weight"))
    for k in list(w):
        if k.endswith(".bias"):
            w[k] = torch.zeros_like(w[k])
    return w


class _L:
    pass


class BertEncoder:
    def __init__(self, hf: HfConfig, weights, device, dtype=torch.bfloat16):
        self.hf = hf
        self.device = device
        bag = WeightBag(weights, device, dtype)
        H = hf.hidden_size
        self.nh = hf.num_attention_heads
        self.hd = H // self.nh
        self.eps = hf.layer_norm_eps
        self.tok = bag.dense("token_embd.weight")
        self.pos = bag.dense("position_embd.weight")
        types = bag.find("token_types.weight")
        self.type0 = types[0:1] if types is not None else None
        self.emb_ln = (bag.require("token_embd_norm.weight"), bag.require("token_embd_norm.bias"))
        self.layers = []
        for i in range(hf.num_hidden_layers):
            p = f"blk.{i}."
            L = _L()
            L.wqkv = torch.cat([bag.dense(p + "attn_q.weight"), bag.dense(p + "attn_k.weight"),
                                bag.dense(p + "attn_v.weight")], 0).contiguous()
            L.bqkv = torch.cat([bag.require(p + "attn_q.bias"), bag.require(p + "attn_k.bias"),
                                bag.require(p + "attn_v.bias")], 0).contiguous()
            L.wo, L.bo = bag.dense(p + "attn_output.weight"), bag.require(p + "attn_output.bias")
            L.ln1 = (bag.require(p + "attn_output_norm.weight"), bag.require(p + "attn_output_norm.bias"))
            L.wup, L.bup = bag.dense(p + "ffn_up.weight"), bag.require(p + "ffn_up.bias")
            L.wdown, L.bdown = bag.dense(p + "ffn_down.weight"), bag.require(p + "ffn_down.bias")
            L.ln2 = (bag.require(p + "layer_output_norm.weight"), bag.require(p + "layer_output_norm.bias"))
            L.attn = BidirectionalAttention(self.nh, self.hd, self.hd ** -0.5)
            self.layers.append(L)

    @torch.inference_mode()
    def encode_packed(self, ids: torch.Tensor, positions: torch.Tensor, cu: torch.Tensor, max_len: int) -> torch.Tensor:
        x = ops.embedding(self.tok, ids)
        pos = ops.embedding(self.pos, positions)
        x = ops.layer_norm(x, *self.emb_ln, self.eps, residual=self._add_type(pos, x.shape[0]))
        for L in self.layers:
            qkv = ops.linear(x, L.wqkv)
            ops.bias_act_(qkv, L.bqkv)
            a = L.attn(qkv, cu, max_len)
            a = ops.linear(a, L.wo)
            ops.bias_act_(a, L.bo)
            x = ops.layer_norm(a, *L.ln1, self.eps, residual=x)
            f = ops.linear(x, L.wup)
            ops.bias_act_(f, L.bup, ops.BIAS_ACT_GELU_TANH)
            f = ops.linear(f, L.wdown)
            ops.bias_act_(f, L.bdown)
            x = ops.layer_norm(f, *L.ln2, self.eps, residual=x)
        return ops.mean_pool_l2(x, cu)

    def _add_type(self, pos: torch.Tensor, n: int) -> torch.Tensor:
        if self.type0 is None:
            return pos
        return (pos.float() + self.type0.float()).to(pos.dtype)

    def embed_ids(self, batch: List[List[int]], max_tokens: int = 65536, keep_device: bool = False) -> torch.Tensor:
        """Mean-pooled, L2-normalised embeddings [N, H] (fp32) for token-id sequences, packed in chunks
        (returned on the encoder's device with ``keep_device``, else on the host)."""
        outs = []
        i = 0
        while i < len(batch):
            j = i
            tokens = 0
            while j < len(batch) and (tokens + len(batch[j]) <= max_tokens or j == i):
                tokens += len(batch[j])
                j += 1
            chunk = batch[i:j]
            # flat ids, positions and cu_seqlens built in numpy (a Python list per token cost ~5x more host time
            # than the encoder pass leaves per chunk)
            lens = np.fromiter((len(s) for s in chunk), dtype=np.int64, count=len(chunk))
            cu_np = np.zeros(len(chunk) + 1, dtype=np.int64)
            np.cumsum(lens, out=cu_np[1:])
            T = int(cu_np[-1])
            ids = torch.from_numpy(np.fromiter(itertools.chain.from_iterable(chunk), dtype=np.int64, count=T))
            pos = torch.from_numpy(np.arange(T, dtype=np.int64) - np.repeat(cu_np[:-1], lens))
            cu = torch.from_numpy(cu_np.astype(np.int32))
            ids, pos, cu = (t.to(self.device) for t in (ids, pos, cu))
            e = self.encode_packed(ids, pos, cu, int(lens.max())).float()
            outs.append(e if keep_device else e.cpu())
            i = j
        return torch.cat(outs, 0)
