"""Gemma4 QAT (quantization-aware-trained mobile) checkpoints: packed int2 / int4 / int8 weights.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/models/llmarch/Gemma4QatLoader.java:33-297 and
models/internal/{GemmaQat.java:14-138, GemmaQatWeight.java:26-133}.

Checkpoint layout (a Hugging Face folder of safetensors shards):
* language tensors under ``model.language_model.*`` (canonicalised to ``model.*``); vision / audio towers and
  their embedders, and ``k_cache_scale`` / ``v_cache_scale``, are skipped;
* a packed module is ``<m>.weight`` (U8 for 2/4-bit, I8 for 8-bit) or ``<m>.embedding_quantized``, with
  ``<m>.weight_scale`` / ``<m>.embedding_scale`` [rows, scale_cols] and optional scalar
  ``<m>.input_activation_scale`` / ``<m>.output_activation_scale`` (static-range activation quantisation);
* bits: I8 -> 8; the token embedding and the LM head -> 2; MLPs of KV-shared layers -> 2; everything else -> 4;
  unpacked width = packed width * 8 / bits;
* 4-bit: low nibble first, value = nibble - 8; 2-bit: crumbs low to high, value = crumb - 2; then value *=
  scale[row, col // (cols / scale_cols)].

Here a packed module stays packed (``QatWeight``) until the model graph asks for it on its device, where the
unpack + scale runs as a handful of vectorised tensor ops.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Dict, Optional

import torch

from ..config import HfConfig
from ..exceptions import ModelLoadException
from .safetensors import SafetensorsCheckpoint

LANGUAGE_PREFIX = "model.language_model."
_SKIP = ("vision_tower", "audio_tower", "embed_vision", "embed_audio")


def packed_width(cols: int, bits: int) -> int:
    if bits == 2:
        return (cols + 3) // 4
    if bits == 4:
        return (cols + 1) // 2
    if bits == 8:
        return cols
    raise ValueError(f"unsupported QAT bit width: {bits}")


def infer_bits_from_width(pw: int, cols: int) -> int:
    if pw == cols:
        return 8
    if pw == (cols + 1) // 2:
        return 4
    if pw == (cols + 3) // 4:
        return 2
    raise ValueError(f"cannot infer QAT bits from packed width {pw} and {cols} columns")


@dataclass
class QatWeight:
    name: str
    packed: torch.Tensor        # uint8 [rows, packed_width] (2/4-bit) or int8 [rows, cols] (8-bit)
    scales: torch.Tensor        # fp32 [rows, scale_cols]
    rows: int
    cols: int
    bits: int
    scale_cols: int
    in_scale: float = 0.0
    out_scale: float = 0.0

    def __post_init__(self):
        if self.rows <= 0 or self.cols <= 0:
            raise ValueError("QAT weight shape must be positive")
        if self.packed.numel() != self.rows * packed_width(self.cols, self.bits):
            raise ValueError(f"{self.name}: packed bytes {self.packed.numel()} != rows {self.rows} x "
                             f"packed width {packed_width(self.cols, self.bits)}")
        if self.scale_cols <= 0 or self.cols % self.scale_cols:
            raise ValueError(f"{self.name}: scale_cols {self.scale_cols} does not divide cols {self.cols}")
        if self.scales.numel() != self.rows * self.scale_cols:
            raise ValueError(f"{self.name}: scale count {self.scales.numel()} != rows x scale_cols")

    @property
    def shape(self):
        return (self.rows, self.cols)

    def to_device(self, device) -> "QatWeight":
        return QatWeight(self.name, self.packed.to(device), self.scales.to(device), self.rows, self.cols, self.bits,
                         self.scale_cols, self.in_scale, self.out_scale)

    def unpack(self) -> torch.Tensor:
        """Integer values as fp32 [rows, cols] (before scaling)."""
        p = self.packed.reshape(self.rows, -1)
        if self.bits == 8:
            return p.view(torch.int8).float()[:, :self.cols]
        b = p.to(torch.int16)
        if self.bits == 4:
            v = torch.stack([(b & 0xF) - 8, (b >> 4) - 8], dim=-1)
        else:
            v = torch.stack([(b & 3) - 2, ((b >> 2) & 3) - 2, ((b >> 4) & 3) - 2, (b >> 6) - 2], dim=-1)
        return v.reshape(self.rows, -1)[:, :self.cols].float()

    def dequantize(self, dtype=torch.bfloat16) -> torch.Tensor:
        block = self.cols // self.scale_cols
        s = self.scales.reshape(self.rows, self.scale_cols).float().repeat_interleave(block, dim=1)
        return (self.unpack() * s).to(dtype)

    def to_gguf_blocks(self):
        """The same integers as GGUF blocks the dequant-fused GEMM multiplies in place: int4 and int2 codes as
        Q4_0 (value = nibble - 8; 2-bit codes ride in the 4-bit container), int8 as Q8_0.  Every 32-element
        block takes its (row, column block) scale rounded to fp16 -- the only change to the values: a relative
        error of at most 2^-11 on each scale, finer than the bf16 rounding of every weight that expanding to
        bf16 would cost.  None when the layout cannot be expressed (scale blocks not a multiple of 32 columns,
        or a width the fused kernel does not take)."""
        from ..ops.quant import STEP, GgufPacked
        block = self.cols // self.scale_cols
        if block % 32 or self.cols % STEP:
            return None
        q = self.unpack().to(torch.int16)                                      # [rows, cols]
        s32 = self.scales.reshape(self.rows, self.scale_cols).float().repeat_interleave(block // 32, dim=1)
        d = s32.to(torch.float16).contiguous().view(torch.uint8).reshape(self.rows, -1, 2)
        nblk = self.cols // 32
        if self.bits == 8:
            codes = q.to(torch.int8).reshape(self.rows, nblk, 32).view(torch.uint8)
            blocks, t = torch.cat([d, codes], -1), 8                           # Q8_0: d | 32 x int8
        else:
            u = (q + 8).to(torch.uint8).reshape(self.rows, nblk, 32)
            codes = u[..., :16] | (u[..., 16:] << 4)                           # Q4_0: element i low, i + 16 high
            blocks, t = torch.cat([d, codes], -1), 2
        return GgufPacked(blocks.reshape(-1).contiguous(), t, self.rows, self.cols)

    def dequantize_row(self, r: int) -> torch.Tensor:
        one = QatWeight(self.name, self.packed.reshape(self.rows, -1)[r:r + 1].contiguous(),
                        self.scales.reshape(self.rows, -1)[r:r + 1].contiguous(), 1, self.cols, self.bits,
                        self.scale_cols)
        return one.dequantize(torch.float32)[0]


def quantize(name: str, w: torch.Tensor, bits: int, scale_cols: int, in_scale: float = 0.0,
             out_scale: float = 0.0) -> QatWeight:
    """Symmetric per-(row, column block) quantisation to the QAT layout (for tests and checkpoint writers)."""
    rows, cols = w.shape
    block = cols // scale_cols
    qmax = {2: 1, 4: 7, 8: 127}[bits]
    qmin = {2: -2, 4: -8, 8: -128}[bits]
    wf = w.float().reshape(rows, scale_cols, block)
    s = (wf.abs().amax(-1) / qmax).clamp_min(1e-8)
    q = torch.round(wf / s[..., None]).clamp(qmin, qmax).reshape(rows, cols).to(torch.int16)
    if bits == 8:
        packed = q.to(torch.int8)
    else:
        per = 8 // bits
        pad = (-cols) % per
        if pad:
            q = torch.cat([q, torch.zeros(rows, pad, dtype=torch.int16)], 1)
        u = (q - qmin).reshape(rows, -1, per)
        packed = torch.zeros(u.shape[:2], dtype=torch.int16)
        for i in range(per):
            packed |= u[..., i] << (bits * i)
        packed = packed.to(torch.uint8)
    return QatWeight(name, packed.contiguous(), s.contiguous(), rows, cols, bits, scale_cols, in_scale, out_scale)


def _layer_index(param: str) -> Optional[int]:
    m = "model.layers."
    i = param.find(m)
    if i < 0:
        return None
    j = param.find(".", i + len(m))
    try:
        return int(param[i + len(m):j])
    except ValueError:
        return None


def infer_bits(param: str, dtype: str, hf: HfConfig) -> int:
    if dtype == "I8":
        return 8
    if "lm_head" in param or ("embed_tokens.weight" in param and "per_layer" not in param):
        return 2
    li = _layer_index(param)
    if li is not None and ".mlp." in param and hf.is_kv_shared_layer(li):
        return 2
    return 4


def canonical(raw: str) -> str:
    return "model." + raw[len(LANGUAGE_PREFIX):] if raw.startswith(LANGUAGE_PREFIX) else raw


def _role(name: str, dtype: str):
    for suffix, role in ((".embedding_quantized", "quant"), (".embedding_scale", "scale"), (".weight_scale", "scale"),
                         (".input_activation_scale", "in"), (".output_activation_scale", "out")):
        if name.endswith(suffix):
            return role, name[:-len(suffix)] + ".weight"
    if name.endswith(".weight") and dtype in ("U8", "I8"):
        return "quant", name
    return None, name


def load_gemma4_qat(path: str, hf: HfConfig) -> Dict[str, object]:
    ck = SafetensorsCheckpoint(path)
    dense: Dict[str, torch.Tensor] = {}
    modules: Dict[str, Dict[str, str]] = {}
    for raw in ck.keys():
        if any(s in raw for s in _SKIP) or raw.endswith("k_cache_scale") or raw.endswith("v_cache_scale"):
            continue
        name = canonical(raw)
        role, param = _role(name, ck.dtype_name(raw))
        if role is None:
            dense[name] = ck.get(raw)
        else:
            modules.setdefault(param, {})[role] = raw
    if not dense and not modules:
        raise ModelLoadException(f"no Gemma 4 language tensors in {path}")
    out: Dict[str, object] = dict(dense)
    for param, parts in modules.items():
        if "quant" not in parts or "scale" not in parts:
            raise ModelLoadException(f"QAT module {param} lacks its packed payload or scale")
        q = parts["quant"]
        shape = ck.shape(q)
        bits = infer_bits(param, ck.dtype_name(q), hf)
        rows, pw = shape[0], shape[-1]
        cols = pw if bits == 8 else pw * (8 // bits)
        sc = ck.get(parts["scale"]).float()
        scale_cols = sc.shape[-1] if sc.dim() >= 2 else 1
        scalar = lambda role: float(ck.get(parts[role]).float().reshape(-1)[0]) if role in parts else 0.0  # noqa
        payload = ck.get(q)
        payload = payload.view(torch.int8) if bits == 8 and payload.dtype == torch.uint8 else payload
        out[param] = QatWeight(param, payload.reshape(rows, pw), sc.reshape(rows, scale_cols), rows, cols, bits,
                               scale_cols, scalar("in"), scalar("out"))
    if "lm_head.weight" not in out and "model.embed_tokens.weight" in out:
        out["lm_head.weight"] = out["model.embed_tokens.weight"]
    return out


def write_gemma4_qat_folder(path: str, hf: HfConfig, weights: Dict[str, torch.Tensor], scale_cols: int = 1,
                            srq: Optional[Dict[str, tuple]] = None, tokenizer_json: Optional[dict] = None) -> str:
    """Quantise dense weights into a QAT checkpoint folder (packed linears/embeddings, dense norms / scalars /
    the PLE model projection), under the ``model.language_model.`` prefix like the published checkpoints."""
    import json
    from .safetensors import save_file
    os.makedirs(path, exist_ok=True)
    tensors = {}
    for name, w in weights.items():
        packed = (w.dim() == 2 and name.endswith(".weight") and "norm" not in name
                  and "per_layer_model_projection" not in name)
        raw = LANGUAGE_PREFIX + name[len("model."):] if name.startswith("model.") else name
        if not packed:
            tensors[raw] = w.contiguous()
            continue
        bits = infer_bits(name, "U8", hf)
        sc = scale_cols if w.shape[1] % scale_cols == 0 else 1
        qw = quantize(name, w, bits, sc)
        base = raw[:-len(".weight")]
        if "embed_tokens" in name:
            tensors[base + ".embedding_quantized"] = qw.packed
            tensors[base + ".embedding_scale"] = qw.scales
        else:
            tensors[raw] = qw.packed
            tensors[base + ".weight_scale"] = qw.scales
        if srq and name in srq:
            tensors[base + ".input_activation_scale"] = torch.tensor([srq[name][0]], dtype=torch.float32)
            tensors[base + ".output_activation_scale"] = torch.tensor([srq[name][1]], dtype=torch.float32)
    save_file(tensors, os.path.join(path, "model.safetensors"))
    cfg = hf.to_dict()
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f)
    if tokenizer_json is not None:
        with open(os.path.join(path, "tokenizer.json"), "w") as f:
            json.dump(tokenizer_json, f)
    return path
