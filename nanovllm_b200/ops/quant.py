"""GGUF weights kept in their block format on the GPU, multiplied by the dequant-fused GEMM (csrc/qgemm.cu).

The reference multiplies quantized tensors by decoding GGML blocks inside its CPU matmul loops
(nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/internal/GgufDequant.java:15-90).  ``GgufPacked``
holds a 2-D weight [N, K] as its raw GGUF rows ([N, K / block * block_bytes] uint8) so the linear layers can
shard (rows, or K at 256-element boundaries), concatenate and permute it exactly like a dense tensor; the first
GPU multiply repacks it once into the kernel's tile-major layout (a lossless byte permutation, see
``repack_tiles``).  Decode-sized batches (M <= 256) run the fused kernel on the packed bytes; larger ones
dequantize into a bf16 scratch and use the tensor-core GEMM; CPU tensors fall back to the torch decoders.
"""
from __future__ import annotations

import math
from typing import List, Optional, Sequence

import torch

from ..loaders import dequant as DQ

# types the fused kernel decodes, with the bytes of one 256-element row step in the repacked layout
FUSED_TYPES = {2: 144, 3: 160, 6: 176, 7: 192, 8: 272, 10: 96, 11: 112, 12: 144, 13: 176, 14: 224, 20: 144, 23: 144,
               34: 64, 35: 80, 39: 144, 40: 144}
STEP = 256
TILE_ROWS = 128


def fused_supported(ggml_type: int, shape: Sequence[int]) -> bool:
    return ggml_type in FUSED_TYPES and len(shape) == 2 and shape[1] % STEP == 0


def _pair_adjacent(qs: torch.Tensor, groups: int) -> torch.Tensor:
    """FP4 code bytes of one block [..., nbytes] from GGUF order (per group of 2g codes: byte u holds codes u and
    u + g) to pair-adjacent order (byte t holds codes 2t and 2t + 1, low nibble first): the order in which the
    hardware e2m1x2 -> f16x2 conversion produces adjacent elements."""
    shp = qs.shape
    g = qs.reshape(*shp[:-1], groups, shp[-1] // groups)
    codes = torch.cat([g & 0xF, g >> 4], -1).reshape(*shp[:-1], 2 * shp[-1])  # block element order
    pairs = codes.reshape(*shp[:-1], shp[-1], 2)
    return (pairs[..., 0] | (pairs[..., 1] << 4)).to(torch.uint8)


def repack_tiles(raw: torch.Tensor, ggml_type: int, N: int, K: int) -> torch.Tensor:
    """Raw GGUF rows [N, row_bytes] -> flat uint8 [ceil(N/128), K/256, 128, bprs]: per 256-element row step the
    block fields are regrouped structure-of-arrays (scales, then quant bytes) and padded to 16-byte multiples;
    rows past N are zero (they decode to 0)."""
    be, bb = DQ.block_info(ggml_type)
    S = K // STEP
    nb = STEP // be
    B = raw.reshape(N, S, nb, bb)
    dev = raw.device

    def z(n):
        return torch.zeros(N, S, n, dtype=torch.uint8, device=dev)

    def f(a, b):  # field bytes [a, b) of every block of the step, concatenated block by block
        return B[..., a:b].reshape(N, S, nb * (b - a))

    t = ggml_type
    if t in (2, 20):                       # Q4_0 / IQ4_NL: d[8] | qs[8][16]
        step = torch.cat([f(0, 2), f(2, 18)], -1)
    elif t == 3:                           # Q4_1: d[8] | m[8] | qs[8][16]
        step = torch.cat([f(0, 2), f(2, 4), f(4, 20)], -1)
    elif t == 6:                           # Q5_0: d[8] | qh[8] (u32) | qs[8][16]
        step = torch.cat([f(0, 2), f(2, 6), f(6, 22)], -1)
    elif t == 7:                           # Q5_1: d[8] | m[8] | qh[8] (u32) | qs[8][16]
        step = torch.cat([f(0, 2), f(2, 4), f(4, 8), f(8, 24)], -1)
    elif t == 8:                           # Q8_0: d[8] | qs[8][32]
        step = torch.cat([f(0, 2), f(2, 34)], -1)
    elif t in (10, 11, 34, 35):            # Q2_K / Q3_K / TQ1_0 / TQ2_0: one super-block, zero-padded to 16 B
        step = torch.cat([B.reshape(N, S, bb), z(FUSED_TYPES[t] - bb)], -1)
    elif t == 39:                          # MXFP4: e[8] | pad 8 | qs[8][16] (pair-adjacent codes)
        step = torch.cat([f(0, 1), z(8), _pair_adjacent(B[..., 1:17], 1).reshape(N, S, 128)], -1)
    elif t == 40:                          # NVFP4 (4 blocks of 64): scales[4][4] | qs[4][32] (pair-adjacent codes)
        step = torch.cat([f(0, 4), _pair_adjacent(B[..., 4:36], 4).reshape(N, S, 128)], -1)
    elif t in (12, 13):                    # Q4_K / Q5_K: one super-block, already grouped
        step = B.reshape(N, S, bb)
    elif t == 14:                          # Q6_K: ql | qh | scales | d, padded 210 -> 224
        step = torch.cat([B.reshape(N, S, bb), z(14)], -1)
    elif t == 23:                          # IQ4_XS: d | scales_h | scales_l | pad 8 | qs[8][16]
        step = torch.cat([B[..., 0:8].reshape(N, S, 8), z(8), B[..., 8:136].reshape(N, S, 128)], -1)
    else:
        raise ValueError(f"no fused layout for GGML type {t}")
    bprs = FUSED_TYPES[t]
    assert step.shape[-1] == bprs, (t, step.shape)
    tiles = (N + TILE_ROWS - 1) // TILE_ROWS
    if tiles * TILE_ROWS != N:
        step = torch.cat([step, torch.zeros(tiles * TILE_ROWS - N, S, bprs, dtype=torch.uint8, device=dev)], 0)
    return step.reshape(tiles, TILE_ROWS, S, bprs).permute(0, 2, 1, 3).contiguous().reshape(-1)


class GgufPacked:
    """A [N, K] GGUF weight in block format (rows independent, K in whole blocks)."""

    is_packed = True

    def __init__(self, raw: torch.Tensor, ggml_type: int, N: int, K: int):
        be, bb = DQ.block_info(ggml_type)
        assert K % be == 0 and raw.dtype == torch.uint8 and raw.numel() == N * (K // be) * bb
        self.raw = raw.reshape(N, (K // be) * bb)
        self.ggml_type = int(ggml_type)
        self.N, self.K = int(N), int(K)
        self._tiles: Optional[torch.Tensor] = None

    # ---------------------------------------------------------------- tensor-like surface
    @property
    def shape(self):
        return torch.Size([self.N, self.K])

    @property
    def dtype(self):
        return torch.bfloat16

    @property
    def device(self):
        return (self.raw if self.raw is not None else self._tiles).device

    def dim(self) -> int:
        return 2

    def contiguous(self) -> "GgufPacked":
        return self

    def to_device(self, device) -> "GgufPacked":
        if self.device == torch.device(device):
            return self
        return GgufPacked(self._need_raw().to(device), self.ggml_type, self.N, self.K)

    def dequantize(self, dtype=torch.bfloat16) -> torch.Tensor:
        if self.raw is None:
            return self.dense_cuda().to(dtype)
        flat = self.raw.reshape(-1)
        return DQ.dequantize(flat, self.ggml_type, self.N * self.K, device=flat.device,
                             dtype=torch.float32).reshape(self.N, self.K).to(dtype)

    # ---------------------------------------------------------------- sharding (row-parallel splits K)
    def rows(self, a: int, b: int) -> "GgufPacked":
        return GgufPacked(self._need_raw()[a:b].clone(), self.ggml_type, b - a, self.K)  # a copy, not a view

    def cols(self, a: int, b: int) -> "GgufPacked":
        be, bb = DQ.block_info(self.ggml_type)
        if a % STEP or b % STEP:
            raise ValueError(f"packed K slice [{a}, {b}) must fall on 256-element boundaries")
        return GgufPacked(self._need_raw()[:, a // be * bb:b // be * bb].contiguous(), self.ggml_type, self.N, b - a)

    def permute_rows(self, index: torch.Tensor) -> "GgufPacked":
        raw = self._need_raw()
        return GgufPacked(raw[index.to(raw.device)], self.ggml_type, self.N, self.K)

    @staticmethod
    def cat_rows(parts: List["GgufPacked"]) -> "GgufPacked":
        t = parts[0].ggml_type
        if any(p.ggml_type != t or p.K != parts[0].K for p in parts):
            raise ValueError("cannot concatenate packed weights of different types / widths")
        return GgufPacked(torch.cat([p._need_raw() for p in parts], 0), t, sum(p.N for p in parts), parts[0].K)

    # ---------------------------------------------------------------- multiply
    def tiles(self) -> torch.Tensor:
        """The tile-major copy the kernels read.  On the GPU the raw rows are dropped once it exists (sharding
        and concatenation happen at layer construction, before the first multiply)."""
        if self._tiles is None:
            if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
                raise RuntimeError("packed weight must be repacked before CUDA graph capture")
            self._tiles = repack_tiles(self.raw, self.ggml_type, self.N, self.K)
            if self._tiles.is_cuda:
                self.raw = None
        return self._tiles

    def _need_raw(self) -> torch.Tensor:
        if self.raw is None:
            raise RuntimeError("packed weight was already repacked for the GPU kernels; shard it before use")
        return self.raw

    def dense_cuda(self) -> torch.Tensor:
        from . import _cuda_ext, add_launches
        out = torch.empty(self.N, self.K, dtype=torch.bfloat16, device=self.device)
        _cuda_ext().qdequant(self.tiles(), self.ggml_type, self.N, self.K, out)
        add_launches(1)
        return out

    def linear(self, x: torch.Tensor, out: Optional[torch.Tensor] = None, partial_ok: bool = False):
        """x [M, K] @ W^T.  Decode-sized M on CUDA runs the fused kernel; ``partial_ok`` may return the
        unreduced split-K partials as a ``SplitK`` for a consumer that sums them."""
        from . import SplitK, _cuda_ext, add_launches, error_word, library_gemm, linear as dense_linear, materialize
        from . import reference_cpu as ref
        x = materialize(x)
        if not x.is_cuda:
            y = ref.linear(x, self.dequantize(torch.float32).to(x.dtype), 0)
            if out is not None:
                out.copy_(y)
                return out
            return y
        M = x.shape[0]
        if library_gemm() or M > 256:
            w = self.dense_cuda()
            return torch.matmul(x, w.t(), out=out) if library_gemm() else dense_linear(x, w, out=out)
        C = _cuda_ext()
        S = C.qgemm_splits(M, self.N, self.K, self.ggml_type)
        parts = torch.empty(S, M, self.N, dtype=torch.float32, device=x.device) if S > 1 else None
        if out is None:
            out = torch.empty(M, self.N, dtype=torch.bfloat16, device=x.device)
        C.qgemm(x, self.tiles(), self.ggml_type, self.N, self.K, out, parts, error_word(x.device),
                bool(partial_ok and parts is not None))
        if parts is not None and partial_ok:
            add_launches(1)
            return SplitK(parts)
        add_launches(2 if parts is not None else 1)
        return out

    def __repr__(self) -> str:
        return f"GgufPacked({DQ.type_name(self.ggml_type)}, [{self.N}, {self.K}], {self.device})"


def is_packed(w) -> bool:
    return getattr(w, "is_packed", False)


def shard_rows(w, rank: int, size: int):
    """Column-parallel row shard; a dense shard is a copy, so the full tensor is freed once the loader drops it
    (a row slice is a view that would keep all TP shards alive on every rank)."""
    n = w.shape[0]
    assert n % size == 0, f"dimension {n} not divisible by TP={size}"
    k = n // size
    return w.rows(rank * k, (rank + 1) * k) if is_packed(w) else w[rank * k:(rank + 1) * k].clone()


def shard_cols(w, rank: int, size: int):
    """Row-parallel K shard.  A packed weight stays packed when the shard falls on 256-element boundaries; a
    shard that would cut GGML super-blocks (e.g. LFM2's ffn_down K 10752 over TP 4 or 8) is expanded to bf16."""
    n = w.shape[1]
    assert n % size == 0, f"dimension {n} not divisible by TP={size}"
    k = n // size
    if is_packed(w):
        if k % STEP == 0:
            return w.cols(rank * k, (rank + 1) * k)
        w = w.dequantize(torch.bfloat16)
    return w[:, rank * k:(rank + 1) * k]


def cat_rows(parts):
    if any(is_packed(p) for p in parts):
        if not all(is_packed(p) for p in parts):
            raise ValueError("cannot mix packed and dense weights in one projection")
        return GgufPacked.cat_rows(list(parts))
    return torch.cat(list(parts), 0)


def _f16_bytes(v: float, device) -> torch.Tensor:
    return torch.tensor([v], dtype=torch.float16).view(torch.uint8).to(device)


def random_packed(ggml_type: int, N: int, K: int, seed: int, device, std: float = 0.02) -> GgufPacked:
    """Random blocks generated on ``device`` whose dequantized values spread like N(0, std) (random codes, block
    scales chosen for that spread): the random-init stand-in for a quantized checkpoint, without a file."""
    be, bb = DQ.block_info(ggml_type)
    nblk = N * K // be
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    raw = torch.randint(0, 256, (nblk, bb), dtype=torch.uint8, device=device, generator=g)
    t = ggml_type
    if t == 40:                                      # NVFP4: ue4m3 sub-scales 4 * 2^-10
        raw[:, 0:4] = 4
    elif t == 39:                                    # MXFP4: 2^(e - 128) times the doubled e2m1 grid
        raw[:, 0] = 128 + int(round(math.log2(std / 5.7)))
    elif t == 12:                                    # Q4_K: 6-bit scales / mins of 32, codes centred by dmin
        d = std / (32 * 4.6)
        raw[:, 0:2] = _f16_bytes(d, device)
        raw[:, 2:4] = _f16_bytes(d * 7.5, device)
        raw[:, 4:12] = 0xA0
        raw[:, 12:16] = 0
    elif t == 14:                                    # Q6_K: int8 scales 16, codes -32..31
        raw[:, 192:208] = 16
        raw[:, 208:210] = _f16_bytes(std / (16 * 18.5), device)
    elif t == 8:                                     # Q8_0
        raw[:, 0:2] = _f16_bytes(std / 74.0, device)
    elif t == 2:                                     # Q4_0
        raw[:, 0:2] = _f16_bytes(std / 4.6, device)
    else:
        raise ValueError(f"random packing not provided for {DQ.type_name(t)}")
    return GgufPacked(raw.reshape(-1), t, N, K)
