"""GGML block formats: type table and vectorised dequantisation in torch (CPU or GPU tensors).

Covers every type of the reference catalogue (nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/internal/
GgufDequant.java:15-90 and GgufIqDequant.java:28-420): floats / ints, legacy Q4_0 Q4_1 Q5_0 Q5_1 Q8_0 Q8_1, the
low-bit Q1_0 / Q2_0, K-quants Q2_K..Q8_K, IQ1_S IQ1_M IQ2_XXS IQ2_XS IQ2_S IQ3_XXS IQ3_S IQ4_NL IQ4_XS, ternary
TQ1_0 / TQ2_0, and the FP4 block formats MXFP4 (e8m0 scale / 32) and NVFP4 (4 ue4m3 sub-scales / 64).

Instead of a per-element loop, each function views the packed bytes as a [blocks, block_bytes] uint8 tensor
and decodes all blocks at once with integer tensor ops, so the same code dequantises on the GPU at load time.
The IQ formats index ggml's published lattice grids; those tables are data that the format defines bit for bit,
so they are taken from the ``gguf`` package (ggml's own Python package) instead of being restated here.
"""
from __future__ import annotations

import math
from typing import Dict, Tuple

import numpy as np
import torch

# id -> (name, elements per block, bytes per block)
GGML_TYPES: Dict[int, Tuple[str, int, int]] = {
    0: ("F32", 1, 4), 1: ("F16", 1, 2), 2: ("Q4_0", 32, 18), 3: ("Q4_1", 32, 20), 6: ("Q5_0", 32, 22),
    7: ("Q5_1", 32, 24), 8: ("Q8_0", 32, 34), 9: ("Q8_1", 32, 36), 10: ("Q2_K", 256, 84), 11: ("Q3_K", 256, 110),
    12: ("Q4_K", 256, 144), 13: ("Q5_K", 256, 176), 14: ("Q6_K", 256, 210), 15: ("Q8_K", 256, 292),
    16: ("IQ2_XXS", 256, 66), 17: ("IQ2_XS", 256, 74), 18: ("IQ3_XXS", 256, 98), 19: ("IQ1_S", 256, 50),
    20: ("IQ4_NL", 32, 18), 21: ("IQ3_S", 256, 110), 22: ("IQ2_S", 256, 82), 23: ("IQ4_XS", 256, 136),
    24: ("I8", 1, 1), 25: ("I16", 1, 2), 26: ("I32", 1, 4), 27: ("I64", 1, 8), 28: ("F64", 1, 8),
    29: ("IQ1_M", 256, 56), 30: ("BF16", 1, 2), 34: ("TQ1_0", 256, 54), 35: ("TQ2_0", 256, 66),
    39: ("MXFP4", 32, 17), 40: ("NVFP4", 64, 36), 41: ("Q1_0", 128, 18), 42: ("Q2_0", 64, 18),
}
TYPE_BY_NAME = {v[0]: k for k, v in GGML_TYPES.items()}

KVALUES_IQ4NL = (-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113)
KVALUES_FP4 = (0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12)  # e2m1 grid doubled
IQ1_DELTA = 0.125


def type_name(t: int) -> str:
    return GGML_TYPES[t][0] if t in GGML_TYPES else f"type{t}"


def block_info(t: int) -> Tuple[int, int]:
    if t not in GGML_TYPES:
        raise ValueError(f"unsupported GGML type {t}")
    return GGML_TYPES[t][1], GGML_TYPES[t][2]


def packed_nbytes(t: int, numel: int) -> int:
    be, bb = block_info(t)
    if numel % be != 0:
        raise ValueError(f"{numel} elements is not a whole number of {type_name(t)} blocks")
    return numel // be * bb


# ----------------------------------------------------------------------------------------------- helpers
def _f16(b: torch.Tensor) -> torch.Tensor:
    """[..., 2] uint8 little-endian -> float32 [...]"""
    return b.contiguous().view(torch.float16).squeeze(-1).float()


def _u16(b: torch.Tensor) -> torch.Tensor:
    b = b.to(torch.int32)
    return b[..., 0] | (b[..., 1] << 8)


def _u32(b: torch.Tensor) -> torch.Tensor:
    b = b.to(torch.int64)
    return b[..., 0] | (b[..., 1] << 8) | (b[..., 2] << 16) | (b[..., 3] << 24)


def _lo_hi(q: torch.Tensor) -> torch.Tensor:
    """qs [..., n] bytes -> [..., 2n]: low nibbles (elements 0..n-1) then high nibbles (n..2n-1)."""
    q = q.to(torch.int32)
    return torch.cat([q & 0xF, q >> 4], dim=-1)


_GRIDS: Dict[str, torch.Tensor] = {}


def _grid(name: str, device) -> torch.Tensor:
    key = f"{name}:{device}"
    g = _GRIDS.get(key)
    if g is None:
        try:
            import gguf.quants as gq
        except ImportError as e:  # pragma: no cover - the package ships with the image
            raise RuntimeError("IQ lattice grids need the gguf package") from e
        cls = getattr(gq, name)
        cls.init_grid()
        g = torch.from_numpy(np.array(cls.grid, dtype=np.float32).reshape(cls.grid_shape)).to(device)
        _GRIDS[key] = g
    return g


def _ksigns(device) -> torch.Tensor:
    key = f"ksigns:{device}"
    g = _GRIDS.get(key)
    if g is None:
        import gguf.quants as gq
        g = torch.tensor(list(gq.IQ2_XXS.ksigns), dtype=torch.int32, device=device)
        _GRIDS[key] = g
    return g


def _sign_bits(byte: torch.Tensor, n: int = 8) -> torch.Tensor:
    """[...] int -> [..., n] of +1 / -1 from bit j."""
    bits = (byte.unsqueeze(-1) >> torch.arange(n, device=byte.device)) & 1
    return 1.0 - 2.0 * bits.float()


# ----------------------------------------------------------------------------------------------- legacy
def _q4_0(b):
    d = _f16(b[:, 0:2])
    return d[:, None] * (_lo_hi(b[:, 2:18]) - 8).float()


def _q4_1(b):
    d, m = _f16(b[:, 0:2]), _f16(b[:, 2:4])
    return d[:, None] * _lo_hi(b[:, 4:20]).float() + m[:, None]


def _q5(b, has_min):
    off = 4 if has_min else 2
    d = _f16(b[:, 0:2])
    qh = _u32(b[:, off:off + 4])
    qs = b[:, off + 4:off + 20].to(torch.int64)
    j = torch.arange(16, device=b.device)
    h0 = ((qh[:, None] >> j) & 1) << 4
    h1 = ((qh[:, None] >> (j + 16)) & 1) << 4
    x = torch.cat([(qs & 0xF) | h0, (qs >> 4) | h1], dim=-1).float()
    if has_min:
        return d[:, None] * x + _f16(b[:, 2:4])[:, None]
    return d[:, None] * (x - 16)


def _q8_0(b):
    return _f16(b[:, 0:2])[:, None] * b[:, 2:34].view(torch.int8).float()


def _q8_1(b):
    return _f16(b[:, 0:2])[:, None] * b[:, 4:36].view(torch.int8).float()


def _q1_0(b):
    d = _f16(b[:, 0:2])
    bits = (b[:, 2:18].to(torch.int32).unsqueeze(-1) >> torch.arange(8, device=b.device)) & 1
    return d[:, None] * (bits.reshape(b.shape[0], 128).float() * 2 - 1)


def _q2_0(b):
    d = _f16(b[:, 0:2])
    q = (b[:, 2:18].to(torch.int32).unsqueeze(-1) >> (2 * torch.arange(4, device=b.device))) & 3
    return d[:, None] * (q.reshape(b.shape[0], 64).float() - 1)


# ----------------------------------------------------------------------------------------------- K-quants
def _q2_k(b):
    n = b.shape[0]
    sc = b[:, 0:16].to(torch.int32)
    qs = b[:, 16:80].to(torch.int32).reshape(n, 2, 32)
    d, dmin = _f16(b[:, 80:82]), _f16(b[:, 82:84])
    shifts = 2 * torch.arange(4, device=b.device)
    q = (qs[:, :, None, :] >> shifts[None, None, :, None]) & 3  # [n, half, j, 32]
    q = q.reshape(n, 2, 4, 2, 16)  # (l < 16 -> first scale, l >= 16 -> second)
    s = sc.reshape(n, 2, 4, 2)
    dl = d[:, None, None, None] * (s & 0xF).float()
    ml = dmin[:, None, None, None] * (s >> 4).float()
    return (dl[..., None] * q.float() - ml[..., None]).reshape(n, 256)


def _k_scales_6bit(sc: torch.Tensor):
    """12-byte packed 6-bit scale/min pairs (Q4_K / Q5_K) -> (scale[8], min[8])"""
    q = sc.to(torch.int32)
    s_lo = q[:, 0:4] & 63
    m_lo = q[:, 4:8] & 63
    s_hi = (q[:, 8:12] & 0xF) | ((q[:, 0:4] >> 6) << 4)
    m_hi = (q[:, 8:12] >> 4) | ((q[:, 4:8] >> 6) << 4)
    return torch.cat([s_lo, s_hi], 1), torch.cat([m_lo, m_hi], 1)


def _q3_k(b):
    n = b.shape[0]
    hm = b[:, 0:32].to(torch.int32)
    qs = b[:, 32:96].to(torch.int32).reshape(n, 2, 32)
    raw = b[:, 96:108].to(torch.int64)
    d = _f16(b[:, 108:110])
    a0, a1, a2 = _u32(raw[:, 0:4]), _u32(raw[:, 4:8]), _u32(raw[:, 8:12])
    k1, k2 = 0x03030303, 0x0F0F0F0F
    s0 = (a0 & k2) | (((a2 >> 0) & k1) << 4)
    s1 = (a1 & k2) | (((a2 >> 2) & k1) << 4)
    s2 = ((a0 >> 4) & k2) | (((a2 >> 4) & k1) << 4)
    s3 = ((a1 >> 4) & k2) | (((a2 >> 6) & k1) << 4)
    words = torch.stack([s0, s1, s2, s3], 1)  # [n, 4]
    # 16 six-bit scales stored with a +32 bias
    scales = (((words[:, :, None] >> (8 * torch.arange(4, device=b.device))) & 0xFF).reshape(n, 16) - 32).to(torch.int32)
    shifts = 2 * torch.arange(4, device=b.device)
    q = (qs[:, :, None, :] >> shifts[None, None, :, None]) & 3  # [n, half, j, 32]
    mbit = torch.arange(8, device=b.device).reshape(2, 4)  # bit index per (half, j)
    h = (hm[:, None, None, :] >> mbit[None, :, :, None]) & 1
    val = q - 4 * (1 - h)
    val = val.reshape(n, 2, 4, 2, 16)
    dl = d[:, None, None, None] * scales.reshape(n, 2, 4, 2).float()
    return (dl[..., None] * val.float()).reshape(n, 256)


def _q4_k(b):
    n = b.shape[0]
    d, dmin = _f16(b[:, 0:2]), _f16(b[:, 2:4])
    sc, mn = _k_scales_6bit(b[:, 4:16])
    qs = b[:, 16:144].to(torch.int32).reshape(n, 4, 32)
    q = torch.stack([qs & 0xF, qs >> 4], 2).reshape(n, 8, 32)
    return (d[:, None, None] * sc[:, :, None].float() * q.float() - dmin[:, None, None] * mn[:, :, None].float()).reshape(n, 256)


def _q5_k(b):
    n = b.shape[0]
    d, dmin = _f16(b[:, 0:2]), _f16(b[:, 2:4])
    sc, mn = _k_scales_6bit(b[:, 4:16])
    qh = b[:, 16:48].to(torch.int32)
    qs = b[:, 48:176].to(torch.int32).reshape(n, 4, 32)
    lo = torch.stack([qs & 0xF, qs >> 4], 2).reshape(n, 8, 32)
    hb = (qh[:, None, :] >> torch.arange(8, device=b.device)[None, :, None]) & 1  # bit i for sub-block i
    q = lo + 16 * hb
    return (d[:, None, None] * sc[:, :, None].float() * q.float() - dmin[:, None, None] * mn[:, :, None].float()).reshape(n, 256)


def _q6_k(b):
    n = b.shape[0]
    ql = b[:, 0:128].to(torch.int32).reshape(n, 2, 64)
    qh = b[:, 128:192].to(torch.int32).reshape(n, 2, 32)
    sc = b[:, 192:208].view(torch.int8).to(torch.float32).reshape(n, 2, 8)
    d = _f16(b[:, 208:210])
    q1 = (ql[:, :, 0:32] & 0xF) | (((qh >> 0) & 3) << 4)
    q2 = (ql[:, :, 32:64] & 0xF) | (((qh >> 2) & 3) << 4)
    q3 = (ql[:, :, 0:32] >> 4) | (((qh >> 4) & 3) << 4)
    q4 = (ql[:, :, 32:64] >> 4) | (((qh >> 6) & 3) << 4)
    q = torch.stack([q1, q2, q3, q4], 2) - 32  # [n, half, 4, 32]
    # scale index for element l of quarter k: 2*k + l // 16
    s = sc.reshape(n, 2, 4, 2)
    val = q.reshape(n, 2, 4, 2, 16).float() * s[..., None]
    return (d[:, None, None, None, None] * val).reshape(n, 256)


def _q8_k(b):
    d = b[:, 0:4].contiguous().view(torch.float32).squeeze(-1)
    return d[:, None] * b[:, 4:260].view(torch.int8).float()


# ----------------------------------------------------------------------------------------------- IQ / TQ / FP4
def _iq4_nl(b):
    kv = torch.tensor(KVALUES_IQ4NL, dtype=torch.float32, device=b.device)
    return _f16(b[:, 0:2])[:, None] * kv[_lo_hi(b[:, 2:18]).long()]


def _iq4_xs(b):
    n = b.shape[0]
    kv = torch.tensor(KVALUES_IQ4NL, dtype=torch.float32, device=b.device)
    d = _f16(b[:, 0:2])
    sh = _u16(b[:, 2:4])
    sl = b[:, 4:8].to(torch.int32)
    ib = torch.arange(8, device=b.device)
    lo = (sl[:, ib // 2] >> (4 * (ib % 2))) & 0xF
    hi = (sh[:, None] >> (2 * ib)) & 3
    ls = (lo | (hi << 4)) - 32
    qs = b[:, 8:136].reshape(n, 8, 16)
    q = _lo_hi(qs)  # [n, 8, 32]
    return (d[:, None, None] * ls[:, :, None].float() * kv[q.long()]).reshape(n, 256)


def _tq1_0(b):
    n = b.shape[0]
    pow3 = torch.tensor([1, 3, 9, 27, 81, 243], dtype=torch.int32, device=b.device)
    d = _f16(b[:, 52:54])

    def trits(x, k):  # x [n, m] bytes -> [n, k, m] trits, digit-major
        q = (x.to(torch.int32)[:, None, :] * pow3[:k, None]) & 0xFF
        return ((q * 3) >> 8) - 1

    a = trits(b[:, 0:32], 5).reshape(n, 160)
    c = trits(b[:, 32:48], 5).reshape(n, 80)
    h = trits(b[:, 48:52], 4).reshape(n, 16)
    return d[:, None] * torch.cat([a, c, h], 1).float()


def _tq2_0(b):
    n = b.shape[0]
    d = _f16(b[:, 64:66])
    qs = b[:, 0:64].to(torch.int32).reshape(n, 2, 32)
    q = (qs[:, :, None, :] >> (2 * torch.arange(4, device=b.device))[None, None, :, None]) & 3
    return d[:, None] * (q.reshape(n, 256).float() - 1)


def _e8m0_half(e: torch.Tensor) -> torch.Tensor:
    return torch.pow(2.0, e.to(torch.float64) - 128.0).to(torch.float32)


def _ue4m3_half(x: torch.Tensor) -> torch.Tensor:
    x = x.to(torch.int32)
    e = (x >> 3) & 0xF
    m = x & 7
    normal = (8 + m).to(torch.float64) * torch.pow(2.0, e.to(torch.float64) - 10.0)
    sub = m.to(torch.float64) * 2.0 ** -9
    v = torch.where(e == 0, sub, normal)
    v = torch.where((x == 0) | (x == 0x7F), torch.zeros_like(v), v)
    return (v * 0.5).to(torch.float32)


def _mxfp4(b):
    kv = torch.tensor(KVALUES_FP4, dtype=torch.float32, device=b.device)
    return _e8m0_half(b[:, 0])[:, None] * kv[_lo_hi(b[:, 1:17]).long()]


def _nvfp4(b):
    n = b.shape[0]
    kv = torch.tensor(KVALUES_FP4, dtype=torch.float32, device=b.device)
    d = _ue4m3_half(b[:, 0:4])  # [n, 4]
    qs = b[:, 4:36].reshape(n, 4, 8)
    q = _lo_hi(qs)  # [n, 4, 16]
    return (d[:, :, None] * kv[q.long()]).reshape(n, 64)


def _iq2_xxs(b):
    n = b.shape[0]
    grid = _grid("IQ2_XXS", b.device)
    ks = _ksigns(b.device)
    d = _f16(b[:, 0:2])
    q = b[:, 2:66].reshape(n, 8, 8)
    a0 = q[:, :, 0:4].to(torch.int64)  # grid indices
    a1 = _u32(q[:, :, 4:8])
    db = d[:, None] * (0.5 + (a1 >> 28).float()) * 0.25  # [n, 8]
    l = torch.arange(4, device=b.device)
    signs = ks[((a1[:, :, None] >> (7 * l)) & 127)]  # [n, 8, 4]
    g = grid[a0]  # [n, 8, 4, 8]
    return (db[:, :, None, None] * g * _sign_bits(signs)).reshape(n, 256)


def _iq2_xs(b):
    n = b.shape[0]
    grid = _grid("IQ2_XS", b.device)
    ks = _ksigns(b.device)
    d = _f16(b[:, 0:2])
    qs = _u16(b[:, 2:66].reshape(n, 32, 2)).reshape(n, 8, 4)
    sc = b[:, 66:74].to(torch.int32)
    db = torch.stack([d[:, None] * (0.5 + (sc & 0xF).float()) * 0.25, d[:, None] * (0.5 + (sc >> 4).float()) * 0.25], 2)
    g = grid[(qs & 511).long()]  # [n, 8, 4, 8]
    signs = ks[qs >> 9]
    dl = db[:, :, torch.tensor([0, 0, 1, 1], device=b.device)]  # [n, 8, 4]
    return (dl[..., None] * g * _sign_bits(signs)).reshape(n, 256)


def _iq2_s(b):
    n = b.shape[0]
    grid = _grid("IQ2_S", b.device)
    d = _f16(b[:, 0:2])
    qs = b[:, 2:34].to(torch.int32).reshape(n, 8, 4)
    signs = b[:, 34:66].to(torch.int32).reshape(n, 8, 4)
    qh = b[:, 66:74].to(torch.int32)
    sc = b[:, 74:82].to(torch.int32)
    l = torch.arange(4, device=b.device)
    idx = qs | ((qh[:, :, None] << (8 - 2 * l)) & 0x300)
    db = torch.stack([d[:, None] * (0.5 + (sc & 0xF).float()) * 0.25, d[:, None] * (0.5 + (sc >> 4).float()) * 0.25], 2)
    dl = db[:, :, torch.tensor([0, 0, 1, 1], device=b.device)]
    return (dl[..., None] * grid[idx.long()] * _sign_bits(signs)).reshape(n, 256)


def _iq3_xxs(b):
    n = b.shape[0]
    grid = _grid("IQ3_XXS", b.device)
    ks = _ksigns(b.device)
    d = _f16(b[:, 0:2])
    qs = b[:, 2:66].to(torch.int64).reshape(n, 8, 8)
    aux = _u32(b[:, 66:98].reshape(n, 8, 4))
    db = d[:, None] * (0.5 + (aux >> 28).float()) * 0.5
    l = torch.arange(4, device=b.device)
    signs = ks[(aux[:, :, None] >> (7 * l)) & 127]  # [n, 8, 4]
    g = grid[qs].reshape(n, 8, 4, 8)  # pairs of 4-value grid rows -> 8 values per l
    return (db[:, :, None, None] * g * _sign_bits(signs)).reshape(n, 256)


def _iq3_s(b):
    n = b.shape[0]
    grid = _grid("IQ3_S", b.device)
    d = _f16(b[:, 0:2])
    qs = b[:, 2:66].to(torch.int32).reshape(n, 8, 4, 2)
    qh = b[:, 66:74].to(torch.int32)  # one byte per 32 elements
    signs = b[:, 74:106].to(torch.int32).reshape(n, 8, 4)
    sc = b[:, 106:110].to(torch.int32)
    l = torch.arange(4, device=b.device)
    hi0 = (qh[:, :, None] << (8 - 2 * l)) & 256
    hi1 = (qh[:, :, None] << (7 - 2 * l)) & 256
    g0 = grid[(qs[..., 0] | hi0).long()]  # [n, 8, 4, 4]
    g1 = grid[(qs[..., 1] | hi1).long()]
    g = torch.cat([g0, g1], -1)  # [n, 8, 4, 8]
    ib = torch.arange(8, device=b.device)
    s = (sc[:, ib // 2] >> (4 * (ib % 2))) & 0xF
    db = d[:, None] * (1 + 2 * s).float()
    return (db[:, :, None, None] * g * _sign_bits(signs)).reshape(n, 256)


def _iq1_s(b):
    n = b.shape[0]
    grid = _grid("IQ1_S", b.device)
    d = _f16(b[:, 0:2])
    qs = b[:, 2:34].to(torch.int32).reshape(n, 8, 4)
    qh = _u16(b[:, 34:50].reshape(n, 8, 2))
    l = torch.arange(4, device=b.device)
    idx = qs | (((qh[:, :, None] >> (3 * l)) & 7) << 8)
    dl = d[:, None] * (2 * ((qh >> 12) & 7) + 1).float()
    delta = torch.where((qh & 0x8000) != 0, -IQ1_DELTA, IQ1_DELTA)
    return (dl[:, :, None, None] * (grid[idx.long()] + delta[:, :, None, None])).reshape(n, 256)


def _iq1_m(b):
    n = b.shape[0]
    grid = _grid("IQ1_M", b.device)
    qs = b[:, 0:32].to(torch.int32).reshape(n, 8, 4)
    qh = b[:, 32:48].to(torch.int32).reshape(n, 8, 2)
    sc = _u16(b[:, 48:56].reshape(n, 4, 2))  # [n, 4]
    scale_u16 = (sc[:, 0] >> 12) | ((sc[:, 1] >> 8) & 0x00F0) | ((sc[:, 2] >> 4) & 0x0F00) | (sc[:, 3] & 0xF000)
    d = scale_u16.to(torch.int16).view(torch.float16).float()
    ib = torch.arange(8, device=b.device)
    s = sc[:, ib // 2]
    sh = 6 * (ib % 2)
    dl1 = d[:, None] * (2 * ((s >> sh) & 7) + 1).float()
    dl2 = d[:, None] * (2 * ((s >> (sh + 3)) & 7) + 1).float()
    idx = torch.stack([qs[..., 0] | ((qh[..., 0] << 8) & 0x700), qs[..., 1] | ((qh[..., 0] << 4) & 0x700),
                       qs[..., 2] | ((qh[..., 1] << 8) & 0x700), qs[..., 3] | ((qh[..., 1] << 4) & 0x700)], -1)
    delta = torch.stack([(qh[..., 0] & 0x08) != 0, (qh[..., 0] & 0x80) != 0,
                         (qh[..., 1] & 0x08) != 0, (qh[..., 1] & 0x80) != 0], -1)
    delta = torch.where(delta, -IQ1_DELTA, IQ1_DELTA)
    dl = torch.stack([dl1, dl1, dl2, dl2], -1)  # [n, 8, 4]
    return (dl[..., None] * (grid[idx.long()] + delta[..., None])).reshape(n, 256)


_DECODERS = {
    2: _q4_0, 3: _q4_1, 6: lambda b: _q5(b, False), 7: lambda b: _q5(b, True), 8: _q8_0, 9: _q8_1,
    10: _q2_k, 11: _q3_k, 12: _q4_k, 13: _q5_k, 14: _q6_k, 15: _q8_k, 16: _iq2_xxs, 17: _iq2_xs, 18: _iq3_xxs,
    19: _iq1_s, 20: _iq4_nl, 21: _iq3_s, 22: _iq2_s, 23: _iq4_xs, 29: _iq1_m, 34: _tq1_0, 35: _tq2_0,
    39: _mxfp4, 40: _nvfp4, 41: _q1_0, 42: _q2_0,
}
_PLAIN = {0: torch.float32, 1: torch.float16, 30: torch.bfloat16, 24: torch.int8, 25: torch.int16, 26: torch.int32,
          27: torch.int64, 28: torch.float64}


def dequantize(data, ggml_type: int, numel: int, device="cpu", dtype=torch.float32) -> torch.Tensor:
    """Packed bytes (bytes / memoryview / uint8 tensor) of ``numel`` elements -> flat tensor of ``dtype``."""
    if isinstance(data, torch.Tensor):
        raw = data.to(device).reshape(-1)
    else:
        raw = torch.frombuffer(bytearray(data), dtype=torch.uint8).to(device)
    if ggml_type in _PLAIN:
        t = raw.view(_PLAIN[ggml_type])[:numel]
        return t.to(dtype)
    be, bb = block_info(ggml_type)
    nblocks = numel // be
    blocks = raw[:nblocks * bb].reshape(nblocks, bb)
    dec = _DECODERS.get(ggml_type)
    if dec is None:
        raise ValueError(f"no dequantizer for {type_name(ggml_type)}")
    out = []
    step = 1 << 16  # bound temporaries
    for s in range(0, nblocks, step):
        out.append(dec(blocks[s:s + step]).reshape(-1))
    return torch.cat(out).to(dtype) if len(out) > 1 else out[0].to(dtype)
