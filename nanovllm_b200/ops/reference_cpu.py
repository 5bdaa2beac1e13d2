"""Plain-PyTorch fp32 restatement of every kernel (the CPU oracle and the timed CPU baseline).

Each function restates the reference's CPU math (nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/tensor/
Ops.java, layers/Attention.java, layers/Norms.java, layers/Sampler.java) on torch tensors, computing in float32
and returning the same dtypes as the CUDA kernels so tests can compare the two directly.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import numpy as np
import torch

ACT_NONE, ACT_SILU_MUL, ACT_GELU_MUL = 0, 1, 2
BIAS_ACT_NONE, BIAS_ACT_GELU_ERF, BIAS_ACT_GELU_TANH = 0, 3, 4


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)))


def gelu_erf(x: torch.Tensor) -> torch.Tensor:
    return 0.5 * x * (1.0 + torch.erf(x * 0.7071067811865476))


def silu(x: torch.Tensor) -> torch.Tensor:
    return x / (1.0 + torch.exp(-x))


def _norm_weight(w: Optional[torch.Tensor], mode: int, n: int) -> torch.Tensor:
    if mode == 2 or w is None:
        return torch.ones(n, dtype=torch.float32)
    w = w.float()
    return w + 1.0 if mode == 1 else w


def rms_norm(x: torch.Tensor, weight: Optional[torch.Tensor], eps: float, mode: int = 0,
             residual: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """mode 0: x*w, 1: x*(1+w) (Gemma), 2: weightless.  With ``residual``: residual += x (stored back in the
    residual dtype) and the sum is normalised (Ops.addRmsNorm)."""
    xf = x.float()
    new_res = None
    if residual is not None:
        s = xf + residual.float()
        new_res = s.to(residual.dtype)
        xf = new_res.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    y = xf * inv * _norm_weight(weight, mode, x.shape[-1])
    return y.to(x.dtype), new_res


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float,
               residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    xf = x.float()
    if residual is not None:
        xf = xf + residual.float()
    mean = xf.mean(-1, keepdim=True)
    var = (xf - mean).pow(2).mean(-1, keepdim=True)
    y = (xf - mean) * torch.rsqrt(var + eps) * weight.float() + bias.float()
    return y.to(x.dtype)


def rope_cos_sin(head_dim: int, max_pos: int, base: float, partial_factor: float = 1.0,
                 device="cpu") -> torch.Tensor:
    """[max_pos, head_dim] fp32 table: cos for the hd/2 pair frequencies, then sin.  NeoX pairs (i, i + hd/2)
    with inv_freq = base^(-2i/hd) (Norms.java:171-249).  ``partial_factor`` < 1 zeroes the frequencies past
    partial_factor * hd / 2 (Gemma4 proportional RoPE), i.e. those pairs are not rotated."""
    half = head_dim // 2
    inv = 1.0 / (base ** (torch.arange(0, half, dtype=torch.float64) * 2.0 / head_dim))
    if partial_factor < 1.0:
        keep = int(partial_factor * head_dim / 2)
        inv[keep:] = 0.0
    pos = torch.arange(max_pos, dtype=torch.float64)
    ang = pos[:, None] * inv[None, :]
    return torch.cat([torch.cos(ang), torch.sin(ang)], dim=-1).float().to(device)


def qk_norm_rope_store(qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor,
                       q_w: Optional[torch.Tensor], k_w: Optional[torch.Tensor], norm_mode: int, v_norm: bool,
                       eps: float, k_cache: Optional[torch.Tensor], v_cache: Optional[torch.Tensor],
                       slots: Optional[torch.Tensor], nq: int, nkv: int, hd: int, apply_rope: bool = True):
    T = qkv.shape[0]
    x = qkv.float().reshape(T, nq + 2 * nkv, hd)
    q, k, v = x[:, :nq], x[:, nq:nq + nkv], x[:, nq + nkv:]

    def hnorm(t, w, mode):
        if mode < 0:
            return t
        inv = torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps)
        return t * inv * _norm_weight(w, mode, hd)

    q = hnorm(q, q_w, norm_mode)
    k = hnorm(k, k_w, norm_mode)
    if v_norm:
        v = hnorm(v, None, 2)
    if apply_rope:
        cs = cos_sin[positions.long()]
        half = hd // 2
        c, s = cs[:, None, :half], cs[:, None, half:]

        def rot(t):
            a, b = t[..., :half], t[..., half:]
            return torch.cat([a * c - b * s, b * c + a * s], dim=-1)

        q, k = rot(q), rot(k)
    q_out = q.to(qkv.dtype).contiguous()
    if k_cache is not None and slots is not None:
        bs = k_cache.shape[2]
        for t in range(T):
            sl = int(slots[t])
            if sl < 0:
                continue
            blk, off = sl // bs, sl % bs
            k_cache[blk, :, off, :] = k[t].to(k_cache.dtype)
            v_cache[blk, :, off, :] = v[t].to(v_cache.dtype)
    return q_out, k.to(qkv.dtype), v.to(qkv.dtype)


def _softcap(s: torch.Tensor, cap: float) -> torch.Tensor:
    return cap * torch.tanh(s / cap) if cap and cap > 0 else s


def _attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_pos: torch.Tensor, causal: bool,
            window: int, scale: float, softcap: float) -> torch.Tensor:
    """q [Tq, H, D], k/v [Tk, H, D] (already GQA-expanded), q_pos absolute positions of the queries."""
    s = torch.einsum("qhd,khd->hqk", q.float(), k.float()) * scale
    s = _softcap(s, softcap)
    kpos = torch.arange(k.shape[0])
    mask = torch.ones(q.shape[0], k.shape[0], dtype=torch.bool)
    if causal:
        mask &= kpos[None, :] <= q_pos[:, None]
        if window > 0:
            mask &= kpos[None, :] > (q_pos[:, None] - window)
    s = s.masked_fill(~mask[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)
    return torch.einsum("hqk,khd->qhd", p, v.float())


def _gather_paged(cache: torch.Tensor, table: torch.Tensor, n: int) -> torch.Tensor:
    """cache [NB, nkv, BS, D] -> [n, nkv, D] for the first n tokens of a sequence."""
    bs = cache.shape[2]
    nb = (n + bs - 1) // bs
    blocks = cache[table[:nb].long()]  # [nb, nkv, bs, D]
    return blocks.permute(0, 2, 1, 3).reshape(nb * bs, cache.shape[1], cache.shape[3])[:n]


def paged_decode(q: torch.Tensor, k_cache, v_cache, block_tables, ctx_lens, scale, softcap=0.0, window=0):
    B, nq, D = q.shape
    nkv = k_cache.shape[1]
    G = nq // nkv
    out = torch.empty_like(q)
    for b in range(B):
        n = int(ctx_lens[b])
        k = _gather_paged(k_cache, block_tables[b], n).repeat_interleave(G, dim=1)
        v = _gather_paged(v_cache, block_tables[b], n).repeat_interleave(G, dim=1)
        o = _attend(q[b:b + 1], k, v, torch.tensor([n - 1]), True, window, scale, softcap)
        out[b] = o[0].to(q.dtype)
    return out


def prefill_attention(q: torch.Tensor, cu_q, cu_k, nq, nkv, hd, scale, softcap=0.0, window=0, causal=True,
                      k_cache=None, v_cache=None, block_tables=None, kv_src=None):
    """q [T, nq, hd]; paged K/V via block tables, or contiguous K/V from the packed qkv ``kv_src``."""
    G = nq // nkv
    T = q.shape[0]
    out = torch.zeros(T, nq, hd, dtype=q.dtype)
    for i in range(len(cu_q) - 1):
        q0, q1 = int(cu_q[i]), int(cu_q[i + 1])
        k0, k1 = int(cu_k[i]), int(cu_k[i + 1])
        klen, qlen = k1 - k0, q1 - q0
        if qlen == 0:
            continue
        if k_cache is not None:
            k = _gather_paged(k_cache, block_tables[i], klen)
            v = _gather_paged(v_cache, block_tables[i], klen)
        else:
            src = kv_src[k0:k1].reshape(klen, nq + 2 * nkv, hd)
            k, v = src[:, nq:nq + nkv], src[:, nq + nkv:]
        k = k.repeat_interleave(G, dim=1)
        v = v.repeat_interleave(G, dim=1)
        qpos = torch.arange(klen - qlen, klen)
        out[q0:q1] = _attend(q[q0:q1].reshape(qlen, nq, hd), k, v, qpos, causal, window, scale, softcap).to(q.dtype)
    return out


def interleave_gate_up(gate_up: torch.Tensor, block: int = 128) -> torch.Tensor:
    """[gate(I); up(I)] rows -> blocks [gate_b; up_b] of ``block`` rows each (the layout of the fused kernels)."""
    I = gate_up.shape[0] // 2
    g, u = gate_up[:I], gate_up[I:]
    nb = I // block
    return torch.stack([g.reshape(nb, block, -1), u.reshape(nb, block, -1)], dim=1).reshape(2 * I, -1)


def linear(x: torch.Tensor, w: torch.Tensor, act: int = ACT_NONE, interleaved: bool = True) -> torch.Tensor:
    y = x.float() @ w.float().t()
    if act != ACT_NONE:
        I = y.shape[1] // 2
        if interleaved:
            y3 = y.reshape(y.shape[0], I // 128, 2, 128)
            g, u = y3[:, :, 0].reshape(-1, I), y3[:, :, 1].reshape(-1, I)
        else:
            g, u = y[:, :I], y[:, I:]
        y = (silu(g) if act == ACT_SILU_MUL else gelu_tanh(g)) * u
    return y.to(x.dtype)


def act_mul(x: torch.Tensor, act: int, interleaved: bool = False) -> torch.Tensor:
    y = x.float()
    I = y.shape[1] // 2
    if interleaved:
        y3 = y.reshape(y.shape[0], I // 128, 2, 128)
        g, u = y3[:, :, 0].reshape(-1, I), y3[:, :, 1].reshape(-1, I)
    else:
        g, u = y[:, :I], y[:, I:]
    return ((silu(g) if act == ACT_SILU_MUL else gelu_tanh(g)) * u).to(x.dtype)


def bias_act(x: torch.Tensor, bias: Optional[torch.Tensor], act: int) -> torch.Tensor:
    y = x.float()
    if bias is not None:
        y = y + bias.float()
    if act == BIAS_ACT_GELU_ERF:
        y = gelu_erf(y)
    elif act == BIAS_ACT_GELU_TANH:
        y = gelu_tanh(y)
    return y.to(x.dtype)


def embedding(table: torch.Tensor, ids: torch.Tensor, scale: float = 1.0, vstart: int = 0,
              vend: Optional[int] = None) -> torch.Tensor:
    vend = table.shape[0] + vstart if vend is None else vend
    ids = ids.long()
    inside = (ids >= vstart) & (ids < vend)
    rows = table[(ids - vstart).clamp(0, table.shape[0] - 1)].float() * scale
    rows[~inside] = 0.0
    return rows.to(table.dtype)


def mean_pool_l2(x: torch.Tensor, cu: torch.Tensor) -> torch.Tensor:
    outs = []
    for i in range(len(cu) - 1):
        seg = x[int(cu[i]):int(cu[i + 1])].float()
        m = seg.mean(0)
        outs.append(m / m.norm().clamp_min(1e-12))
    return torch.stack(outs)


# ----------------------------------------------------------------------------------------------- sampler
_M0, _M1, _W0, _W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85


def philox_uniform(idx: np.ndarray, step: int, seq_id: int, seed: int) -> np.ndarray:
    """Philox4x32-10 (Salmon et al., SC'11), counter (i, step, seq_id, 0x6e76), key = seed; first word -> [0,1)."""
    c0 = idx.astype(np.uint64) & 0xFFFFFFFF
    c1 = np.full_like(c0, step & 0xFFFFFFFF)
    c2 = np.full_like(c0, seq_id & 0xFFFFFFFF)
    c3 = np.full_like(c0, 0x6e76)
    k0 = seed & 0xFFFFFFFF
    k1 = (seed >> 32) & 0xFFFFFFFF
    mask = np.uint64(0xFFFFFFFF)
    for _ in range(10):
        p0 = np.uint64(_M0) * c0
        p1 = np.uint64(_M1) * c2
        hi0, lo0 = (p0 >> np.uint64(32)) & mask, p0 & mask
        hi1, lo1 = (p1 >> np.uint64(32)) & mask, p1 & mask
        c0, c1, c2, c3 = (hi1 ^ c1 ^ np.uint64(k0)) & mask, lo1, (hi0 ^ c3 ^ np.uint64(k1)) & mask, lo0
        k0 = (k0 + _W0) & 0xFFFFFFFF
        k1 = (k1 + _W1) & 0xFFFFFFFF
    return (c0 >> np.uint64(8)).astype(np.float64) * (1.0 / 16777216.0)


def sample(logits: torch.Tensor, temps, top_ks, top_ps, seeds, seq_ids, steps, softcap: float = 0.0,
           ids=None) -> torch.Tensor:
    """Per row: top_k == 1 -> argmax; else softmax(x/T) -> top-k -> top-p (keep while cum < p, first always)
    -> argmax p / -log(u) (Sampler.java:69-134) with Philox uniforms instead of ThreadLocalRandom.  ``ids``
    (optional [B, C]): the rows are candidates, column c standing for vocabulary id ids[b, c] (ascending)."""
    out = torch.empty(logits.shape[0], dtype=torch.long)
    x_all = logits.float()
    if softcap and softcap > 0:
        x_all = softcap * torch.tanh(x_all / softcap)
    for r in range(logits.shape[0]):
        x = x_all[r]
        k = int(top_ks[r])
        idmap = None if ids is None else ids[r].long().cpu().numpy()
        if k == 1:
            j = int(torch.argmax(x))  # first maximal index
            out[r] = j if idmap is None else int(idmap[j])
            continue
        t = float(temps[r])
        xs = x / t
        p = torch.exp(xs - xs.max())
        order = torch.sort(-x, stable=True).indices  # value descending, index ascending on ties
        keep = torch.zeros_like(p, dtype=torch.bool)
        keep[order if (k <= 0 or k >= x.numel()) else order[:k]] = True
        topp = float(top_ps[r])
        if topp < 1.0:
            kept_order = order[keep[order]]
            pk = p[kept_order].double()
            z = float(pk.sum())
            before = torch.cumsum(pk, 0) - pk  # mass strictly before each kept token
            n_keep = max(1, int((before < topp * z).sum()))
            keep = torch.zeros_like(keep)
            keep[kept_order[:n_keep]] = True
        idxs = torch.nonzero(keep).flatten().numpy()
        gidx = idxs if idmap is None else idmap[idxs]
        u = philox_uniform(gidx, int(steps[r]), int(seq_ids[r]), int(seeds[r]) & 0xFFFFFFFFFFFFFFFF)
        g = -np.log(np.maximum(1e-10, u))
        score = p[idxs].double().numpy() / np.maximum(1e-10, g)
        out[r] = int(gidx[int(np.argmax(score))])
    return out


def shortconv(proj: torch.Tensor, weight: torch.Tensor, cu: torch.Tensor, rows: torch.Tensor, fresh: torch.Tensor,
              state: torch.Tensor, state_off: int) -> torch.Tensor:
    """LFM2 gated short conv (ShortConv.java:102-243): y = C * causal_conv(B * x), per-sequence state of the last
    L-1 B*x rows (zeros when ``fresh``), updated in place."""
    H, L = weight.shape
    p = proj.float()
    b, c, x = p[:, :H], p[:, H:2 * H], p[:, 2 * H:]
    bx = b * x
    out = torch.empty(proj.shape[0], H, dtype=torch.float32)
    w = weight.float()
    for s in range(len(cu) - 1):
        t0, t1 = int(cu[s]), int(cu[s + 1])
        if t1 <= t0:
            continue
        row = int(rows[s])
        sl = state[row, state_off:state_off + (L - 1) * H].view(L - 1, H)
        prev = torch.zeros(L - 1, H) if bool(fresh[s]) else sl.clone()
        window = torch.cat([prev, bx[t0:t1]], 0)
        for t in range(t1 - t0):
            out[t0 + t] = (window[t:t + L] * w.t()).sum(0)
        sl.copy_(window[-(L - 1):] if L > 1 else sl)
    return (c * out).to(proj.dtype)


# ----------------------------------------------------------------------------------------------- Gemma4
def _gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)))


def rms_norm_post_add(x, residual, weight, eps, mode=0, post_scale=1.0):
    """residual = (residual + rmsnorm(x) * w) * post_scale, in place (Gemma4 sandwich norm + layer_scalar)."""
    n, _ = rms_norm(x, weight, eps, mode)
    residual.copy_(((residual.float() + n.float()) * post_scale).to(residual.dtype))
    return residual


def ple_combine(proj, tok, weight, eps, proj_scale, out_scale):
    """(rmsnorm(proj * proj_scale) * w + tok) * out_scale over rows of width P = weight.numel()."""
    P = weight.numel()
    p = (proj.float() * proj_scale).to(proj.dtype).reshape(-1, P)
    n, _ = rms_norm(p, weight, eps, 0)
    out = (n.float() + tok.reshape(-1, P).float()) * out_scale
    return out.to(proj.dtype).reshape(proj.shape)


def gate_act_mul(gate, other):
    return (_gelu_tanh(gate.float()) * other.float()).to(gate.dtype)


def srq(x: torch.Tensor, scale: float) -> torch.Tensor:
    """Static-range activation fake-quant: clamp(floor(x / s + 0.5), -128, 127) * s (GemmaQat.applySrq)."""
    if scale == 0.0:
        return x
    q = torch.floor(x.float() / scale + 0.5).clamp(-128.0, 127.0)
    return (q * scale).to(x.dtype)
