"""Op layer: CUDA tensors run the sm_100a kernels of ``nanovllm_b200._C``; CPU tensors run the fp32 restatement
in ``reference_cpu`` (the oracle and the timed CPU baseline).

On a CUDA tensor there is no silent fallback: if the extension did not load, the op raises.  The per-device
error word (int32) is passed to every kernel that waits on an mbarrier or a peer flag; ``check_device_errors``
reads it after a synchronisation and raises ``DeviceWaitTimeout`` when a bounded wait gave up.
"""
from __future__ import annotations

import os
from typing import Dict, Optional, Tuple

import torch

from . import reference_cpu as ref
from ..exceptions import DeviceWaitTimeout

ACT_NONE, ACT_SILU_MUL, ACT_GELU_MUL = ref.ACT_NONE, ref.ACT_SILU_MUL, ref.ACT_GELU_MUL
BIAS_ACT_NONE, BIAS_ACT_GELU_ERF, BIAS_ACT_GELU_TANH = ref.BIAS_ACT_NONE, ref.BIAS_ACT_GELU_ERF, ref.BIAS_ACT_GELU_TANH

_C = None
_C_ERROR: Optional[BaseException] = None
try:  # the extension is built in-tree by setup.py / __graft_entry__.build()
    from .. import _C as _C  # type: ignore
except BaseException as e:  # noqa: BLE001 - keep the reason for the loud error below
    _C_ERROR = e


def extension_loaded() -> bool:
    return _C is not None


def _cuda_ext():
    if _C is None:
        raise RuntimeError(f"nanovllm_b200._C is not built or failed to load ({_C_ERROR!r}); "
                           "run `python setup.py build_ext --inplace`")
    return _C


class SplitK:
    """Unreduced output of a split-K decode GEMM: fp32 partials [S, M, N] whose sum is the result.

    Consumers that can fuse the sum (add+RMSNorm, the RoPE/KV-store kernel) take it directly; anything else
    calls ``materialize``.  The partials are summed in split order, so the result is deterministic."""
    __slots__ = ("parts",)

    def __init__(self, parts: torch.Tensor):
        self.parts = parts

    @property
    def shape(self):
        return tuple(self.parts.shape[1:])

    @property
    def dtype(self):
        return torch.bfloat16

    @property
    def device(self):
        return self.parts.device

    @property
    def is_cuda(self):
        return True

    def reshape(self, *shape):
        return materialize(self).reshape(*shape)


class TPPartial:
    """This rank's row-parallel partial sum [T, H], already in the symmetric workspace's ``in`` slot.

    A following RMSNorm (with or without residual) runs the fused all-reduce + residual + RMSNorm kernel over
    peer memory; anything else calls ``materialize`` (a plain fused all-reduce)."""
    __slots__ = ("ws", "T")

    def __init__(self, ws, T: int):
        self.ws, self.T = ws, T

    @property
    def shape(self):
        return (self.T, self.ws.hidden)

    @property
    def dtype(self):
        return torch.bfloat16

    @property
    def device(self):
        return self.ws.buf.device

    @property
    def is_cuda(self):
        return True

    def reshape(self, *shape):
        return materialize(self).reshape(*shape)


def materialize(x):
    """bf16 tensor from a SplitK (one fused sum kernel), a TPPartial (fused all-reduce) or an SPHidden (all-gather
    + final norm), identity otherwise."""
    if isinstance(x, SPHidden):
        return x.materialize()
    if isinstance(x, TPPartial):
        return x.ws.allreduce_norm(x.T, None, 0.0, 3, None)[0]
    if isinstance(x, SplitK):
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
        _cuda_ext().splitk_sum(x.parts, out)
        add_launches(1)
        return out
    return x


_LAUNCHES = [0]


def add_launches(n: int) -> None:
    """Kernel-launch accounting (CUDA-graph replays add the count recorded at capture)."""
    _LAUNCHES[0] += int(n)


def launch_count() -> int:
    return _LAUNCHES[0]


def reset_launch_count() -> None:
    _LAUNCHES[0] = 0


_ERR: Dict[int, torch.Tensor] = {}
_WS: Dict[int, torch.Tensor] = {}


def error_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _ERR.get(idx)
    if t is None:
        with torch.inference_mode(False):  # a normal tensor: the host zeroes it in and outside inference mode
            t = torch.zeros(1, dtype=torch.int32, device=device)
        _ERR[idx] = t
    return t


def check_device_errors(device: Optional[torch.device] = None) -> None:
    dev = device or torch.device("cuda", torch.cuda.current_device())
    code = int(error_word(dev).item())
    if code != 0:
        error_word(dev).zero_()
        raise DeviceWaitTimeout(f"device kernel reported error code {code} (1 = mbarrier wait timeout, "
                                f"2 = peer flag timeout, 3 = bad argument)")


def workspace(device: torch.device, numel: int) -> torch.Tensor:
    """Shared fp32 scratch for split-K partials; grows on demand (pre-size it before CUDA-graph capture)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _WS.get(idx)
    if t is None or t.numel() < numel:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("gemm workspace must be reserved before CUDA graph capture")
        t = torch.empty(max(numel, 1 << 20), dtype=torch.float32, device=device)
        _WS[idx] = t
    return t


def reserve_workspace(device: torch.device, max_m: int, max_n: int, max_k: int) -> None:
    if _C is None:
        return
    splits = max(_C.gemm_splits_for(m, max_n, max_k, 0) for m in (1, 16, 64, 128, 256) if m <= max(1, max_m))
    workspace(device, splits * min(256, max_m) * max_n)


# ------------------------------------------------------------------------------------------------ norms
def rms_norm(x: torch.Tensor, weight: Optional[torch.Tensor], eps: float, mode: int = 0,
             residual: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None
             ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Returns (normed, residual).  With ``residual`` the sum x + residual is written back into it."""
    if isinstance(x, TPPartial):
        return x.ws.allreduce_norm(x.T, weight, eps, mode, residual)
    if not x.is_cuda:
        y, r = ref.rms_norm(x, weight, eps, mode, residual)
        if residual is not None:
            residual.copy_(r)
            r = residual
        return y, r
    if isinstance(x, SplitK):
        if out is None:
            out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
        _cuda_ext().rms_norm(out, out, residual, weight, float(eps), int(mode), x.parts)
        add_launches(1)
        return out, residual
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    _cuda_ext().rms_norm(out, x, residual, weight, float(eps), int(mode), None)
    add_launches(1)
    return out, residual


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float,
               residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    x = materialize(x)
    if not x.is_cuda:
        return ref.layer_norm(x, weight, bias, eps, residual)
    out = torch.empty_like(x)
    _cuda_ext().layer_norm(out, x.contiguous(), residual, weight, bias, float(eps))
    add_launches(1)
    return out


# ------------------------------------------------------------------------------------------------ rope + kv
def qk_norm_rope_store(qkv, positions, cos_sin, q_w, k_w, norm_mode, v_norm, eps, k_cache, v_cache, slots,
                       nq, nkv, hd, apply_rope=True):
    """Returns q [T, nq, hd] (normed + rotated); k and v go into the paged caches at ``slots``."""
    if not qkv.is_cuda:
        q, _, _ = ref.qk_norm_rope_store(qkv, positions, cos_sin, q_w, k_w, norm_mode, v_norm, eps, k_cache,
                                         v_cache, slots, nq, nkv, hd, apply_rope)
        return q.reshape(qkv.shape[0], nq, hd)
    part = None
    if isinstance(qkv, SplitK):
        part = qkv.parts
        qkv = torch.empty(1, part.shape[2], dtype=torch.bfloat16, device=part.device).expand(part.shape[1], -1)
    q = torch.empty(qkv.shape[0], nq, hd, dtype=torch.bfloat16, device=qkv.device)
    _cuda_ext().qk_norm_rope_store(qkv, positions, cos_sin, q_w, k_w, int(norm_mode), bool(v_norm), float(eps), q,
                                   k_cache, v_cache, slots, int(nq), int(nkv), int(hd), bool(apply_rope), part)
    add_launches(1)
    return q


# ------------------------------------------------------------------------------------------------ attention
DECODE_TILE = 64


_SMS: Dict[int, int] = {}


def num_sms(device: Optional[torch.device] = None) -> int:
    """SM count of ``device`` (the current CUDA device by default; 148, a B200, without CUDA)."""
    if not torch.cuda.is_available():
        return 148
    idx = device.index if (device is not None and device.index is not None) else torch.cuda.current_device()
    n = _SMS.get(idx)
    if n is None:
        n = torch.cuda.get_device_properties(idx).multi_processor_count
        _SMS[idx] = n
    return n


def decode_partition(batch: int, nkv: int, max_len: int, sms: Optional[int] = None) -> Tuple[int, int]:
    """(tiles per split, number of splits) so that batch * nkv * splits covers ~4 CTAs per SM (the SM count of
    the current device unless given; the allocation-free C entry point uses the same rule and source)."""
    if sms is None:
        sms = num_sms()
    tiles = max(1, (max_len + DECODE_TILE - 1) // DECODE_TILE)
    target = 4 * sms
    per = max(1, min(16, (batch * nkv * tiles + target - 1) // target))
    per = max(per, (tiles + 63) // 64)  # at most 64 splits
    return per, (tiles + per - 1) // per


def paged_decode(q, k_cache, v_cache, block_tables, ctx_lens, scale, softcap=0.0, window=0, max_len=None,
                 out=None, scratch=None):
    if not q.is_cuda:
        return ref.paged_decode(q, k_cache, v_cache, block_tables, ctx_lens, scale, softcap, window)
    B, nq, hd = q.shape
    nkv = k_cache.shape[1]
    if max_len is None:
        max_len = block_tables.shape[1] * k_cache.shape[2]
    per, nsplit = decode_partition(B, nkv, max_len, num_sms(q.device))
    if out is None:
        out = torch.empty_like(q)
    if nsplit > 1:
        need = B * nq * nsplit * (hd + 1)
        if scratch is None or scratch.numel() < need:
            scratch = torch.empty(need, dtype=torch.float32, device=q.device)
        part_o = scratch[:B * nq * nsplit * hd]
        part_lse = scratch[B * nq * nsplit * hd:need]
    else:
        part_o = part_lse = out  # unused
    cnt = _combine_counters(q.device, B * nkv) if nsplit > 1 else None
    _cuda_ext().paged_decode(q, k_cache, v_cache, block_tables, ctx_lens, out, part_o, part_lse, float(scale),
                             float(softcap), int(window), int(per), int(nsplit), error_word(q.device), cnt)
    add_launches(2 if nsplit > 1 and cnt is None else 1)
    return out


_CNT: Dict[int, torch.Tensor] = {}


def _combine_counters(device: torch.device, need: int) -> Optional[torch.Tensor]:
    """Zeroed int32 arrival counters for the in-kernel split-KV merge (the kernel leaves them zeroed).  They are
    created outside stream capture; a capture that finds none uses the separate merge kernel instead."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _CNT.get(idx)
    if t is None or t.numel() < need:
        if torch.cuda.is_current_stream_capturing():
            return None
        t = torch.zeros(max(need, 1 << 16), dtype=torch.int32, device=device)
        _CNT[idx] = t
    return t


def decode_scratch_numel(batch: int, nq: int, nkv: int, hd: int, max_len: int) -> int:
    _, nsplit = decode_partition(batch, nkv, max_len)
    return batch * nq * nsplit * (hd + 1) if nsplit > 1 else 0


def prefill_attention(q, cu_q, cu_k, max_q, nq, nkv, hd, scale, softcap=0.0, window=0, causal=True,
                      k_cache=None, v_cache=None, block_tables=None, kv_src=None, out=None):
    if not q.is_cuda:
        return ref.prefill_attention(q.reshape(q.shape[0], nq, hd), cu_q, cu_k, nq, nkv, hd, scale, softcap, window,
                                     causal, k_cache, v_cache, block_tables, kv_src)
    if out is None:
        out = torch.empty(q.shape[0], nq, hd, dtype=q.dtype, device=q.device)
    _cuda_ext().prefill_attention(q, out, cu_q, cu_k, int(max_q), k_cache, v_cache, block_tables, kv_src, int(nq),
                                  int(nkv), int(hd), float(scale), float(softcap), int(window), bool(causal),
                                  error_word(q.device))
    add_launches(1)
    return out


# ------------------------------------------------------------------------------------------------ linear
def library_gemm() -> bool:
    """``NVB_BASELINE=1``: every projection runs as a cuBLAS GEMM (torch.matmul) with the activation as a
    separate kernel -- the unfused library baseline this engine is compared against."""
    return os.environ.get("NVB_BASELINE", "0") not in ("0", "", "false", "no")


def linear(x: torch.Tensor, w: torch.Tensor, act: int = ACT_NONE, out: Optional[torch.Tensor] = None,
           force_splits: int = 0, partial_ok: bool = False):
    """y = x @ w^T on the tcgen05 GEMM.  act != 0 expects gate/up rows interleaved in 128-row blocks.

    For decode-sized M the K range may be split over CTAs; with ``partial_ok`` the unreduced fp32 partials are
    returned as a ``SplitK`` for a consumer that fuses the sum, otherwise a sum kernel produces bf16."""
    if not x.is_cuda:
        return ref.linear(x, w, act)
    x = materialize(x)
    if library_gemm():
        if act != ACT_NONE:
            return act_mul(torch.matmul(x, w.t()), act, interleaved=True)
        if out is not None:
            return torch.matmul(x, w.t(), out=out)
        return torch.matmul(x, w.t())
    M, K = x.shape
    N = w.shape[0]
    ncols = N // 2 if act != ACT_NONE else N
    C = _cuda_ext()
    parts = None
    splits = 1
    if M <= 256:
        splits = force_splits if force_splits > 0 else C.gemm_splits_for(M, N, K, int(act))
        if splits > 1:
            parts = torch.empty(splits, M, N, dtype=torch.float32, device=x.device)
    if out is None:
        out = torch.empty(M, ncols, dtype=x.dtype, device=x.device)
    used = C.gemm(x, w, out, int(act), parts, int(splits if parts is not None else (force_splits or 0)),
                  error_word(x.device), bool(partial_ok and parts is not None and act == ACT_NONE))
    if parts is not None and used > 1:
        if partial_ok and act == ACT_NONE:
            add_launches(1)
            return SplitK(parts)
        add_launches(2)
        return out
    add_launches(1)
    return out


# ------------------------------------------------------------------------------------------------ SP fused linear
class SPHidden:
    """Hidden states of an SP forward before the final norm: the last producer's partial rows sit in the owners'
    receive buffers.  The LM head fuses the final all-gather + RMSNorm into its GEMM; ``materialize`` runs the
    stand-alone all-gather + norm and returns the gathered normalised rows [T, H] (a view of the workspace)."""
    __slots__ = ("part", "norm_w", "eps", "norm_mode", "_rows")

    def __init__(self, part, norm_w, eps: float, norm_mode: int):
        self.part, self.norm_w, self.eps, self.norm_mode = part, norm_w, eps, norm_mode
        self._rows = None

    @property
    def shape(self):
        return self.part.shape

    @property
    def is_cuda(self):
        return True

    def materialize(self) -> torch.Tensor:
        # once only: the owner's reduce adds the partials into the residual slice in place
        if self._rows is None:
            self._rows = self.part.ws.ag_norm(self.part, self.norm_w, self.eps, self.norm_mode, True)
        return self._rows


def linear_sp_produce(ws, x: torch.Tensor, w: torch.Tensor):
    """Row-parallel projection fused with the reduce-scatter: y = x @ w^T pushed to the row owners."""
    from ..parallel.sp import SPPartial
    x = materialize(x)
    if library_gemm() or not isinstance(w, torch.Tensor):
        y = w.linear(x) if hasattr(w, "linear") else linear(x, w)
        return ws.rs_push(materialize(y).contiguous())
    M, K = x.shape
    N = w.shape[0]
    C = _cuda_ext()
    # split K as the plain decode GEMM does: one CTA streams only ~50 GB/s of weights (measured: down_proj at TP2
    # 28 us with one CTA per 128 rows vs 10.8 us + a 5.5 us split rendezvous with 4 splits); NVB_SP_SPLITK=0 off
    splits = C.gemm_splits_for(M, N, K, 0) if os.environ.get("NVB_SP_SPLITK", "1") == "1" else 1
    parts = workspace(x.device, splits * M * N) if splits > 1 else None
    slot, plan = ws.producer_plan()
    _, grid = C.gemm_sp(x, w, None, 0, parts, error_word(x.device), False, plan, 0.0)
    add_launches(1)
    return SPPartial(ws, slot, int(grid), ws.T)


def linear_sp_consume(part, norm_w, eps: float, norm_mode: int, has_res: bool, w, act: int = ACT_NONE,
                      partial_ok: bool = False):
    """Column-parallel projection whose input is all-gathered + RMSNorm'ed in the GEMM prologue."""
    ws = part.ws
    if library_gemm() or not isinstance(w, torch.Tensor):
        x = ws.ag_norm(part, norm_w, eps, norm_mode, has_res)
        if hasattr(w, "linear"):
            y = w.linear(x)
            return act_mul(y, act, interleaved=True) if act != ACT_NONE else y
        return linear(x, w, act, partial_ok=partial_ok)
    x = ws.gather_view(part.T)
    M, K = x.shape
    N = w.shape[0]
    C = _cuda_ext()
    splits = C.gemm_splits_for(M, N, K, int(act))
    parts = torch.empty(splits, M, N, dtype=torch.float32, device=x.device) if splits > 1 else None
    out = torch.empty(M, N // 2 if act != ACT_NONE else N, dtype=torch.bfloat16, device=x.device)
    plan = ws.consumer_plan(part, norm_w, norm_mode, has_res)
    used, _ = C.gemm_sp(x, w, out, int(act), parts, error_word(x.device), bool(partial_ok and act == ACT_NONE),
                        plan, float(eps))
    if parts is not None and used > 1:
        if partial_ok and act == ACT_NONE:
            add_launches(1)
            return SplitK(parts)
        add_launches(2)
        return out
    add_launches(1)
    return out


def act_mul(x: torch.Tensor, act: int, interleaved: bool = False) -> torch.Tensor:
    x = materialize(x)
    if not x.is_cuda:
        return ref.act_mul(x, act, interleaved)
    out = torch.empty(x.shape[0], x.shape[1] // 2, dtype=x.dtype, device=x.device)
    _cuda_ext().act_mul(out, x, int(act), bool(interleaved))
    add_launches(1)
    return out


def bias_act_(x: torch.Tensor, bias: Optional[torch.Tensor], act: int = BIAS_ACT_NONE) -> torch.Tensor:
    if isinstance(x, SplitK):
        x = materialize(x)
    if not x.is_cuda:
        x.copy_(ref.bias_act(x, bias, act))
        return x
    _cuda_ext().bias_act(x, bias, int(act))
    add_launches(1)
    return x


def embedding(table: torch.Tensor, ids: torch.Tensor, scale: float = 1.0, vstart: int = 0,
              vend: Optional[int] = None) -> torch.Tensor:
    vend = table.shape[0] + vstart if vend is None else vend
    if not table.is_cuda:
        return ref.embedding(table, ids, scale, vstart, vend)
    out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device)
    _cuda_ext().embedding(out, table, ids.long(), float(scale), int(vstart), int(vend))
    add_launches(1)
    return out


def gather_rows(src: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    src = materialize(src)
    if not src.is_cuda:
        return src[idx.long()]
    out = torch.empty(idx.numel(), src.shape[1], dtype=src.dtype, device=src.device)
    _cuda_ext().gather_rows(out, src, idx.long())
    add_launches(1)
    return out


def mean_pool_l2(x: torch.Tensor, cu: torch.Tensor) -> torch.Tensor:
    if not x.is_cuda:
        return ref.mean_pool_l2(x, cu)
    out = torch.empty(cu.numel() - 1, x.shape[1], dtype=torch.float32, device=x.device)
    _cuda_ext().mean_pool_l2(out, x, cu.int())
    add_launches(1)
    return out


def sample(logits, temps, top_ks, top_ps, seeds, seq_ids, steps, softcap: float = 0.0, out=None,
           ids: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Seeded sampling per row.  ``ids`` (optional int32 [B, C]): the rows hold candidate logits, column c
    standing for vocabulary id ids[b, c] (ascending along the row); the draw is keyed and reported by id."""
    if not logits.is_cuda:
        return ref.sample(logits, temps, top_ks, top_ps, seeds, seq_ids, steps, softcap, ids=ids)
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.long, device=logits.device)
    _cuda_ext().sample(logits, temps, top_ks, top_ps, seeds, seq_ids, steps, float(softcap), out, ids)
    add_launches(1)
    return out


def shortconv(proj, weight, cu, rows, fresh, state, state_off: int):
    """LFM2 gated short conv over [B | C | x] projections with the per-sequence recurrent state."""
    proj = materialize(proj)
    if not proj.is_cuda:
        return ref.shortconv(proj, weight, cu, rows, fresh, state, state_off)
    out = torch.empty(proj.shape[0], weight.shape[0], dtype=proj.dtype, device=proj.device)
    _cuda_ext().shortconv(proj, weight, cu, rows, fresh, state, int(state_off), out)
    add_launches(1)
    return out


# ----------------------------------------------------------------------------------------------- Gemma4
def rms_norm_post_add_(x, residual: torch.Tensor, weight: Optional[torch.Tensor], eps: float, mode: int = 0,
                       post_scale: float = 1.0) -> torch.Tensor:
    """residual = (residual + rmsnorm(x) * w) * post_scale, in place."""
    x = materialize(x)
    if not residual.is_cuda:
        return ref.rms_norm_post_add(x, residual, weight, eps, mode, post_scale)
    _cuda_ext().rms_norm_post_add(x, residual, weight, float(eps), int(mode), float(post_scale))
    add_launches(1)
    return residual


def ple_combine(proj, tok: torch.Tensor, weight: torch.Tensor, eps: float, proj_scale: float,
                out_scale: float) -> torch.Tensor:
    proj = materialize(proj)
    if not proj.is_cuda:
        return ref.ple_combine(proj, tok, weight, eps, proj_scale, out_scale)
    out = torch.empty_like(tok)
    _cuda_ext().ple_combine(out, proj.contiguous(), tok, weight, float(eps), float(proj_scale), float(out_scale))
    add_launches(1)
    return out


def gate_act_mul(gate, other: torch.Tensor) -> torch.Tensor:
    """gelu_tanh(gate) * other; ``other`` may be a column slice."""
    gate = materialize(gate)
    if not gate.is_cuda:
        return ref.gate_act_mul(gate, other)
    out = torch.empty(gate.shape, dtype=gate.dtype, device=gate.device)
    _cuda_ext().gate_act_mul(out, gate, other)
    add_launches(1)
    return out


def srq_(x: torch.Tensor, scale: float) -> torch.Tensor:
    """In-place static-range activation fake-quant (no-op for scale 0)."""
    if scale == 0.0:
        return x
    if not x.is_cuda:
        x.copy_(ref.srq(x, scale))
        return x
    _cuda_ext().srq(x, float(scale))
    add_launches(1)
    return x
