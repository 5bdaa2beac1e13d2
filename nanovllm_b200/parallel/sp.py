"""Sequence-parallel (SP) workspace for the fused tensor-parallel decode path.

Between the tensor-parallel regions of a layer the residual stream is sharded by token rows: with T tokens in a
step and R ranks, rank r owns rows [r*per, min(T, (r+1)*per)), per = ceil(T/R).  Row-parallel producers (the
vocab-parallel embedding, o_proj, down_proj) push their partial rows to the owners (reduce-scatter inside the
GEMM epilogue); the next column-parallel consumer (qkv, gate_up, the LM head) reduces its slice, adds the
residual, applies RMSNorm and broadcasts the normalised rows to every rank (all-gather inside the GEMM
prologue).  The kernels and the flag protocol are in ``csrc/sp_comm.cuh``; this module owns the buffers.

Every rank allocates one symmetric buffer with the same layout (exported as a CUDA IPC handle and mapped by
its peers once):

  [0, 256)                 epoch (uint32, local; bumped once per SP forward by ``begin``)
  rs_flags                 uint32 [slots][8][256]    one flag per (source rank, producer CTA) per slot
  ag_flags                 uint32 [slots][256]       one flag per gathered row per slot
  split_flags              uint32 [slots][256]       split-K rendezvous of a producer's CTAs (local)
  recv                     bf16   [R][per_max][H]    partial rows pushed to this rank (its SP slice)
  gather                   bf16   [max_tokens][H]    normalised rows of all ranks (the consumer GEMM's input)
  residual                 bf16   [per_max][H]       this rank's slice of the residual stream
  exch / exch_flags        (f32, u32) [R][256] and uint32 [R][256]: the distributed greedy sampler's exchange

A forward takes its flag slots in call order (``producer_plan`` / ``consumer_plan``), so the same graph replays
the same slots with a new epoch.  The reference names the TP decomposition (nano-vllm-java/.../layers/
Linear.java:269-405, VocabParallelEmbedding.java:21-253) but never shards; nothing here mirrors its code.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist

from . import state as ps

MAX_RANKS = 8
MAX_PROD = 256
MAX_ROWS = 256
SLOTS = 256
ALIGN = 4096

_WS: Optional["SPWorkspace"] = None


def _round(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


def sp_enabled() -> bool:
    """The fused sequence-parallel decode path, ``NVB_SP=1``.  Off by default: at TP2 on B200 the replicated-
    residual path (decode GEMM writing its partial into symmetric memory -> fused all-reduce + residual + RMSNorm
    kernel) measured faster (11.0k vs 10.0k decode tok/s), because each SP junction serialises two NVLink
    hand-offs.  ``NVB_BASELINE=1`` turns every fused collective off."""
    if os.environ.get("NVB_BASELINE", "0") not in ("0", "", "false", "no"):
        return False
    if os.environ.get("NVB_TP_FUSED", "1") in ("0", "false", "no"):
        return False
    return os.environ.get("NVB_SP", "0") not in ("0", "false", "no")


@dataclass
class SPPartial:
    """A row-parallel partial that producers pushed into flag slot ``slot`` with ``n_prod`` CTAs per rank."""
    ws: "SPWorkspace"
    slot: int
    n_prod: int
    T: int

    @property
    def shape(self):
        return (self.T, self.ws.hidden)

    @property
    def is_cuda(self):
        return True


class SPWorkspace:
    def __init__(self, max_tokens: int, hidden: int, device: torch.device, wait_ns: int = 0):
        from .. import ops
        self.C = ops._cuda_ext()
        self.R, self.rank = ps.tp_size(), ps.tp_rank()
        assert self.R <= MAX_RANKS, "at most 8 ranks"
        self.max_tokens = min(int(max_tokens), MAX_ROWS)
        self.hidden = int(hidden)
        # reduce-scatter to the row owner, then all-gather of the normalised rows (two hand-offs, 2 (R-1)/R x the
        # bytes); every source's slot holds up to max_tokens rows
        self.per_max = self.max_tokens
        self.wait_ns = int(wait_ns)
        H = self.hidden
        self.off_rs = 256
        self.off_ag = self.off_rs + _round(SLOTS * MAX_RANKS * MAX_PROD * 4)
        self.off_split = self.off_ag + _round(SLOTS * MAX_ROWS * 4)
        self.off_recv = self.off_split + _round(SLOTS * MAX_PROD * 4)
        self.off_gather = self.off_recv + _round(self.R * self.per_max * H * 2)
        self.off_res = self.off_gather + _round(MAX_ROWS * H * 2)
        self.off_exch = self.off_res + _round(self.per_max * H * 2)
        self.off_xflag = self.off_exch + _round(MAX_RANKS * MAX_ROWS * 8)
        total = self.off_xflag + _round(MAX_RANKS * MAX_ROWS * 4)
        with torch.cuda.device(device):
            self.buf, handle = self.C.symm_alloc(total)
        self.device = self.buf.device
        handles: List[Optional[bytes]] = [None] * self.R
        dist.all_gather_object(handles, bytes(handle.numpy().tobytes()), group=ps.tp_group())
        self.bases: List[int] = []
        self._opened: List[int] = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.bases.append(self.buf.data_ptr())
            else:
                ptr = self.C.ipc_open(torch.frombuffer(bytearray(h), dtype=torch.uint8))
                self._opened.append(ptr)
                self.bases.append(ptr)
        b = self.buf.data_ptr()
        self.epoch_ptr = b
        self.gather_buf = self.buf[self.off_gather:self.off_gather + MAX_ROWS * H * 2].view(torch.bfloat16).view(MAX_ROWS, H)
        self.res_buf = self.buf[self.off_res:self.off_res + self.per_max * H * 2].view(torch.bfloat16).view(self.per_max, H)
        self.slot = 0
        self.T = 0
        self.per = 0
        self.sample_epoch = 0
        # optional phase trace of CTA 0 of every fused kernel (NVB_SP_TRACE=1): int64 [SLOTS][2][16] globaltimer
        # stamps, row 0 the slot's producer, row 1 its consumer (see ``trace_report``)
        self.trace = None
        if os.environ.get("NVB_SP_TRACE", "0") == "1":
            self.trace = torch.zeros(SLOTS, 2, 16, dtype=torch.int64, device=self.device)
        ps.barrier()

    # ------------------------------------------------------------------ per forward
    def fits(self, T: int, H: int) -> bool:
        return H == self.hidden and 0 < T <= self.max_tokens

    def begin(self, T: int) -> None:
        """Start an SP forward of T tokens: bump the epoch (one tiny kernel) and restart the slot sequence."""
        self.T = int(T)
        self.per = (self.T + self.R - 1) // self.R
        self.slot = 0
        self.C.sp_begin(self.epoch_ptr)
        from .. import ops
        ops.add_launches(1)

    def owned_rows(self) -> int:
        r0 = self.rank * self.per
        return max(0, min(self.T, r0 + self.per) - r0)

    def gather_view(self, T: Optional[int] = None) -> torch.Tensor:
        return self.gather_buf[:(T or self.T)]

    def residual_view(self) -> torch.Tensor:
        """This rank's residual rows (valid after the last consumer of the forward ran): its SP slice."""
        return self.res_buf[:self.owned_rows()]

    def owned_range(self):
        """Global rows [r0, r1) of ``residual_view``."""
        r0 = self.rank * self.per
        return r0, r0 + self.owned_rows()

    def _plan(self, mode: int, slot: int, n_prod: int = 0, has_res: int = 0, norm_mode: int = 2,
              norm_w: Optional[torch.Tensor] = None) -> List[int]:
        assert slot < SLOTS, "too many SP call sites in one forward"
        rs = [p + self.off_rs + slot * MAX_RANKS * MAX_PROD * 4 for p in self.bases]
        ag = [p + self.off_ag + slot * MAX_ROWS * 4 for p in self.bases]
        recv = [p + self.off_recv for p in self.bases]
        gather = [p + self.off_gather for p in self.bases]
        pad = [0] * (MAX_RANKS - self.R)
        me = self.bases[self.rank]
        trace = 0
        if self.trace is not None:
            trace = self.trace.data_ptr() + (slot * 2 + (1 if mode == 1 else 0)) * 16 * 8
        return ([mode, self.rank, self.R, self.T, self.per, self.per_max, self.hidden, int(n_prod), int(has_res),
                 int(norm_mode), self.wait_ns, self.epoch_ptr, me + self.off_split + slot * MAX_PROD * 4,
                 me + self.off_recv, rs[self.rank], me + self.off_res,
                 norm_w.data_ptr() if norm_w is not None else 0]
                + recv + pad + rs + pad + gather + pad + ag + pad + [trace])

    def producer_plan(self):
        """(slot, plan) for the next reduce-scatter producer of this forward."""
        slot = self.slot
        self.slot += 1
        return slot, self._plan(2, slot)

    def consumer_plan(self, part: SPPartial, norm_w: Optional[torch.Tensor], norm_mode: int, has_res: bool):
        return self._plan(1, part.slot, part.n_prod, 1 if has_res else 0, norm_mode, norm_w)

    # ------------------------------------------------------------------ stand-alone kernels
    def ag_norm(self, part: SPPartial, norm_w, eps: float, norm_mode: int, has_res: bool) -> torch.Tensor:
        """All-gather + RMSNorm as its own kernel; returns the gathered normalised rows [T, H] (a view)."""
        from .. import ops
        self.C.sp_ag_norm(self.consumer_plan(part, norm_w, norm_mode, has_res), float(eps), ops.error_word(self.device))
        ops.add_launches(1)
        return self.gather_view(part.T)

    def rs_push(self, x: torch.Tensor) -> SPPartial:
        """Reduce-scatter of a materialised partial [T, H] (no fused GEMM epilogue available)."""
        from .. import ops
        slot, plan = self.producer_plan()
        n = self.C.sp_rs_push(x, plan)
        ops.add_launches(1)
        return SPPartial(self, slot, int(n), self.T)

    def argmax(self, logits: torch.Tensor, ncols: int, col0: int, softcap: float = 0.0) -> torch.Tensor:
        """Greedy tokens [T] over the vocab-parallel logits: each rank's slice is [T, >= ncols] for global token
        ids [col0, col0 + ncols); exact (ties to the lowest id), 8 bytes per row and rank over NVLink."""
        from .. import ops
        self.sample_epoch += 1  # host-side, equal on every rank (ranks step in lock-step)
        out = torch.empty(logits.shape[0], dtype=torch.long, device=logits.device)
        self.C.sp_argmax(logits, int(ncols), int(col0), float(softcap), out, self.rank,
                         [p + self.off_exch for p in self.bases], [p + self.off_xflag for p in self.bases],
                         self.sample_epoch & 0x7FFFFFFF, self.wait_ns, ops.error_word(self.device))
        ops.add_launches(1)
        return out

    def trace_report(self, slots: int) -> str:
        """Phase durations (us) of CTA 0 of each fused kernel of the last traced forward (NVB_SP_TRACE=1).

        producer: mainloop (pdl wait -> accumulators ready), split rendezvous, reduce + push, publish;
        consumer: RS wait (pdl wait -> all partial flags), own rows (reduce + norm + broadcast), AG wait (-> all
        rows here), mainloop; ``hop``: producer publish -> consumer saw every flag (includes the peers' lag)."""
        if self.trace is None:
            return "trace off (set NVB_SP_TRACE=1 before the workspace is built)"
        t = self.trace.cpu().double() / 1000.0
        lines = ["slot  prod: main  rdv   push  pub  | cons: rswait own   agwait main  | hop"]
        for k in range(slots):
            p, c = t[k, 0], t[k, 1]

            def d(a, b, row):
                return f"{(row[b] - row[a]).item():6.1f}" if row[a] > 0 and row[b] > 0 else "     -"
            hop = f"{(c[2] - p[8]).item():6.1f}" if c[2] > 0 and p[8] > 0 else "     -"
            lines.append(f"{k:4d}  {d(1, 5, p)}{d(5, 6, p)}{d(6, 7, p)}{d(7, 8, p)} |       {d(1, 2, c)}{d(2, 3, c)}"
                         f"{d(3, 4, c)}{d(4, 5, c)} | {hop}")
        return "\n".join(lines)

    def close(self) -> None:
        for p in self._opened:
            try:
                self.C.ipc_close(p)
            except Exception:  # noqa: BLE001
                pass
        self._opened = []


def init_workspace(max_tokens: int, hidden: int, device: torch.device) -> Optional[SPWorkspace]:
    """Collective: every rank must call it at the same point (after the process group is up)."""
    global _WS
    if ps.tp_size() <= 1 or not sp_enabled() or device.type != "cuda":
        _WS = None
        return None
    if _WS is not None and _WS.hidden == hidden and _WS.max_tokens >= min(max_tokens, MAX_ROWS):
        return _WS
    _WS = SPWorkspace(max_tokens, hidden, device)
    return _WS


def workspace() -> Optional[SPWorkspace]:
    return _WS


def active_for(T: int, H: int, is_cuda: bool) -> Optional[SPWorkspace]:
    """The workspace when this forward (T tokens of width H) takes the SP path, else None."""
    ws = _WS
    if ws is None or not is_cuda or not sp_enabled() or not ws.fits(T, H):
        return None
    return ws


def release_workspace() -> None:
    global _WS
    if _WS is not None:
        _WS.close()
    _WS = None
