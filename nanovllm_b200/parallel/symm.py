"""Symmetric per-rank workspace for the fused tensor-parallel collectives.

Every rank allocates one zeroed device buffer with the same layout and exports it as a CUDA IPC handle; the
handles are exchanged once over the process group and each rank maps its peers' buffers, so kernels can load
from and store to any rank's buffer over NVLink.  Layout (byte offsets, identical on every rank):

  [0, 64 KiB)        signal pads  uint32 [2 phases][1024 blocks][8 ranks]
  [64 KiB, 68 KiB)   per-block epoch counters (int32 [1024], local only)
  in                 bf16 [max_tokens, hidden]  row-parallel partial sums (written by the local GEMM)
  res                bf16 [max_tokens, hidden]  residual stream
  out                bf16 [max_tokens, hidden]  normalised (all-gathered) output

``TPWorkspace.allreduce_norm`` launches the fused two-shot all-reduce + residual add + RMSNorm + all-gather
kernel (csrc/tp_comm.cu).  The workspace is only built for CUDA process groups; the NCCL path stays available
(``NVB_TP_FUSED=0``) as the unfused baseline.
"""
from __future__ import annotations

import os
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from . import state as ps

SIG_BYTES = 2 * 1024 * 8 * 4
CNT_BYTES = 1024 * 4
ALIGN = 4096
MAX_BLOCKS = 148  # at most one CTA per SM: every block of a launch is co-resident with its peers' blocks

_WS: Optional["TPWorkspace"] = None


def fused_enabled() -> bool:
    if os.environ.get("NVB_BASELINE", "0") not in ("0", "", "false", "no"):
        return False  # the library baseline all-reduces through NCCL
    return os.environ.get("NVB_TP_FUSED", "1") not in ("0", "false", "no")


def _round(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


class TPWorkspace:
    def __init__(self, max_tokens: int, hidden: int, device: torch.device):
        from .. import ops
        self.C = ops._cuda_ext()
        self.R, self.rank = ps.tp_size(), ps.tp_rank()
        self.max_tokens, self.hidden = int(max_tokens), int(hidden)
        slot = _round(self.max_tokens * self.hidden * 2)
        self.off_in = _round(SIG_BYTES + CNT_BYTES)
        self.off_res = self.off_in + slot
        self.off_out = self.off_res + slot
        total = self.off_out + slot
        with torch.cuda.device(device):
            self.buf, handle = self.C.symm_alloc(total)
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
        self.counters = self.buf[SIG_BYTES:SIG_BYTES + CNT_BYTES].view(torch.int32)
        self.sig_ptrs = list(self.bases)
        self.in_ptrs = [b + self.off_in for b in self.bases]
        self.res_ptrs = [b + self.off_res for b in self.bases]
        self.out_ptrs = [b + self.off_out for b in self.bases]
        self._no_res = [0] * self.R
        n = self.max_tokens * self.hidden * 2
        self.in_buf = self.buf[self.off_in:self.off_in + n].view(torch.bfloat16).view(self.max_tokens, self.hidden)
        self.res_buf = self.buf[self.off_res:self.off_res + n].view(torch.bfloat16).view(self.max_tokens, self.hidden)
        self.out_buf = self.buf[self.off_out:self.off_out + n].view(torch.bfloat16).view(self.max_tokens, self.hidden)
        ps.barrier()

    def fits(self, T: int, H: int) -> bool:
        return H == self.hidden and 0 < T <= self.max_tokens

    def in_view(self, T: int) -> torch.Tensor:
        return self.in_buf[:T]

    def allreduce_norm(self, T: int, weight: Optional[torch.Tensor], eps: float, mode: int,
                       residual: Optional[torch.Tensor], oneshot: int = -1
                       ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        """Sum the ranks' partials in ``in[:T]``; with ``residual``: residual += sum (kept in the workspace);
        returns (rmsnorm(result) or the plain sum for mode 3, new residual).  ``oneshot``: 1 every rank reads
        all rows from every peer, 0 two-shot (reduce-scatter + all-gather), -1 pick by message size."""
        from .. import ops
        res_ptrs = self._no_res
        res_view = None
        if residual is not None:
            res_view = self.res_buf[:T]
            if residual.data_ptr() != res_view.data_ptr():
                res_view.copy_(residual)
            res_ptrs = self.res_ptrs
        self.C.tp_allreduce_norm(self.in_ptrs, res_ptrs, self.out_ptrs, self.sig_ptrs, self.rank, int(T),
                                 self.hidden, weight if mode in (0, 1) else None, float(eps), int(mode),
                                 self.counters, ops.error_word(self.buf.device), MAX_BLOCKS, int(oneshot))
        ops.add_launches(1)
        return self.out_buf[:T], res_view

    def close(self) -> None:
        for p in self._opened:
            try:
                self.C.ipc_close(p)
            except Exception:
                pass
        self._opened = []


def init_workspace(max_tokens: int, hidden: int, device: torch.device) -> Optional[TPWorkspace]:
    """Collective: every rank must call it at the same point (after the process group is up)."""
    global _WS
    if ps.tp_size() <= 1 or not fused_enabled() or device.type != "cuda":
        _WS = None
        return None
    if _WS is not None and _WS.hidden == hidden and _WS.max_tokens >= max_tokens:
        return _WS
    _WS = TPWorkspace(max_tokens, hidden, device)
    return _WS


def workspace() -> Optional[TPWorkspace]:
    return _WS


def release_workspace() -> None:
    global _WS
    if _WS is not None:
        _WS.close()
    _WS = None
