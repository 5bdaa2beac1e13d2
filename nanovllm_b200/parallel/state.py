"""Process-group state for tensor parallelism (one process per GPU).

The reference has no parallelism beyond JVM threads; its layer names (Linear.Column/Row/Merged/Qkv,
VocabParallelEmbedding, ParallelLMHead -- nano-vllm-java/.../layers/Linear.java:269-405 and
VocabParallelEmbedding.java:21-253) describe a TP decomposition that never shards.  Here they shard for real:
``init_tp`` joins the default process group (NCCL on GPUs, Gloo on CPU for tests) and every layer reads its
rank/size from this module.  Engines run SPMD: every rank runs the same scheduler on the same requests and
the sampler is deterministic, so ranks stay in lock-step without a per-step broadcast.
"""
from __future__ import annotations

import datetime
import os
from typing import Optional

import torch
import torch.distributed as dist

_TP_SIZE = 1
_TP_RANK = 0
_GROUP = None


def init_tp(backend: Optional[str] = None, timeout_s: float = 120.0) -> None:
    """Join the default group from RANK/WORLD_SIZE/MASTER_* env vars (torchrun) when WORLD_SIZE > 1."""
    global _TP_SIZE, _TP_RANK, _GROUP
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        _TP_SIZE, _TP_RANK, _GROUP = 1, 0, None
        return
    if not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
    _TP_SIZE = dist.get_world_size()
    _TP_RANK = dist.get_rank()
    _GROUP = dist.group.WORLD


def set_tp_for_testing(rank: int, size: int, group=None) -> None:
    global _TP_SIZE, _TP_RANK, _GROUP
    _TP_RANK, _TP_SIZE, _GROUP = rank, size, group


def tp_size() -> int:
    return _TP_SIZE


def tp_rank() -> int:
    return _TP_RANK


def tp_group():
    return _GROUP


def all_reduce(x: torch.Tensor) -> torch.Tensor:
    if _TP_SIZE > 1:
        dist.all_reduce(x, group=_GROUP)
    return x


def all_gather_last(x: torch.Tensor) -> torch.Tensor:
    """Concatenate per-rank shards along the last dimension."""
    if _TP_SIZE == 1:
        return x
    x = x.contiguous()
    if x.is_cuda:
        parts = torch.empty((_TP_SIZE,) + tuple(x.shape), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(parts, x, group=_GROUP)
        chunks = list(parts.unbind(0))
    else:
        chunks = [torch.empty_like(x) for _ in range(_TP_SIZE)]
        dist.all_gather(chunks, x, group=_GROUP)
    return torch.cat(chunks, dim=-1)


def reduce_scatter_rows(x: torch.Tensor) -> torch.Tensor:
    """Sum over ranks, each rank keeps its contiguous 1/TP slice of rows (Megatron SP layout)."""
    if _TP_SIZE == 1:
        return x
    out = torch.empty((x.shape[0] // _TP_SIZE,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.reduce_scatter_tensor(out, x.contiguous(), group=_GROUP)
    return out


def all_gather_rows(x: torch.Tensor) -> torch.Tensor:
    if _TP_SIZE == 1:
        return x
    out = torch.empty((x.shape[0] * _TP_SIZE,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x.contiguous(), group=_GROUP)
    return out


def barrier() -> None:
    if _TP_SIZE > 1:
        dist.barrier(group=_GROUP)


def destroy() -> None:
    global _TP_SIZE, _TP_RANK, _GROUP
    if dist.is_initialized():
        dist.destroy_process_group()
    _TP_SIZE, _TP_RANK, _GROUP = 1, 0, None
