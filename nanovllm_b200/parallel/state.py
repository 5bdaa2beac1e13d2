"""Process-group state for tensor parallelism (one process per GPU).

The reference has no parallelism beyond JVM threads; its layer names (Linear.Column/Row/Merged/Qkv,
VocabParallelEmbedding, ParallelLMHead -- nano-vllm-java/.../layers/Linear.java:269-405 and
VocabParallelEmbedding.java:21-253) describe a TP decomposition that never shards.  Here they shard for real:
``init_tp`` joins the default process group (NCCL on GPUs, Gloo on CPU for tests) and every layer reads its
rank/size from this module.  Engines run SPMD: every rank runs the same scheduler on the same requests and
the sampler is deterministic, so ranks stay in lock-step without a per-step broadcast.

Failure propagation: a rank whose step fails (a device wait that gave up, a host exception) publishes the
reason under one key of the rendezvous TCP store (``signal_abort``).  Every rank runs a watcher thread blocked
on that key, so the others learn of it on the host without a per-step round trip; ``check_abort`` (called at
the start of every engine step) then raises ``TensorParallelAbort`` before the rank launches another kernel or
collective.  A rank already blocked inside a collective with the failed peer is released by the process
group's timeout and reports the same abort reason.
"""
from __future__ import annotations

import atexit
import datetime
import os
import threading
from typing import Optional

import torch
import torch.distributed as dist

from ..exceptions import TensorParallelAbort

_TP_SIZE = 1
_TP_RANK = 0
_GROUP = None

_ABORT_KEY = "nanovllm_b200/abort"
_ABORT = threading.Event()
_ABORT_REASON = [""]
_WATCH_STOP = threading.Event()
_WATCH: Optional[threading.Thread] = None
_STORE = None


def _store():
    """A client of the rendezvous TCP store (MASTER_ADDR:MASTER_PORT) owned by this module."""
    global _STORE
    if _STORE is None:
        _STORE = dist.TCPStore(os.environ.get("MASTER_ADDR", "127.0.0.1"), int(os.environ["MASTER_PORT"]),
                               is_master=False, timeout=datetime.timedelta(seconds=30), wait_for_workers=False)
    return _STORE


def _watch_abort() -> None:
    try:
        st = dist.TCPStore(os.environ.get("MASTER_ADDR", "127.0.0.1"), int(os.environ["MASTER_PORT"]),
                           is_master=False, timeout=datetime.timedelta(seconds=30), wait_for_workers=False)
    except Exception:  # noqa: BLE001 - no store to watch (single process); nothing to propagate
        return
    while not _WATCH_STOP.is_set():
        try:
            if not st.check([_ABORT_KEY]):  # non-blocking: a blocking wait would log every time it times out
                _WATCH_STOP.wait(0.2)
                continue
        except Exception:  # noqa: BLE001 - the store is gone (the job is shutting down): nothing left to watch
            return
        try:
            _ABORT_REASON[0] = st.get(_ABORT_KEY).decode("utf-8", "replace")
        except Exception:  # noqa: BLE001
            _ABORT_REASON[0] = "a peer rank aborted"
        _ABORT.set()
        return


def _stop_watcher() -> None:
    global _WATCH
    _WATCH_STOP.set()
    if _WATCH is not None:
        _WATCH.join(timeout=2.0)
    _WATCH = None


def _start_watcher() -> None:
    global _WATCH
    if _WATCH is not None or "MASTER_PORT" not in os.environ:
        return
    _ABORT.clear()
    _WATCH_STOP.clear()
    _WATCH = threading.Thread(target=_watch_abort, name="nvb-tp-abort-watch", daemon=True)
    _WATCH.start()
    atexit.register(_stop_watcher)  # stop it before interpreter shutdown tears the store client down


def signal_abort(reason: str) -> None:
    """Tell every rank that this rank's step failed (idempotent; the first reason wins)."""
    if _TP_SIZE <= 1:
        return
    _ABORT_REASON[0] = _ABORT_REASON[0] or f"rank {_TP_RANK}: {reason}"
    _ABORT.set()
    try:
        st = _store()
        st.compare_set(_ABORT_KEY, "", f"rank {_TP_RANK}: {reason}")
    except Exception:  # noqa: BLE001 - the store is gone too: the peers' collective timeouts end them
        pass


def abort_requested() -> bool:
    return _ABORT.is_set()


def peer_aborted(wait_s: float = 0.0) -> bool:
    """Whether a peer has signalled a failure, asking the store directly (not only the watcher's last poll) and
    waiting up to ``wait_s`` for the signal to appear."""
    if _ABORT.is_set():
        return True
    if _TP_SIZE <= 1 or "MASTER_PORT" not in os.environ:
        return False
    import time
    deadline = time.monotonic() + wait_s
    while True:
        try:
            st = _store()
            if st.check([_ABORT_KEY]):
                _ABORT_REASON[0] = st.get(_ABORT_KEY).decode("utf-8", "replace")
                _ABORT.set()
                return True
        except Exception:  # noqa: BLE001 - store unreachable: nothing to learn from it
            return False
        if time.monotonic() >= deadline:
            return False
        time.sleep(0.05)


def abort_reason() -> str:
    return _ABORT_REASON[0]


def check_abort() -> None:
    """Raise TensorParallelAbort when any rank has signalled a failure (called between engine steps)."""
    if _ABORT.is_set():
        raise TensorParallelAbort(_ABORT_REASON[0] or "a peer rank aborted")


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
    _start_watcher()


_CTRL = None


def control_group():
    """A Gloo group over all ranks for host-side control messages (step plans).  Created on first use, which must
    happen at the same point on every rank; its timeout is long because a serving worker waits for the next
    plan for as long as the server is idle (a failed peer is noticed through the abort flag instead)."""
    global _CTRL
    if _CTRL is None:
        _CTRL = dist.new_group(backend="gloo", timeout=datetime.timedelta(days=7))
    return _CTRL


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


def barrier() -> None:
    if _TP_SIZE > 1:
        dist.barrier(group=_GROUP)


def destroy() -> None:
    global _TP_SIZE, _TP_RANK, _GROUP, _STORE, _CTRL
    _stop_watcher()
    _STORE = None
    _CTRL = None
    if dist.is_initialized():
        dist.destroy_process_group()
    _TP_SIZE, _TP_RANK, _GROUP = 1, 0, None
