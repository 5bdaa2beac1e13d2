"""NVTX ranges around engine phases, for timeline tools (Nsight Systems and the like).

``NVB_NVTX=1`` turns them on: every engine step is a range (``step:prefill`` / ``step:decode``) with nested
ranges for scheduling, input preparation, the forward (or CUDA-graph replay), sampling and post-processing.
Off (the default) the context manager costs one dictionary lookup.  The reference has no tracer; its only
timing is the whole-generate wall clock (nano-vllm-java/.../llm/GenerationStats.java:23-63).
"""
from __future__ import annotations

import contextlib
import os

_ON = os.environ.get("NVB_NVTX", "0") == "1"


def enabled() -> bool:
    return _ON


def set_enabled(on: bool) -> None:
    global _ON
    _ON = bool(on)


@contextlib.contextmanager
def nvtx(name: str):
    if not _ON:
        yield
        return
    import torch
    if not torch.cuda.is_available():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()
