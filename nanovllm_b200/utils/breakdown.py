"""Per-kernel device-time breakdown of engine steps (CUPTI through ``torch.profiler``).

The reference has no tracer (its only timing is the whole-generate wall clock in GenerationStats,
nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/llm/GenerationStats.java:23-63).  Here a few decode steps
(CUDA-graph replays included: CUPTI reports every kernel node of a replayed graph) are traced and the device
time is summed per kernel name and per op class, so a TP step can be split into GEMM / attention / collective /
sampler costs on each rank.  Numbers taken under the tracer are for attribution only, never a benchmark value.
"""
from __future__ import annotations

import re
from typing import Callable, Dict, List, Tuple

# op classes by kernel-name pattern, first match wins
_CLASSES: List[Tuple[str, str]] = [
    ("tp_fused", r"gemm_rs|ag_norm|sp_"),
    ("allreduce_norm", r"tp_allreduce"),
    ("nccl", r"nccl"),
    ("gemm_decode", r"gemm_decode"),
    ("gemm_prefill", r"gemm_tc"),
    ("gemm_quant", r"qgemm|qdequant"),
    ("gemm_library", r"gemm|cutlass|cublas|sm100_xmma|nvjet"),
    ("splitk_sum", r"splitk"),
    ("attention", r"paged_decode|attn|prefill_attn"),
    ("rope_kv", r"rope"),
    ("norm", r"rms_norm|layer_norm"),
    ("sampler", r"sample"),
    ("embedding", r"embedding|gather_rows"),
]


def classify(name: str) -> str:
    for cls, pat in _CLASSES:
        if re.search(pat, name, re.IGNORECASE):
            return cls
    return "other"


def kernel_breakdown(step: Callable[[], object], steps: int) -> Dict[str, object]:
    """Run ``step`` ``steps`` times under the CUDA tracer; per-step device microseconds by kernel and class."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            step()
        torch.cuda.synchronize()
    per_kernel: Dict[str, List[float]] = {}
    for ev in prof.events():
        if ev.device_type is None or "cuda" not in str(ev.device_type).lower():
            continue
        dur = getattr(ev, "device_time", None)
        if dur is None:
            dur = getattr(ev, "cuda_time", 0.0)
        if not dur:
            continue
        slot = per_kernel.setdefault(ev.name, [0.0, 0])
        slot[0] += float(dur)
        slot[1] += 1
    kernels = sorted(((n, t / steps, c // steps) for n, (t, c) in per_kernel.items()), key=lambda r: -r[1])
    classes: Dict[str, float] = {}
    for n, t, _ in kernels:
        classes[classify(n)] = classes.get(classify(n), 0.0) + t
    return {"steps": steps, "total_us": sum(t for _, t, _ in kernels),
            "classes_us": dict(sorted(classes.items(), key=lambda kv: -kv[1])),
            "kernels": [{"name": n[:120], "us_per_step": round(t, 2), "launches_per_step": c} for n, t, c in kernels]}


def format_breakdown(bd: Dict[str, object], top: int = 25) -> str:
    lines = [f"device time per step: {bd['total_us']:.1f} us (sum of kernel durations, {bd['steps']} steps traced)",
             "by class:"]
    for cls, t in bd["classes_us"].items():
        lines.append(f"  {cls:<16} {t:10.1f} us  {100.0 * t / max(bd['total_us'], 1e-9):5.1f} %")
    lines.append(f"top {top} kernels (us per step, launches per step):")
    for k in bd["kernels"][:top]:
        lines.append(f"  {k['us_per_step']:10.1f}  {k['launches_per_step']:5d}  {k['name']}")
    return "\n".join(lines)
