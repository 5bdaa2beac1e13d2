"""Collective microbenchmark: fused all-reduce + residual + RMSNorm over peer memory vs NCCL all-reduce followed
by the RMSNorm kernel, on the residual-stream shapes of a TP decode / prefill step.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        -m nanovllm_b200.parallel.bench_comm [--hidden 4096] [--tokens 1,128,2048,16384] [--iters 50]

Timing: ``iters`` calls captured in one CUDA graph, CUDA events around one replay (after a warm-up replay and a
barrier), max over ranks, microseconds per call.  The roofline of the fused path is its NVLink traffic per
rank over the measured 770 GB/s per direction: the smaller of one-shot (reads (R-1) * T*H*2 bytes) and
two-shot (reduce-scatter reads (R-1)/R * T*H*2, the all-gather writes 2 * (R-1)/R * T*H*2: new residual and
normalised rows).
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

from .. import ops
from . import state as ps
from . import symm

LINK_GBS = 770.0


def _time(fn, iters: int) -> float:
    """GPU time per call: ``iters`` calls captured in one CUDA graph (the decode path replays graphs, so host
    launch overhead is not part of the cost being compared)."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            for _ in range(iters):
                fn()
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    us = torch.tensor([a.elapsed_time(b) * 1000.0 / iters], device="cuda")
    del g
    dist.all_reduce(us, op=dist.ReduceOp.MAX)
    return float(us.item())


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--tokens", default="1,16,128,512,2048,16384")
    ap.add_argument("--iters", type=int, default=50)
    a = ap.parse_args()
    ps.init_tp("nccl", timeout_s=120)
    R, rank = ps.tp_size(), ps.tp_rank()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    Ts = [int(t) for t in a.tokens.split(",")]
    H = a.hidden
    ws = symm.init_workspace(max(Ts), H, dev)
    w = torch.ones(H, dtype=torch.bfloat16, device=dev)
    rows = []
    for T in Ts:
        part = torch.randn(T, H, device=dev).bfloat16()
        res = torch.randn(T, H, device=dev).bfloat16()
        ws.in_view(T).copy_(part)
        ws.res_buf[:T].copy_(res)

        def fused1():
            ws.allreduce_norm(T, w, 1e-6, 0, ws.res_buf[:T], oneshot=1)

        def fused2():
            ws.allreduce_norm(T, w, 1e-6, 0, ws.res_buf[:T], oneshot=0)

        y = part.clone()
        r2 = res.clone()

        def nccl():
            dist.all_reduce(y)
            ops.rms_norm(y, w, 1e-6, 0, r2)

        t_1 = _time(fused1, a.iters)
        t_2 = _time(fused2, a.iters)
        t_n = _time(nccl, a.iters)
        t_f = min(t_1, t_2)
        # fewest bytes either algorithm must move over NVLink per rank (one-shot reads R-1 full partials;
        # two-shot reads (R-1)/R of them and writes (R-1)/R of the residual and of the output)
        link_bytes = min(float(R - 1), 3.0 * (R - 1) / R) * T * H * 2
        roof_us = link_bytes / (LINK_GBS * 1e3)
        rows.append({"T": T, "H": H, "ranks": R, "oneshot_us": round(t_1, 2), "twoshot_us": round(t_2, 2),
                     "fused_us": round(t_f, 2), "nccl_plus_norm_us": round(t_n, 2),
                     "speedup": round(t_n / t_f, 2), "nvlink_bytes_per_rank": int(link_bytes),
                     "roofline_us": round(roof_us, 2), "frac_of_roofline": round(roof_us / t_f, 3)})
    ops.check_device_errors(dev)
    if rank == 0:
        for r in rows:
            print(json.dumps(r), flush=True)
    symm.release_workspace()
    ps.barrier()
    ps.destroy()


if __name__ == "__main__":
    main()
