"""Microbenchmark of one tensor-parallel decode layer's projections + collectives (attention excluded).

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        -m nanovllm_b200.parallel.bench_sp [--tokens 16,128] [--iters 20] [--trace]

Three arms on the Qwen3-8B shapes (H 4096, qkv 6144, I 12288; weights sharded over N ranks):
  sp      the fused sequence-parallel path: [AG + RMSNorm + qkv GEMM] [o_proj GEMM + RS]
          [AG + RMSNorm + gate_up GEMM + SiLU*up] [down GEMM + RS] (csrc/sp_comm.cuh, csrc/gemm.cu);
  ar      this engine without SP: [qkv GEMM] [o_proj GEMM] [fused all-reduce + residual + RMSNorm]
          [gate_up GEMM] [down GEMM] [fused all-reduce + residual + RMSNorm] (csrc/tp_comm.cu);
  nccl    the library baseline: cuBLAS GEMMs, NCCL all-reduce, RMSNorm and activation kernels.
Timing: ``iters`` layers captured in one CUDA graph, CUDA events around one replay after a warm-up replay and a
barrier, max over ranks.  Roofline per layer and rank: the slower of the weight bytes over the measured HBM
bandwidth and the NVLink bytes (2 reduce-scatters + 2 all-gathers of T x H bf16 rows, (R-1)/R each) over
770 GB/s per direction; the FLOPs (2 T N K) are negligible at decode sizes.
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

from .. import ops
from . import sp as spmod
from . import state as ps
from . import symm

LINK_GBS = 770.0


def _peak_hbm() -> float:
    try:
        with open(os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"])
    except Exception:  # noqa: BLE001
        return 6448.0


def _time(fn, iters: int) -> float:
    for _ in range(2):
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
    ap.add_argument("--tokens", default="16,128")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--trace", action="store_true", help="print the in-kernel phase trace of one SP layer")
    args = ap.parse_args()
    if args.trace:
        os.environ["NVB_SP_TRACE"] = "1"
    ps.init_tp("nccl", timeout_s=120)
    R, rank = ps.tp_size(), ps.tp_rank()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    H, QKV, I = 4096, 6144, 12288
    g = torch.Generator(device=dev).manual_seed(1 + rank)

    def rnd(*shape, std=0.02):
        return (torch.randn(*shape, generator=g, device=dev) * std).bfloat16()

    wqkv, wo = rnd(QKV // R, H), rnd(H, H // R)
    wgu, wd = rnd(2 * I // R, H), rnd(H, I // R)
    nw = torch.ones(H, dtype=torch.bfloat16, device=dev)
    ws_rs = spmod.SPWorkspace(256, H, dev)
    ws_ar = symm.init_workspace(256, H, dev)
    peak = _peak_hbm()
    rows = []
    for T in [int(t) for t in args.tokens.split(",")]:
        attn = rnd(T, H // R, std=0.5)
        x0 = rnd(T, H, std=0.5)
        res = rnd(T, H, std=0.5)
        ws_ar.res_buf[:T].copy_(res)

        def sp_layer(ws_sp):
            ws_sp.begin(T)
            part = ws_sp.rs_push(x0)
            ops.materialize(ops.linear_sp_consume(part, nw, 1e-6, 0, False, wqkv, partial_ok=True))
            part = ops.linear_sp_produce(ws_sp, attn, wo)
            h = ops.linear_sp_consume(part, nw, 1e-6, 0, True, wgu, ops.ACT_SILU_MUL)
            part = ops.linear_sp_produce(ws_sp, h, wd)
            ws_sp.ag_norm(part, nw, 1e-6, 0, True)

        def ar_layer():
            xn, _ = ops.rms_norm(x0, nw, 1e-6)
            ops.materialize(ops.linear(xn, wqkv, partial_ok=True))
            ops.linear(attn, wo, out=ws_ar.in_view(T))
            xn, _ = ws_ar.allreduce_norm(T, nw, 1e-6, 0, ws_ar.res_buf[:T])
            h = ops.linear(xn, wgu, ops.ACT_SILU_MUL)
            ops.linear(h, wd, out=ws_ar.in_view(T))
            ws_ar.allreduce_norm(T, nw, 1e-6, 0, ws_ar.res_buf[:T])

        res2 = res.clone()

        def nccl_layer():
            xn, _ = ops.rms_norm(x0, nw, 1e-6)
            torch.matmul(xn, wqkv.t())
            y = torch.matmul(attn, wo.t())
            dist.all_reduce(y)
            xn, _ = ops.rms_norm(y, nw, 1e-6, residual=res2)
            h = ops.act_mul(torch.matmul(xn, wgu.t()), ops.ACT_SILU_MUL, interleaved=True)
            y = torch.matmul(h, wd.t())
            dist.all_reduce(y)
            ops.rms_norm(y, nw, 1e-6, residual=res2)

        t_rs = _time(lambda: sp_layer(ws_rs), args.iters)
        t_ar = _time(ar_layer, args.iters)
        t_nc = _time(nccl_layer, args.iters)
        wbytes = (wqkv.numel() + wo.numel() + wgu.numel() + wd.numel()) * 2
        link = 4 * (R - 1) / R * T * H * 2
        roof = max(wbytes / (peak * 1e3), link / (LINK_GBS * 1e3))
        rows.append({"tokens": T, "sp_rsag_us": round(t_rs, 2),
                     "ar_us": round(t_ar, 2), "nccl_cublas_us": round(t_nc, 2),
                     "roofline_us": round(roof, 2), "sp_frac_of_roofline": round(roof / t_rs, 3),
                     "weights_MB": round(wbytes / 1e6, 1), "nvlink_MB": round(link / 1e6, 3)})
        if args.trace:
            for name, w_ in (("rsag", ws_rs),):
                for _ in range(3):  # a few traced layers back to back; the last one is reported
                    dist.barrier()
                    sp_layer(w_)
                torch.cuda.synchronize()
                rep = w_.trace_report(4)
                if rank == 0:
                    print(f"trace {name} T={T} rank 0 (us):\n{rep}", flush=True)
    ops.check_device_errors(dev)
    if rank == 0:
        for r in rows:
            print(json.dumps({"tp": R, **r}), flush=True)
    ws_os.close()
    ws_rs.close()
    symm.release_workspace()
    ps.barrier()
    ps.destroy()


if __name__ == "__main__":
    main()
