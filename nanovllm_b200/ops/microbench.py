"""Per-kernel microbenchmarks (CUDA-event timed, L2-defeating operand rotation) with roofline fractions.

    python -m nanovllm_b200.ops.microbench [--only gemm,decode,prefill,norm,rope,sample] [--iters N]

Each case allocates enough copies of its operands that one sweep over them exceeds the 126 MB L2, and cycles
through the copies between timed launches, so DRAM numbers are not L2 hits.  Bandwidth fractions are against
MEASURED_PEAKS.json (hbm_gbs, bf16_tflops) when present, else the pool fallback (6650 GB/s, 1590 TFLOP/s).
GEMM cases also time torch.matmul (cuBLAS) on the same operands for comparison.
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from .. import ops

L2_BYTES = 126 << 20


def peaks():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def _copies(bytes_per_copy: int) -> int:
    return max(1, min(64, (3 * L2_BYTES) // max(1, bytes_per_copy) + 1))


def time_fn(fns, iters: int, warmup: int = 3) -> float:
    """Mean GPU microseconds per call, cycling through ``fns`` (one per operand copy).  The ``iters`` calls are
    captured in one CUDA graph and replayed, so host launch overhead (Python, argument marshalling) is not
    counted -- the engine's decode path replays graphs the same way."""
    for i in range(warmup):
        fns[i % len(fns)]()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            for i in range(iters):
                fns[i % len(fns)]()
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    del g
    return a.elapsed_time(b) * 1000.0 / iters


def bench_gemm(M, N, K, iters, act=0, splits=0):
    dev = "cuda"
    wbytes = N * K * 2
    n = _copies(wbytes + M * K * 2)
    ws = [(torch.randn(N, K, device=dev) * 0.02).bfloat16() for _ in range(n)]
    xs = [torch.randn(M, K, device=dev).bfloat16() for _ in range(n)]
    ours = time_fn([lambda w=w, x=x: ops.linear(x, w, act, force_splits=splits) for w, x in zip(ws, xs)], iters)
    cublas = time_fn([lambda w=w, x=x: torch.matmul(x, w.t()) for w, x in zip(ws, xs)], iters)
    # the model's consumers (add+RMSNorm, RoPE, the TP all-reduce) sum split-K slices themselves: time the
    # GEMM kernel alone as well when it splits
    sp = splits or (ops._cuda_ext().gemm_splits_for(M, N, K, act) if M <= 256 else 1)
    gemm_only = None
    if sp > 1 and not act:
        gemm_only = time_fn([lambda w=w, x=x: ops.linear(x, w, act, force_splits=splits, partial_ok=True)
                             for w, x in zip(ws, xs)], iters)
    out_cols = N // 2 if act else N
    byts = wbytes + M * K * 2 + M * out_cols * 2
    flops = 2.0 * M * N * K
    return {"case": f"gemm M={M} N={N} K={K}" + (" act" if act else "") + (f" S={splits}" if splits else ""),
            "us": round(ours, 2), "splits": sp,
            "gemm_only_us": None if gemm_only is None else round(gemm_only, 2),
            "cublas_us": round(cublas, 2), "TBps": round(byts / ours / 1e6, 3), "TFLOPs": round(flops / ours / 1e6, 1)}


def bench_qgemm(ggml_type, M, N, K, iters):
    """Dequant-fused GEMM on packed GGUF weights vs cuBLAS on the same weights in bf16; bandwidth counts the
    packed bytes actually streamed (tile-major repack) plus activations and output."""
    import numpy as np
    from ..loaders import dequant as DQ
    from ..loaders.gguf import pack_random_blocks
    from .quant import FUSED_TYPES, GgufPacked
    dev = "cuda"
    raw = torch.from_numpy(np.frombuffer(pack_random_blocks(ggml_type, (N, K), 0), dtype=np.uint8).copy()).to(dev)
    base = GgufPacked(raw, ggml_type, N, K)
    pbytes = base.tiles().numel()
    n = _copies(pbytes + M * K * 2)
    ws = [GgufPacked(raw, ggml_type, N, K) for _ in range(n)]
    for w in ws:
        w._tiles = base.tiles().clone()
    xs = [torch.randn(M, K, device=dev).bfloat16() for _ in range(n)]
    ours = time_fn([lambda w=w, x=x: w.linear(x) for w, x in zip(ws, xs)], iters)
    ours_p = time_fn([lambda w=w, x=x: w.linear(x, partial_ok=True) for w, x in zip(ws, xs)], iters)
    dense = base.dense_cuda()
    nd = _copies(N * K * 2 + M * K * 2)
    ds = [dense.clone() for _ in range(nd)]
    cublas = time_fn([lambda w=w, x=x: torch.matmul(x, w.t()) for w, x in zip(ds, [xs[i % n] for i in range(nd)])], iters)
    byts = pbytes + M * K * 2 + M * N * 2
    return {"case": f"qgemm {DQ.type_name(ggml_type)} M={M} N={N} K={K}", "us": round(ours, 2),
            "gemm_only_us": round(ours_p, 2), "cublas_bf16_us": round(cublas, 2),
            "speedup_vs_bf16_cublas": round(cublas / ours, 2), "packed_MB": round(pbytes / 1e6, 2),
            "TBps": round(byts / ours_p / 1e6, 3)}


def trace_qgemm(ggml_type, M, N, K):
    """Per-role clock64 timeline of CTA 0 of one dequant-fused GEMM launch (cycles from the end of set-up):
    for every row step the producer's ring slot free time, each dequant group's (packed data ready, TMEM slot
    free, decoded) times and the MMA waiter's (operands seen, handed to the issuer) times; then the per-unit
    epilogue."""
    import numpy as np
    from ..loaders.gguf import pack_random_blocks
    from .quant import GgufPacked
    C = ops._cuda_ext()
    raw = torch.from_numpy(np.frombuffer(pack_random_blocks(ggml_type, (N, K), 0), dtype=np.uint8).copy()).cuda()
    w = GgufPacked(raw, ggml_type, N, K)
    x = torch.randn(M, K, device="cuda").bfloat16()
    for _ in range(3):
        w.linear(x)
    torch.cuda.synchronize()
    tr = torch.zeros(6, 64, 4, dtype=torch.int64, device="cuda")
    torch.empty(2 * L2_BYTES, dtype=torch.uint8, device="cuda").fill_(1)  # the weights come from DRAM
    C.qgemm_set_trace(tr)
    try:
        w.linear(x)
        torch.cuda.synchronize()
    finally:
        C.qgemm_set_trace(None)
    t = tr.cpu()
    t0 = int(t[5, 0, 0])
    rel = lambda v: int(v) - t0 if int(v) else -1
    lines = []
    for it in range(64):
        mma_ready, mma_done = rel(t[1, it, 0]), rel(t[1, it, 1])
        if mma_ready < 0 and mma_done < 0:
            break
        g = it & 1
        lines.append(f"step {it:2d}: producer slot {rel(t[0, it, 0]):7d} | dequant g{g} data {rel(t[2 + g, it, 0]):7d} "
                     f"slot {rel(t[2 + g, it, 1]):7d} decoded {rel(t[2 + g, it, 2]):7d} | operands seen {mma_ready:7d} "
                     f"handed to MMA {mma_done:7d}")
    for u in range(64):
        if int(t[4, u, 0]) == 0:
            break
        lines.append(f"unit {u:2d}: epilogue start {rel(t[4, u, 0]):7d} end {rel(t[4, u, 1]):7d}")
    return lines


def bench_decode(B, ctx, nq, nkv, hd, iters):
    dev = "cuda"
    BS = 256
    nblk = (ctx + BS - 1) // BS
    kv_bytes = 2 * B * ctx * nkv * hd * 2
    n = _copies(kv_bytes)
    caches = []
    for _ in range(n):
        kc = torch.randn(B * nblk, nkv, BS, hd, device=dev).bfloat16()
        vc = torch.randn(B * nblk, nkv, BS, hd, device=dev).bfloat16()
        caches.append((kc, vc))
    bt = torch.arange(B * nblk, device=dev, dtype=torch.int32).view(B, nblk)
    lens = torch.full((B,), ctx, device=dev, dtype=torch.int32)
    q = torch.randn(B, nq, hd, device=dev).bfloat16()
    scratch = torch.empty(ops.decode_scratch_numel(B, nq, nkv, hd, ctx) + 1, device=dev)
    us = time_fn([lambda c=c: ops.paged_decode(q, c[0], c[1], bt, lens, hd ** -0.5, max_len=ctx, scratch=scratch)
                  for c in caches], iters)
    return {"case": f"decode_attn B={B} ctx={ctx} nq={nq} nkv={nkv} hd={hd}", "us": round(us, 2),
            "TBps": round(kv_bytes / us / 1e6, 3)}


def bench_prefill(T, nq, nkv, hd, iters):
    dev = "cuda"
    BS = 256
    nblk = (T + BS - 1) // BS
    kc = torch.randn(nblk, nkv, BS, hd, device=dev).bfloat16()
    vc = torch.randn(nblk, nkv, BS, hd, device=dev).bfloat16()
    bt = torch.arange(nblk, device=dev, dtype=torch.int32).view(1, nblk)
    q = torch.randn(T, nq, hd, device=dev).bfloat16()
    cu = torch.tensor([0, T], device=dev, dtype=torch.int32)
    us = time_fn([lambda: ops.prefill_attention(q, cu, cu, T, nq, nkv, hd, hd ** -0.5, 0.0, 0, True, kc, vc, bt)],
                 iters)
    flops = 4.0 * T * T / 2 * hd * nq
    return {"case": f"prefill_attn T={T} nq={nq} nkv={nkv} hd={hd} causal", "us": round(us, 2),
            "TFLOPs": round(flops / us / 1e6, 1)}


def bench_norm(T, H, iters):
    dev = "cuda"
    n = _copies(3 * T * H * 2)
    xs = [torch.randn(T, H, device=dev).bfloat16() for _ in range(n)]
    rs = [torch.randn(T, H, device=dev).bfloat16() for _ in range(n)]
    w = torch.ones(H, device=dev).bfloat16()
    us = time_fn([lambda x=x, r=r: ops.rms_norm(x, w, 1e-6, 0, r) for x, r in zip(xs, rs)], iters)
    return {"case": f"add_rms_norm T={T} H={H}", "us": round(us, 2), "TBps": round(4 * T * H * 2 / us / 1e6, 3)}


def bench_rope(T, nq, nkv, hd, iters):
    dev = "cuda"
    qkv = torch.randn(T, (nq + 2 * nkv) * hd, device=dev).bfloat16()
    pos = torch.arange(T, device=dev)
    cs = ops.ref.rope_cos_sin(hd, T + 1, 1e6, device=dev)
    nb = (T + 255) // 256
    kc = torch.zeros(nb, nkv, 256, hd, device=dev).bfloat16()
    vc = torch.zeros_like(kc)
    slots = torch.arange(T, device=dev, dtype=torch.int32)
    w = torch.ones(hd, device=dev).bfloat16()
    us = time_fn([lambda: ops.qk_norm_rope_store(qkv, pos, cs, w, w, 0, False, 1e-6, kc, vc, slots, nq, nkv, hd)],
                 iters)
    return {"case": f"qk_norm_rope_store T={T} nq={nq} nkv={nkv} hd={hd}", "us": round(us, 2),
            "TBps": round(2 * T * (nq + 2 * nkv) * hd * 2 / us / 1e6, 3)}


def bench_misc(iters):
    """The small memory-bound kernels: gated activation, embedding gather, mean-pool + L2, LFM2 short conv."""
    dev = "cuda"
    rows = []
    x = torch.randn(128, 24576, device=dev).bfloat16()
    us = time_fn([lambda: ops.act_mul(x, ops.ACT_SILU_MUL, interleaved=True)], iters)
    rows.append({"case": "act_mul silu T=128 2x12288", "us": round(us, 2), "TBps": round(128 * 24576 * 3 / us / 1e6, 3)})
    table = torch.randn(151936, 4096, device=dev).bfloat16()
    ids = torch.randint(0, 151936, (128,), device=dev)
    us = time_fn([lambda: ops.embedding(table, ids)], iters)
    rows.append({"case": "embedding 128 ids H=4096", "us": round(us, 2), "TBps": round(128 * 4096 * 4 / us / 1e6, 3)})
    xb = torch.randn(256 * 256, 384, device=dev).bfloat16()
    cu = torch.arange(0, 256 * 256 + 1, 256, device=dev, dtype=torch.int32)
    us = time_fn([lambda: ops.mean_pool_l2(xb, cu)], iters)
    rows.append({"case": "mean_pool_l2 256 seqs x 256 tok H=384", "us": round(us, 2),
                 "TBps": round(xb.numel() * 2 / us / 1e6, 3)})
    H, L, B = 2048, 3, 128
    proj = torch.randn(B, 3 * H, device=dev).bfloat16()
    w = torch.randn(H, L, device=dev)
    cus = torch.arange(0, B + 1, device=dev, dtype=torch.int32)
    srows = torch.arange(B, device=dev)
    fresh = torch.zeros(B, dtype=torch.bool, device=dev)
    state = torch.randn(B, 2 * (L - 1) * H, device=dev)
    us = time_fn([lambda: ops.shortconv(proj, w, cus, srows, fresh, state, (L - 1) * H)], iters)
    rows.append({"case": "shortconv decode B=128 H=2048 L=3", "us": round(us, 2),
                 "TBps": round((proj.numel() * 2 + B * H * 2 + 2 * B * (L - 1) * H * 4) / us / 1e6, 3)})
    return rows


def bench_sample(B, V, iters, greedy, top_k=50, temp=0.8):
    dev = "cuda"
    logits = torch.randn(B, V, device=dev).bfloat16()
    f = lambda n, v, dt: torch.full((n,), v, device=dev, dtype=dt)  # noqa: E731
    k = 1 if greedy else top_k
    args = (f(B, temp, torch.float32), f(B, k, torch.int32), f(B, 1.0 if greedy else 0.9, torch.float32),
            f(B, 1, torch.int64), torch.arange(B, device=dev), f(B, 3, torch.int32))
    us = time_fn([lambda: ops.sample(logits, *args)], iters)
    what = "greedy" if greedy else (f"top-k{top_k}/top-p0.9" if top_k > 0 else f"T{temp}/top-p0.9")
    return {"case": f"sample B={B} V={V} {what}", "us": round(us, 2)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="gemm,decode,prefill,norm,rope,sample,misc")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--out", default=None)
    ap.add_argument("--gemm", default=None, help="GEMM cases M,N,K[,act[,splits]] separated by ';' (e.g. for an ncu capture)")
    ap.add_argument("--decode", default=None, help="single decode-attention case B,ctx,nq,nkv,hd")
    ap.add_argument("--prefill", default=None, help="single causal prefill attention case T,nq,nkv,hd")
    ap.add_argument("--qgemm", default=None, help="packed GGUF GEMM cases TYPE,M,N,K separated by ';' (TYPE e.g. Q4_K)")
    ap.add_argument("--qtrace", default=None, help="per-role timeline of one packed GEMM launch TYPE,M,N,K")
    a = ap.parse_args()
    hbm, tflops, src = peaks()
    only = set(a.only.split(","))
    rows = []
    if a.qtrace:
        from ..loaders.dequant import TYPE_BY_NAME
        f = a.qtrace.split(",")
        print("\n".join(trace_qgemm(TYPE_BY_NAME[f[0]], int(f[1]), int(f[2]), int(f[3]))))
        return
    if a.qgemm:
        from ..loaders.dequant import TYPE_BY_NAME
        for case in a.qgemm.split(";"):
            f = case.split(",")
            rows.append(bench_qgemm(TYPE_BY_NAME[f[0]], int(f[1]), int(f[2]), int(f[3]), a.iters))
        only = set()
    if a.prefill:
        v = [int(x) for x in a.prefill.split(",")]
        rows.append(bench_prefill(v[0], v[1], v[2], v[3], a.iters))
        only = set()
    if a.gemm or a.decode:
        only = set()
        if a.gemm:
            for case in a.gemm.split(";"):
                v = [int(x) for x in case.split(",")]
                rows.append(bench_gemm(v[0], v[1], v[2], a.iters, v[3] if len(v) > 3 else 0, v[4] if len(v) > 4 else 0))
        if a.decode:
            v = [int(x) for x in a.decode.split(",")]
            rows.append(bench_decode(v[0], v[1], v[2], v[3], v[4], a.iters))
    if "gemm" in only or "gemmd" in only:
        # Qwen3-8B decode (M = batch) and prefill (M = chunk) shapes
        for M in (1, 32, 128, 256):
            for N, K, act in ((6144, 4096, 0), (4096, 4096, 0), (24576, 4096, 1), (4096, 12288, 0)):
                rows.append(bench_gemm(M, N, K, a.iters, act))
        rows.append(bench_gemm(128, 151936, 4096, a.iters))
    if "gemm" in only:
        for M in (2048, 8192):
            for N, K, act in ((6144, 4096, 0), (24576, 4096, 1), (4096, 12288, 0)):
                rows.append(bench_gemm(M, N, K, max(5, a.iters // 5), act))
    if "decode" in only:
        for B, ctx in ((1, 4096), (32, 2048), (128, 4352), (128, 8192)):
            rows.append(bench_decode(B, ctx, 32, 8, 128, a.iters))
    if "prefill" in only:
        for T in (2048, 8192):
            rows.append(bench_prefill(T, 32, 8, 128, max(5, a.iters // 5)))
    if "norm" in only:
        rows.append(bench_norm(128, 4096, a.iters))
        rows.append(bench_norm(8192, 4096, a.iters))
    if "rope" in only:
        rows.append(bench_rope(128, 32, 8, 128, a.iters))
        rows.append(bench_rope(8192, 32, 8, 128, a.iters))
    if "misc" in only:
        rows.extend(bench_misc(a.iters))
    if "sample" in only:
        rows.append(bench_sample(128, 151936, a.iters, True))
        rows.append(bench_sample(128, 151936, a.iters, False))
        rows.append(bench_sample(64, 262144, a.iters, False, top_k=0, temp=0.7))  # Gemma3-270M serving config
    for r in rows:
        if "TBps" in r:
            r["hbm_frac_" + src] = round(r["TBps"] * 1000 / hbm, 3)
        if "TFLOPs" in r:
            r["tensor_frac_" + src] = round(r["TFLOPs"] / tflops, 3)
        print(json.dumps(r), flush=True)
    if a.out:
        with open(a.out, "w") as f:
            for r in rows:
                f.write(json.dumps(r) + "\n")


if __name__ == "__main__":
    main()
