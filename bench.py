"""Headline benchmark: decode tokens/s (max over ranks) on the Qwen3-8B-shaped model, bf16, TP = N GPUs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference|baseline]
                    [--weights bf16|nvfp4|q4_k|q8_0|mxfp4]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1: tensor parallel over NCCL)

Workload (BASELINE config 5 shape): random-init Qwen3-8B architecture (36 layers, hidden 4096, 32 q / 8 kv heads,
head_dim 128, SwiGLU 12288, vocab 151936, seed 4); B concurrent requests with prompt lengths uniform in
[512, 8192] (random ids) are prefilled through the engine (their TTFT is recorded), then W warm-up and K timed
decode steps run through ``LLM.step()``.

* ``value``: decode tokens / device time.  Device time is measured with CUDA events recorded inside the model
  runner around each decode step's GPU work (H2D of the step metadata, CUDA-graph replay of the forward + LM
  head, sampler) and summed over the K steps; max over ranks.
* ``e2e``: the same tokens / wall-clock of the K ``LLM.step()`` calls (host scheduling, pinned H2D of each step's
  inputs, D2H read of the sampled tokens included); max over ranks.
* ``p50_ttft_ms``: after the timed region, ``--ttft-probe`` new requests join the running batch one at a time;
  TTFT is add_request -> first sampled token (the prefill-first scheduler runs the newcomer's prefill next).
* ``--impl baseline``: the same engine with every projection as a cuBLAS GEMM (activation as its own kernel)
  and NCCL all-reduces -- the unfused library baseline.
The weights (16 GB) and the KV cache (tens of GB) are far larger than the 126 MB L2, so no explicit L2 flush is
needed between steps.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

BASELINE_VALUE = None  # the reference publishes no decode tok/s figure


def _clock_sampler_start(path: str):
    try:
        return subprocess.Popen(
            ["nvidia-smi", "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
             "--format=csv,noheader,nounits", "-lms", "200"],
            stdout=open(path, "w"), stderr=subprocess.DEVNULL)
    except Exception:
        return None


def _clock_summary(path: str, gpu_index: int):
    sms, maxs, reasons = [], [], set()
    try:
        for line in open(path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) != gpu_index:
                continue
            sm, mx = float(parts[1]), float(parts[2])
            sms.append(sm)
            maxs.append(mx)
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for n, v in zip(names, parts[5:9]):
                if v.lower() in ("active", "1", "yes"):
                    reasons.add(n)
    except Exception:
        pass
    if not sms:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
    return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxs), "reasons": sorted(reasons)}


def qwen3_8b_config():
    from nanovllm_b200.config import HfConfig
    return HfConfig(vocab_size=151936, hidden_size=4096, intermediate_size=12288, num_hidden_layers=36,
                    num_attention_heads=32, num_key_value_heads=8, head_dim=128, max_position_embeddings=40960,
                    rms_norm_eps=1e-6, rope_theta=1_000_000.0, tie_word_embeddings=False, model_type="qwen3",
                    architectures=["Qwen3ForCausalLM"], torch_dtype="bfloat16")


def gemma3_270m_config():
    """Gemma3-270M architecture (5:1 sliding(512) / global interleave, head_dim 256)."""
    from nanovllm_b200.config import HfConfig
    return HfConfig(vocab_size=262144, hidden_size=640, intermediate_size=2048, num_hidden_layers=18,
                    num_attention_heads=4, num_key_value_heads=1, head_dim=256, max_position_embeddings=32768,
                    rms_norm_eps=1e-6, rope_theta=1_000_000.0, rope_local_base_freq=10000.0, sliding_window=512,
                    query_pre_attn_scalar=256, tie_word_embeddings=True, model_type="gemma3_text",
                    architectures=["Gemma3ForCausalLM"], torch_dtype="bfloat16",
                    layer_types=(["sliding_attention"] * 5 + ["full_attention"]) * 3)


LFM2_ATTENTION_LAYERS = (2, 5, 8, 10, 12, 14, 16, 18)  # 8 GQA layers among 30; the other 22 are short-conv


def lfm2_2_6b_config():
    """LFM2-2.6B-shaped hybrid (22 short-conv + 8 GQA layers, hidden 2048, FFN 10752)."""
    from nanovllm_b200.config import HfConfig
    kv = [8 if i in LFM2_ATTENTION_LAYERS else 0 for i in range(30)]
    return HfConfig(vocab_size=65536, hidden_size=2048, intermediate_size=10752, num_hidden_layers=30,
                    num_attention_heads=32, num_key_value_heads=8, head_dim=64, max_position_embeddings=128000,
                    rms_norm_eps=1e-5, rope_theta=1_000_000.0, model_type="lfm2", architectures=["Lfm2ForCausalLM"],
                    layer_types=["full_attention" if k else "conv" for k in kv], layer_kv_heads=kv, conv_l_cache=3,
                    tie_word_embeddings=True, torch_dtype="bfloat16")


# model -> (config builder, init seed, default batch, default prompt range, sampling, label)
MODELS = {
    "qwen3-8b": (qwen3_8b_config, 4, 128, (512, 8192), "greedy",
                 "Qwen3-8B-shape (36L, H4096, 32/8 heads, hd128, I12288, V151936)"),
    "gemma3-270m": (gemma3_270m_config, 2, 64, (128, 2048), "t0.7-p0.9",
                    "Gemma3-270M-shape (18L, H640, 4/1 heads, hd256, GeGLU 2048, V262144, 5:1 sliding 512/global)"),
    "lfm2-2.6b": (lfm2_2_6b_config, 3, 128, (256, 4096), "greedy",
                  "LFM2-2.6B-shape (30L: 22 short-conv + 8 GQA 32/8 hd64, H2048, I10752, V65536)"),
}


def _pack_lfm2_q4_k_m(weights, dev):
    """The Q4_K_M copy of config 4: projections as random Q4_K blocks, ffn_down as Q6_K (embeddings bf16)."""
    import re
    from nanovllm_b200.loaders.dequant import TYPE_BY_NAME
    from nanovllm_b200.ops.quant import random_packed
    proj = re.compile(r"(attn_q|attn_k|attn_v|attn_output|ffn_gate|ffn_up|ffn_down|in_proj|out_proj)\.weight$")
    for i, name in enumerate(sorted(weights)):
        if proj.search(name):
            N, K = weights[name].shape
            t = "Q6_K" if "ffn_down" in name else "Q4_K"
            weights[name] = random_packed(TYPE_BY_NAME[t], N, K, 6000 + i, dev)


def run_reference(args):
    line = {"impl": "reference",
            "unavailable": "the reference is a Java 21 / Maven CPU library: pip cannot install it (no setup.py or "
                           "pyproject.toml) and this image has no JDK or Maven to build or run it"}
    print(json.dumps(line))


def run_ours(args):
    from nanovllm_b200 import ops
    from nanovllm_b200.config import EngineConfig
    from nanovllm_b200.llm import LLM
    from nanovllm_b200.models.registry import init_random_weights
    from nanovllm_b200.parallel import state as ps
    from nanovllm_b200.sampling_params import SamplingParams

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        ps.init_tp("nccl", timeout_s=300)
    rank = ps.tp_rank()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg_fn, seed, _, _, sampling_kind, label = MODELS[args.model]
    hf = cfg_fn()
    weights = init_random_weights(hf, seed=seed, device=dev)
    if args.weights == "q4_k_m":
        _pack_lfm2_q4_k_m(weights, dev)
        torch.cuda.empty_cache()
    elif args.weights != "bf16":
        # the GGUF copy of config 5: every projection as random packed blocks, multiplied packed
        import re
        from nanovllm_b200.loaders.dequant import TYPE_BY_NAME
        from nanovllm_b200.ops.quant import random_packed
        proj = re.compile(r"(q_proj|k_proj|v_proj|o_proj|gate_proj|up_proj|down_proj)\.weight$")
        for i, name in enumerate(sorted(weights)):
            if proj.search(name):
                N, K = weights[name].shape
                weights[name] = random_packed(TYPE_BY_NAME[args.weights.upper()], N, K, 4000 + i, dev)
        torch.cuda.empty_cache()
    B = args.batch
    gen = torch.Generator().manual_seed(1234)
    lens = torch.randint(args.min_prompt, args.max_prompt + 1, (B,), generator=gen).tolist()
    prompts = [torch.randint(1, hf.vocab_size - 1, (n,), generator=gen).tolist() for n in lens]
    extra = 4 * args.ttft_probe + args.profile_steps + 4
    max_len = args.max_prompt + args.warmup + args.steps + extra + 64
    cfg = EngineConfig(max_num_seqs=B, max_model_len=max_len, max_num_batched_tokens=args.prefill_chunk,
                       gpu_memory_utilization=0.92, stop_on_degenerate=False, cuda_graph_max_bs=B)
    llm = LLM((hf, weights), cfg, device=dev)
    del weights
    n_new = args.warmup + args.steps + extra + 8
    if sampling_kind == "greedy":
        sps = [SamplingParams(max_tokens=n_new, ignore_eos=True).deterministic()] * B
    else:  # config 3: temperature 0.7 / top-p 0.9, a fixed seed per request
        sps = [SamplingParams(max_tokens=n_new, ignore_eos=True, temperature=0.7, top_p=0.9, seed=1000 + i)
               for i in range(B)]
    seqs = [llm.add_request(p, sp) for p, sp in zip(prompts, sps)]
    torch.cuda.synchronize()
    t_pf = time.perf_counter()
    while any(s.num_completion_tokens == 0 for s in seqs):
        llm.step()
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t_pf
    ttfts = sorted(s.t_first_token - s.t_arrival for s in seqs)
    p50_ttft_burst = ttfts[len(ttfts) // 2]
    prefill_tokens = sum(lens)
    running = len(llm.scheduler.running)

    runner = llm.runner
    step_ms = []

    def timed_step():
        runner.step_events = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        seqs_, is_prefill, _ = llm.step()
        assert not is_prefill
        step_ms.append(runner.step_events[0].elapsed_time(runner.step_events[1]))
        return len(seqs_)

    for _ in range(args.warmup):
        timed_step()
    step_ms.clear()
    if args.profile_steps > 0:
        # a capture window for `ncu --profile-from-start off`: only these decode steps are profiled
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStart()
        for _ in range(args.profile_steps):
            timed_step()
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        step_ms.clear()
    ops.reset_launch_count()
    clock_path = args.clock_log or os.path.join(tempfile.gettempdir(), f"nvb_bench_clocks_{os.getpid()}_r{rank}.csv")
    sampler = _clock_sampler_start(clock_path) if rank == 0 else None
    ps.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    tokens = 0
    for _ in range(args.steps):
        tokens += timed_step()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    ps.barrier()
    if sampler is not None:
        time.sleep(0.3)
        sampler.terminate()
        sampler.wait()
    launches = ops.launch_count()
    dev_ms = sum(step_ms)
    h2d = runner.last_h2d_bytes
    runner.step_events = None
    if args.breakdown:
        # per-kernel device time of a few more decode steps, traced per rank (attribution only, not the value)
        from nanovllm_b200.utils.breakdown import format_breakdown, kernel_breakdown
        bd = kernel_breakdown(lambda: llm.step(), 3)
        with open(f"{args.breakdown}.r{rank}.txt", "w") as f:
            f.write(f"tp{world} rank {rank}, batch {running}, impl {args.impl}, weights {args.weights}\n")
            f.write(format_breakdown(bd, top=40) + "\n")
        with open(f"{args.breakdown}.r{rank}.json", "w") as f:
            json.dump(bd, f)
    # TTFT under load: new requests (prompt lengths from the same distribution) join the running batch one at a
    # time, two decode steps apart; TTFT = add_request -> first sampled token on the host
    probe = []
    for _ in range(args.ttft_probe):
        n = int(torch.randint(args.min_prompt, args.max_prompt + 1, (1,), generator=gen))
        req = llm.add_request(torch.randint(1, hf.vocab_size - 1, (n,), generator=gen).tolist(),
                              SamplingParams(max_tokens=2, ignore_eos=True).deterministic())
        while req.num_completion_tokens == 0:
            llm.step()
        probe.append(req.t_first_token - req.t_arrival)
        for _ in range(2):
            llm.step()
    probe.sort()
    p50_ttft = probe[len(probe) // 2] if probe else p50_ttft_burst
    t = torch.tensor([dev_ms, wall * 1000.0], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    dev_ms, wall_ms = float(t[0]), float(t[1])
    llm.close()
    if rank == 0:
        value = tokens / (dev_ms / 1000.0)
        e2e = tokens / (wall_ms / 1000.0)
        line = {
            "impl": args.impl,
            "metric": ("decode tok/s (box, max over ranks) Qwen3-8B-shape TP1/2/4/8; p50 TTFT"
                       if args.model == "qwen3-8b" else f"decode tok/s (box, max over ranks) {args.model}"),
            "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None if BASELINE_VALUE is None else value / BASELINE_VALUE,
            "dtype": "bf16", "data": "synthetic: random-init weights (seed 4), random prompt ids",
            "config": {"model": label, "sampling": sampling_kind,
                       "weights": "bf16" if args.weights == "bf16" else
                                  "GGUF Q4_K_M: projections Q4_K, ffn_down Q6_K, packed (dequant-fused GEMM); "
                                  "embeddings / LM head bf16" if args.weights == "q4_k_m" else
                                  f"projections GGUF {args.weights.upper()} packed ("
                                  + ("dequantized per multiply, then cuBLAS" if args.impl == "baseline"
                                     else "dequant-fused GEMM") + "); embeddings / LM head bf16",
                       "global_batch": running, "seq_len": f"prompts U[{args.min_prompt},{args.max_prompt}]",
                       "parallelism": f"tp{world}", "l2": "inputs larger than L2 (weights of several GB + KV cache)",
                       "prefill_tokens": prefill_tokens, "prefill_s": round(prefill_s, 3),
                       "p50_ttft_ms": round(p50_ttft * 1000, 1),
                       "ttft_note": f"p50 over {len(probe)} requests joining a running batch of {running}; "
                                    f"the initial burst of {B} prompts had p50 {round(p50_ttft_burst * 1000, 1)} ms"},
            "e2e": {"value": round(e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": 8 * running + 4},  # sampled ids + device error word
            "gpu_launches": launches,
            "clocks": _clock_summary(clock_path, local),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        ps.destroy()


def gte_small_config():
    """gte-small-shaped BERT encoder (12 layers, hidden 384, 12 heads, GELU FFN 1536)."""
    from nanovllm_b200.config import HfConfig
    return HfConfig(vocab_size=30522, hidden_size=384, intermediate_size=1536, num_hidden_layers=12,
                    num_attention_heads=12, num_key_value_heads=12, head_dim=32, max_position_embeddings=512,
                    layer_norm_eps=1e-12, model_type="bert", architectures=["BertModel"], torch_dtype="float16")


def run_embed(args):
    """sentence embeddings, data-parallel over N GPUs (one replica per rank).

    Every step embeds a global batch of ``--batch`` (default 256) sequences of random ids with lengths U[16, 512]:
    the sequences are dealt to the ranks by token count (``parallel/dp.py``), each rank encodes its share as
    packed varlen batches (tcgen05 GEMMs, varlen bidirectional attention, fused LayerNorm / GELU epilogues,
    mean-pool + L2) and one all-gather returns all [batch, 384] embeddings to every rank.  ``value``: sequences
    per second of device time (CUDA events around the step, max over ranks); ``e2e``: the same over host wall
    time including the host->device copies of each step's ids and the device->host read of its embeddings."""
    from nanovllm_b200.models.bert import BertEncoder
    from nanovllm_b200.models.registry import init_random_weights
    from nanovllm_b200.parallel import state as ps
    from nanovllm_b200.parallel.dp import DataParallelEmbedder

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        ps.init_tp("nccl", timeout_s=300)
    rank = ps.tp_rank()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    hf = gte_small_config()
    weights = init_random_weights(hf, seed=1, device=dev)
    if args.weights == "q8_0":  # the GGUF Q8_0 copy: packed blocks, expanded once at load for the encoder GEMMs
        from nanovllm_b200.loaders.dequant import TYPE_BY_NAME
        from nanovllm_b200.ops.quant import random_packed
        for i, name in enumerate(sorted(weights)):
            if name.startswith("blk.") and name.endswith(".weight") and weights[name].dim() == 2:
                N, K = weights[name].shape
                weights[name] = random_packed(TYPE_BY_NAME["Q8_0"], N, K, 7000 + i, dev)
    enc = BertEncoder(hf, weights, dev)
    del weights
    dp = DataParallelEmbedder(enc)
    B = args.batch or 256
    gen = torch.Generator().manual_seed(99)
    batches = []
    for _ in range(args.warmup + args.steps):
        lens = torch.randint(16, 513, (B,), generator=gen)
        batches.append([[101] + torch.randint(1000, hf.vocab_size, (int(n) - 2,), generator=gen).tolist() + [102]
                        for n in lens])
    for b in batches[:args.warmup]:
        dp.embed_ids(b)
    torch.cuda.synchronize()
    ps.barrier()
    dev_ms, tokens = 0.0, 0
    t0 = time.perf_counter()
    for b in batches[args.warmup:]:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        out = dp.embed_ids(b)
        e1.record()
        host = out.cpu()  # the step's result read back (D2H)
        dev_ms += e0.elapsed_time(e1)
        tokens += sum(len(x) for x in b)
    torch.cuda.synchronize()
    wall_ms = (time.perf_counter() - t0) * 1000.0
    ps.barrier()
    t = torch.tensor([dev_ms, wall_ms], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    dev_ms, wall_ms = float(t[0]), float(t[1])
    ok = bool(torch.allclose(host.norm(dim=1), torch.ones(B), atol=1e-2))
    if rank == 0:
        seqs = B * args.steps
        print(json.dumps({
            "impl": args.impl, "metric": "embeddings/s (sequences, max over ranks) gte-small-shape DP1/2/4/8",
            "value": round(seqs / (dev_ms / 1000.0), 1), "unit": "sequences/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: random-init weights (seed 1), random ids, lengths U[16,512]",
            "config": {"model": "gte-small-shape BERT (12L, H384, 12 heads, FFN 1536, V30522, pos 512)",
                       "weights": "GGUF Q8_0 blocks expanded at load" if args.weights == "q8_0" else "bf16",
                       "global_batch": B, "seq_len": "U[16,512]", "parallelism": f"dp{world}",
                       "tokens_per_s": round(tokens / (dev_ms / 1000.0), 1), "unit_norm_ok": ok},
            "e2e": {"value": round(seqs / (wall_ms / 1000.0), 1), "unit": "sequences/s",
                    "h2d_bytes_per_step": 16 * tokens // args.steps, "d2h_bytes_per_step": 4 * B * hf.hidden_size},
        }), flush=True)
    if world > 1:
        ps.destroy()


def run_serve(args):
    """BASELINE config 5 as a serving run: ``--serve-requests`` requests arrive as a Poisson process of rate
    ``--serve-rate`` req/s (exponential gaps, fixed seed), prompts U[min_prompt, max_prompt] random ids, outputs
    U[128, 1024] tokens (ignore_eos); continuous batching through ``LLM.add_request`` / ``LLM.step``.

    Rank 0's host clock decides which requests have arrived before each step and broadcasts the count, so every
    TP rank admits the same requests at the same step.  Reported: output tokens / wall time of the whole run
    (max over ranks), p50 / p99 TTFT over all requests (scheduled arrival -> first sampled token on the host),
    p50 TPOT.  A throw-away batch warms the engine up before the first arrival."""
    import random
    from nanovllm_b200.config import EngineConfig
    from nanovllm_b200.llm import LLM
    from nanovllm_b200.models.registry import init_random_weights
    from nanovllm_b200.parallel import state as ps
    from nanovllm_b200.sampling_params import SamplingParams

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        ps.init_tp("nccl", timeout_s=600)
    rank = ps.tp_rank()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    hf = qwen3_8b_config()
    weights = init_random_weights(hf, seed=4, device=dev)
    rnd = random.Random(2024)
    N = args.serve_requests
    arrivals, t = [], 0.0
    for _ in range(N):
        t += rnd.expovariate(args.serve_rate)
        arrivals.append(t)
    plens = [rnd.randint(args.min_prompt, args.max_prompt) for _ in range(N)]
    olens = [rnd.randint(128, 1024) for _ in range(N)]
    cfg = EngineConfig(max_num_seqs=args.batch, max_model_len=args.max_prompt + 1024 + 64,
                       max_num_batched_tokens=args.prefill_chunk, gpu_memory_utilization=0.92,
                       stop_on_degenerate=False, cuda_graph_max_bs=args.batch)
    llm = LLM((hf, weights), cfg, device=dev)
    del weights
    gen = torch.Generator().manual_seed(77)
    for _ in range(4):
        llm.add_request(torch.randint(1, hf.vocab_size - 1, (600,), generator=gen).tolist(),
                        SamplingParams(max_tokens=args.warmup + 2, ignore_eos=True).deterministic())
    while llm.has_unfinished():
        llm.step()
    prompts = [torch.randint(1, hf.vocab_size - 1, (n,), generator=gen).tolist() for n in plens]
    flag = torch.zeros(1, dtype=torch.int64, device=dev)
    seqs = []
    admitted = steps = 0
    ps.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    while admitted < N or llm.has_unfinished():
        due = admitted
        if rank == 0:  # only rank 0's clock decides: the others follow the broadcast count
            now = time.perf_counter() - t0
            if not llm.has_unfinished() and admitted < N and arrivals[admitted] > now:
                time.sleep(arrivals[admitted] - now)  # idle until the next arrival
                now = time.perf_counter() - t0
            while due < N and arrivals[due] <= now:
                due += 1
        if world > 1:
            flag.fill_(due)
            torch.distributed.broadcast(flag, 0)
            due = int(flag.item())
        for i in range(admitted, due):
            s = llm.add_request(prompts[i], SamplingParams(max_tokens=olens[i], ignore_eos=True).deterministic())
            s.t_arrival = t0 + arrivals[i]  # the scheduled arrival, not the moment the loop noticed it
            seqs.append(s)
        admitted = due
        if llm.has_unfinished():
            llm.step()
            steps += 1
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    ttft = sorted(s.t_first_token - s.t_arrival for s in seqs)
    tpot = sorted((s.t_finish - s.t_first_token) / max(1, s.num_completion_tokens - 1) for s in seqs)
    out_tokens = sum(s.num_completion_tokens for s in seqs)
    tt = torch.tensor([wall, ttft[len(ttft) // 2], ttft[min(len(ttft) - 1, int(len(ttft) * 0.99))],
                       tpot[len(tpot) // 2]], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
    wall, p50, p99, tpot50 = (float(x) for x in tt.tolist())
    llm.close()
    if rank == 0:
        print(json.dumps({
            "impl": args.impl, "metric": "serving: output tok/s and p50 TTFT (Poisson arrivals) Qwen3-8B-shape",
            "value": round(out_tokens / wall, 1), "unit": "output tokens/s", "n_gpus": world,
            "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic: random-init weights (seed 4), random prompt ids",
            "config": {"model": "Qwen3-8B-shape", "requests": N, "rate_per_s": args.serve_rate,
                       "prompt_len": f"U[{args.min_prompt},{args.max_prompt}]", "output_len": "U[128,1024]",
                       "max_num_seqs": args.batch, "parallelism": f"tp{world}"},
            "p50_ttft_ms": round(p50 * 1000, 1), "p99_ttft_ms": round(p99 * 1000, 1),
            "p50_tpot_ms": round(tpot50 * 1000, 2), "wall_s": round(wall, 2), "engine_steps": steps,
            "output_tokens": out_tokens, "prompt_tokens": sum(plens)}), flush=True)
    if world > 1:
        ps.destroy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--model", choices=sorted(MODELS) + ["gte-small"], default="qwen3-8b",
                    help="BASELINE config: qwen3-8b (5, the headline), gemma3-270m (3), lfm2-2.6b (4), gte-small (2)")
    ap.add_argument("--batch", type=int, default=None, help="concurrent requests (default per model)")
    ap.add_argument("--min-prompt", type=int, default=None)
    ap.add_argument("--max-prompt", type=int, default=None)
    ap.add_argument("--prefill-chunk", type=int, default=16384)
    ap.add_argument("--profile-steps", type=int, default=0,
                    help="decode steps run between cudaProfilerStart/Stop before the timed region")
    ap.add_argument("--impl", choices=["ours", "reference", "baseline"], default="ours",
                    help="baseline: this engine with cuBLAS GEMMs (separate activation kernel) and NCCL all-reduce")
    ap.add_argument("--weights", choices=["bf16", "nvfp4", "q4_k", "q8_0", "mxfp4", "q4_k_m"], default=None,
                    help="projection weights: bf16, or random GGUF blocks kept packed (the NVFP4 copy of config 5)")
    ap.add_argument("--breakdown", default="",
                    help="path prefix: write a per-kernel device-time breakdown of 3 traced decode steps per rank")
    ap.add_argument("--clock-log", default="",
                    help="CSV file for the nvidia-smi clock samples taken during the timed region (default: a temp file)")
    ap.add_argument("--serve", action="store_true",
                    help="serving run (BASELINE config 5): Poisson arrivals, output lengths U[128,1024], p50 TTFT")
    ap.add_argument("--serve-requests", type=int, default=512)
    ap.add_argument("--serve-rate", type=float, default=4.0, help="Poisson arrival rate (requests / s)")
    ap.add_argument("--ttft-probe", type=int, default=8,
                    help="requests that join the running batch one at a time after the timed region (p50 TTFT)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.model in MODELS:
        _, _, batch, (lo, hi), _, _ = MODELS[args.model]
        args.batch = args.batch or batch
        args.min_prompt = args.min_prompt or lo
        args.max_prompt = args.max_prompt or hi
    if args.weights is None:
        args.weights = "q4_k_m" if args.model == "lfm2-2.6b" else "bf16"
    if args.impl == "reference":
        run_reference(args)
        return
    if args.impl == "baseline":
        os.environ["NVB_BASELINE"] = "1"  # cuBLAS GEMMs + separate activation + NCCL all-reduce
    if args.serve:
        run_serve(args)
        return
    if args.model == "gte-small":
        run_embed(args)
        return
    run_ours(args)


if __name__ == "__main__":
    main()
