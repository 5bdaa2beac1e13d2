"""Tensor parallel on 2 and 4 GPUs over NCCL: TP greedy decode (CUDA graphs with the collectives captured) matches
the TP=1 engine's logits and the ranks agree.  Children run with a short process-group timeout."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _collect(q, procs, timeout=300):
    """One result per child; fails at once (instead of after ``timeout``) when a child exits without one."""
    import queue as _queue
    import time as _time
    out, deadline = [], _time.monotonic() + timeout
    while len(out) < len(procs):
        try:
            out.append(q.get(timeout=2))
        except _queue.Empty:
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            if dead:
                raise AssertionError(f"a rank exited with {dead} before reporting")
            if _time.monotonic() > deadline:
                raise AssertionError("ranks did not report in time")
    return out


def _tiny():
    from nanovllm_b200.config import HfConfig
    return HfConfig(vocab_size=2048, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                    num_attention_heads=8, num_key_value_heads=2, head_dim=128, max_position_embeddings=4096,
                    model_type="qwen3", tie_word_embeddings=False)


def _prefill_logits(llm, ids):
    from nanovllm_b200.engine.sequence import Sequence
    from nanovllm_b200.sampling_params import SamplingParams
    s = Sequence(ids, SamplingParams(max_tokens=1), 256)
    bm = llm.scheduler.block_manager
    bm.allocate(s, 0)
    s.num_scheduled_tokens = len(ids)
    logits = llm.runner.forward_logits([s], True)
    head = llm.model.lm_head
    if getattr(head, "sharded", False):  # under TP each rank's head scores its vocabulary slice
        logits = head.gather_full(logits)
    out = logits[0].float().cpu()
    bm.deallocate(s)
    return out


def _run(rank, world, port, q, eager, fused="1", spv="1"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NVB_TP_FUSED=fused, NVB_SP=spv)
    from nanovllm_b200.config import EngineConfig
    from nanovllm_b200.llm import LLM
    from nanovllm_b200.models.registry import init_random_weights
    from nanovllm_b200.parallel import state as ps
    from nanovllm_b200.sampling_params import SamplingParams
    ps.init_tp("nccl", timeout_s=60)
    dev = torch.device("cuda", rank)
    hf = _tiny()
    llm = LLM((hf, init_random_weights(hf, 0, device=dev)),
              EngineConfig(max_num_seqs=4, max_model_len=1024, num_kvcache_blocks=16, max_num_batched_tokens=512,
                           enforce_eager=eager, stop_on_degenerate=False), device=dev)
    outs = llm.generate_token_ids([list(range(3, 200)), [5, 6, 7]],
                                  SamplingParams(max_tokens=8, ignore_eos=True).deterministic())
    q.put((rank, [o.token_ids for o in outs], _prefill_logits(llm, list(range(3, 200)))))
    llm.close()
    ps.barrier()
    ps.destroy()


def _tp_matches_tp1(world, eager, fused, spv):
    from nanovllm_b200.config import EngineConfig
    from nanovllm_b200.llm import LLM
    from nanovllm_b200.models.registry import init_random_weights
    hf = _tiny()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, port, q, eager, fused, spv)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for r, toks, logits in _collect(q, procs):
        res[r] = (toks, logits)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(1, world):
        assert res[0][0] == res[r][0], "ranks diverged"
        assert torch.equal(res[0][1], res[r][1]), "ranks computed different logits"
    ref = LLM((hf, init_random_weights(hf, 0, device=torch.device("cuda", 0))),
              EngineConfig(max_num_seqs=4, max_model_len=1024, num_kvcache_blocks=16, max_num_batched_tokens=512,
                           stop_on_degenerate=False), device=torch.device("cuda", 0))
    want = _prefill_logits(ref, list(range(3, 200)))
    # bf16 reductions happen in a different order under TP: compare logits, not near-tie argmaxes
    assert torch.allclose(res[0][1], want, atol=0.06, rtol=0.05), (res[0][1] - want).abs().max()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("eager,fused,spv", [(True, "1", "1"), (False, "1", "1"), (False, "1", "0"),
                                             (False, "0", "1")])
def test_tp2_gpu_matches_tp1(eager, fused, spv):
    """fused + sp: sequence-parallel GEMM+RS / AG+norm+GEMM path for every step of <= 256 tokens; sp 0: GEMM
    then the fused all-reduce + RMSNorm kernel; fused 0: NCCL all-reduces."""
    _tp_matches_tp1(2, eager, fused, spv)


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs 4 GPUs")
@pytest.mark.parametrize("fused,spv", [("1", "0"), ("0", "0"), ("1", "1")])
def test_tp4_gpu_matches_tp1(fused, spv):
    """TP4 with 2 KV heads: each KV head is replicated on two ranks (fewer KV heads than ranks)."""
    _tp_matches_tp1(4, False, fused, spv)


def _ar_run(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NVB_TP_FUSED="1")
    from nanovllm_b200 import ops
    from nanovllm_b200.ops import reference_cpu as ref
    from nanovllm_b200.parallel import state as ps
    from nanovllm_b200.parallel import symm
    ps.init_tp("nccl", timeout_s=60)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    T, H = 203, 1024
    ws = symm.init_workspace(256, H, dev)
    parts = [torch.randn(T, H, generator=torch.Generator().manual_seed(10 + r)).bfloat16() for r in range(world)]
    res0 = torch.randn(T, H, generator=torch.Generator().manual_seed(99)).bfloat16()
    w = (1 + 0.1 * torch.randn(H, generator=torch.Generator().manual_seed(7))).bfloat16()
    total = torch.zeros(T, H)
    for p in parts:
        total += p.float()
    want_res = (total + res0.float()).bfloat16()
    want_out, _ = ref.rms_norm(want_res, w, 1e-6, 0)
    errs = []
    for it in range(3):  # consecutive launches advance the per-block epochs
        ws.in_view(T).copy_(parts[rank].to(dev))
        out, res = ws.allreduce_norm(T, w.to(dev), 1e-6, 0, res0.to(dev))
        torch.cuda.synchronize()
        errs.append(float((res.float().cpu() - want_res.float()).abs().max()))
        errs.append(float((out.float().cpu() - want_out.float()).abs().max()))
    ws.in_view(T).copy_(parts[rank].to(dev))
    plain = ops.materialize(ops.TPPartial(ws, T)).float().cpu()
    errs.append(float((plain - total.bfloat16().float()).abs().max()))
    # captured in a CUDA graph and replayed twice
    x_in = parts[rank].to(dev)
    w_dev = w.to(dev)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            ws.in_view(T).copy_(x_in)
            gout, _ = ws.allreduce_norm(T, w_dev, 1e-6, 0, None)
    torch.cuda.current_stream().wait_stream(s)
    want_plain_norm, _ = ref.rms_norm(total.bfloat16(), w, 1e-6, 0)
    for _ in range(2):
        g.replay()
        torch.cuda.synchronize()
        errs.append(float((gout.float().cpu() - want_plain_norm.float()).abs().max()))
    ops.check_device_errors(dev)
    del g
    q.put((rank, errs))
    symm.release_workspace()
    ps.barrier()
    ps.destroy()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_allreduce_rmsnorm_over_peer_memory(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ar_run, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(_collect(q, procs))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r, errs in res.items():
        # residual: fp32 sum of bf16 partials, rounded once (exact up to one bf16 ulp); outputs bf16-rounded
        assert max(errs) < 0.07, (r, errs)


def _sp_run(rank, world, port, q):
    """Sequence-parallel fused kernels on ``world`` GPUs against an fp32 CPU restatement: embedding gather +
    reduce-scatter, row-parallel GEMM + reduce-scatter (with and without split K), all-gather + RMSNorm fused
    into the column-parallel GEMM (plain, fused SiLU*up, split-K partial output), the stand-alone all-gather,
    and graph replays that advance the epoch."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NVB_TP_FUSED="1", NVB_SP="1")
    from nanovllm_b200 import ops
    from nanovllm_b200.ops import reference_cpu as ref
    from nanovllm_b200.parallel import sp
    from nanovllm_b200.parallel import state as ps
    ps.init_tp("nccl", timeout_s=60)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    H, Kt, V = 1024, 2048, 1000
    ws = sp.init_workspace(256, H, dev)
    g = torch.Generator().manual_seed(5)
    Wrow = (torch.randn(H, Kt, generator=g) * 0.03).bfloat16()          # row-parallel: K sharded
    Wcol = (torch.randn(768, H, generator=g) * 0.03).bfloat16()          # column-parallel: N sharded
    gate = (torch.randn(512, H, generator=g) * 0.03).bfloat16()
    up = (torch.randn(512, H, generator=g) * 0.03).bfloat16()
    table = torch.randn(V, H, generator=g).bfloat16()
    nw = (1 + 0.1 * torch.randn(H, generator=g)).bfloat16()
    ks, kn = Kt // world, 768 // world
    Wrow_r = Wrow[:, rank * ks:(rank + 1) * ks].contiguous().to(dev)
    Wcol_r = Wcol[rank * kn:(rank + 1) * kn].contiguous().to(dev)
    gi = 512 // world
    gu_r = ref.interleave_gate_up(torch.cat([gate[rank * gi:(rank + 1) * gi], up[rank * gi:(rank + 1) * gi]]),
                                  128).contiguous().to(dev) if gi % 128 == 0 else None
    per_v = (V + world - 1) // world
    v0, v1 = rank * per_v, min(V, (rank + 1) * per_v)
    table_r = table[v0:v1].contiguous().to(dev)
    errs = []
    for T in (1, 5, 77, 128, 256):
        x = (torch.randn(T, Kt, generator=torch.Generator().manual_seed(T)) * 0.5).bfloat16()
        ids = torch.randint(0, V, (T,), generator=torch.Generator().manual_seed(100 + T))
        # ---- fp32 restatement: per-rank partials rounded to bf16, summed in rank order, rounded (residual)
        emb = table[ids].float()
        res0 = emb.bfloat16()
        h0, _ = ref.rms_norm(res0, nw, 1e-6, 0)
        y0 = ref.linear(h0, Wcol)
        parts = [(x[:, r * ks:(r + 1) * ks].float() @ Wrow[:, r * ks:(r + 1) * ks].float().t()).bfloat16()
                 for r in range(world)]
        tot = torch.zeros(T, H)
        for p_ in parts:
            tot += p_.float()
        res1 = (tot + res0.float()).bfloat16()
        h1, _ = ref.rms_norm(res1, nw, 1e-6, 0)
        y1 = ref.linear(h1, Wcol)
        act_ref = (ref.silu(ref.linear(h1, gate).float()) * ref.linear(h1, up).float()).bfloat16()
        # ---- device: embedding RS -> AG+norm+GEMM (no residual) ; GEMM RS -> AG+norm+GEMM (residual)
        ws.begin(T)
        from nanovllm_b200.layers.embedding import VocabParallelEmbedding  # noqa: F401 (layer path below)
        slot, plan = ws.producer_plan()
        n = ops._cuda_ext().sp_embed_rs(table_r, ids.to(dev), 1.0, v0, v1, plan)
        part = sp.SPPartial(ws, slot, int(n), T)
        out0 = ops.materialize(ops.linear_sp_consume(part, nw.to(dev), 1e-6, 0, False, Wcol_r, partial_ok=True))
        part = ops.linear_sp_produce(ws, x[:, rank * ks:(rank + 1) * ks].contiguous().to(dev), Wrow_r)
        if gu_r is not None:
            out1 = ops.linear_sp_consume(part, nw.to(dev), 1e-6, 0, True, gu_r, ops.ACT_SILU_MUL)
        else:
            out1 = ops.linear_sp_consume(part, nw.to(dev), 1e-6, 0, True, Wcol_r)
        torch.cuda.synchronize()
        ops.check_device_errors(dev)
        errs.append(("y0", T, float((out0.float().cpu() - y0[:, rank * kn:(rank + 1) * kn].float()).abs().max())))
        if gu_r is not None:
            want = act_ref[:, rank * gi:(rank + 1) * gi]
        else:
            want = y1[:, rank * kn:(rank + 1) * kn]
        # relative to magnitude: SiLU*up outputs reach ~10, where one bf16 ulp is 0.0625
        errs.append(("y1", T, float(((out1.float().cpu() - want.float()).abs() / (1 + want.float().abs())).max())))
        own0, own1 = ws.owned_range()
        if own1 > own0:
            errs.append(("res", T, float((ws.residual_view().float().cpu() - res1[own0:own1].float()).abs().max())))
        gdiff = (ws.gather_view(T).float().cpu() - h1.float()).abs()
        errs.append(("gather", T, float(gdiff.max())))
        if float(gdiff.max()) > 0.06:  # where it goes wrong (rows, first columns) for the failure message
            bad_rows = (gdiff.max(dim=1).values > 0.06).nonzero().flatten().tolist()
            errs.append(("gather_bad_rows", T, float(len(bad_rows)), bad_rows[:8],
                         (gdiff[bad_rows[0]] > 0.06).nonzero().flatten().tolist()[:8]))
    # the stand-alone all-gather + norm after a stand-alone push, replayed from a CUDA graph twice
    T = 64
    xr = torch.randn(T, H, generator=torch.Generator().manual_seed(3 + rank)).bfloat16().to(dev)
    allx = [torch.randn(T, H, generator=torch.Generator().manual_seed(3 + r)).bfloat16() for r in range(world)]
    tot = torch.zeros(T, H)
    for a in allx:
        tot += a.float()
    want_g, _ = ref.rms_norm(tot.bfloat16(), nw, 1e-6, 0)
    nwd = nw.to(dev)
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph):
            ws.begin(T)
            pp = ws.rs_push(xr)
            gout = ws.ag_norm(pp, nwd, 1e-6, 0, False)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        errs.append(("graph", T, float((gout.float().cpu() - want_g.float()).abs().max())))
    ops.check_device_errors(dev)
    del graph
    # distributed greedy sampler over vocab-parallel logits: exact argmax, ties to the lowest id
    from nanovllm_b200.layers.embedding import ParallelLMHead
    V = 1001
    head = ParallelLMHead(torch.zeros(V, 8, dtype=torch.bfloat16, device=dev), V)
    full = torch.randn(200, V, generator=torch.Generator().manual_seed(9)).bfloat16()
    full[3, 5] = full[3, V - 1] = 60.0
    mine = torch.full((200, head.weight.shape[0]), 1e4).bfloat16()
    mine[:, :head.ncols] = full[:, head.vstart:head.vstart + head.ncols]
    for _ in range(2):
        toks = head.argmax(mine.to(dev), 0.0)
        torch.cuda.synchronize()
        n_bad = int((toks.cpu() != torch.argmax(full.float(), 1)).sum())
        errs.append(("argmax", 200, float(n_bad)))
    ops.check_device_errors(dev)
    q.put((rank, errs))
    sp.release_workspace()
    ps.barrier()
    ps.destroy()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sequence_parallel_fused_kernels_match_fp32(world):
    """The GEMM epilogue pushes each tile to the row owner (reduce-scatter); the owner adds the residual, norms
    and broadcasts (all-gather) into the next GEMM's operand."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sp_run, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(_collect(q, procs))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r, errs in res.items():
        bad = [e for e in errs if e[2] > 0.06 or e[0].endswith("bad_rows")]
        assert not bad, (r, bad)
