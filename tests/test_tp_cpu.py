"""Tensor-parallel sharding on CPU ranks (gloo, world size 2): the sharded Qwen3 reproduces the TP=1 logits and
greedy tokens, and ranks stay in lock-step without a per-step broadcast (reference has no TP; this checks the
column / row / merged / qkv / vocab-parallel decomposition the reference only names)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tiny():
    from nanovllm_b200.config import HfConfig
    return HfConfig(vocab_size=302, hidden_size=128, intermediate_size=256, num_hidden_layers=2, num_attention_heads=4,
                    num_key_value_heads=2, head_dim=64, max_position_embeddings=1024, model_type="qwen3",
                    tie_word_embeddings=False)


def _params(mode):
    from nanovllm_b200.sampling_params import SamplingParams
    if mode == "greedy":
        return SamplingParams(max_tokens=6, ignore_eos=True).deterministic()
    if mode == "topk":  # top-k rows exchange candidates instead of the logits
        return SamplingParams(max_tokens=6, ignore_eos=True, temperature=0.8, top_k=20, top_p=0.9, seed=5)
    return SamplingParams(max_tokens=6, ignore_eos=True, temperature=0.8, seed=5)


def _run(rank, world, port, q, greedy=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from nanovllm_b200.config import EngineConfig
    from nanovllm_b200.llm import LLM
    from nanovllm_b200.models.registry import init_random_weights
    from nanovllm_b200.parallel import state as ps
    from nanovllm_b200.sampling_params import SamplingParams
    ps.init_tp("gloo")
    hf = _tiny()
    llm = LLM((hf, init_random_weights(hf, 0)), EngineConfig(max_num_seqs=4, max_model_len=512, num_kvcache_blocks=8,
                                                             max_num_batched_tokens=256), device="cpu")
    sp_ = _params(greedy)
    outs = llm.generate_token_ids([[1, 2, 3, 4, 5], list(range(20, 90))], sp_)
    q.put((rank, [o.token_ids for o in outs]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("greedy", ["sampled", "topk"])
def test_tp2_matches_tp1_on_cpu(greedy):
    """Sampled rows (no top-k) gather the full logits, top-k rows exchange candidates; both must reproduce the
    TP=1 tokens exactly (greedy rows take the distributed
    argmax, checked exactly by test_distributed_argmax_is_exact: on random-init models bf16 logits tie often
    enough that a different summation order legitimately flips a greedy token)."""
    from nanovllm_b200.config import EngineConfig
    from nanovllm_b200.llm import LLM
    from nanovllm_b200.models.registry import init_random_weights
    from nanovllm_b200.sampling_params import SamplingParams
    hf = _tiny()
    ref = LLM((hf, init_random_weights(hf, 0)), EngineConfig(max_num_seqs=4, max_model_len=512, num_kvcache_blocks=8,
                                                             max_num_batched_tokens=256), device="cpu")
    sp_ = _params(greedy)
    want = [o.token_ids for o in ref.generate_token_ids([[1, 2, 3, 4, 5], list(range(20, 90))], sp_)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, 2, port, q, greedy)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got[0] == got[1], "ranks diverged"
    # fp32 math on CPU: sharded reductions change summation order only
    assert got[0] == want


def _cand_run(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from nanovllm_b200.layers.embedding import ParallelLMHead
    from nanovllm_b200.ops import reference_cpu as ref
    from nanovllm_b200.parallel import state as ps
    ps.init_tp("gloo")
    V, T = 301, 8
    head = ParallelLMHead(torch.zeros(V, 8), V)
    g = torch.Generator().manual_seed(3)
    full = (torch.randn(T, V, generator=g) * 3).bfloat16()
    full[2, 10] = full[2, 250] = full[2, 11] = 9.0   # ties inside and across slices
    per = head.weight.shape[0]
    mine = torch.full((T, per), 1e4).bfloat16()
    mine[:, :head.ncols] = full[:, head.vstart:head.vstart + head.ncols]
    temps = torch.full((T,), 0.9)
    topk = torch.tensor([1, 2, 5, 20, 64, 7, 3, 40], dtype=torch.int32)
    topp = torch.tensor([1.0, 0.9, 0.5, 0.95, 0.8, 1.0, 0.3, 0.99])
    seeds = torch.arange(T, dtype=torch.int64) + 11
    sids = torch.arange(T, dtype=torch.int64)
    steps = torch.full((T,), 4, dtype=torch.int32)
    res = []
    for cap in (0.0, 5.0):
        got = head.sample_candidates(mine, temps, topk, topp, seeds, sids, steps, kmax=64, softcap=cap).tolist()
        want = ref.sample(full, temps, topk, topp, seeds, sids, steps, cap).tolist()
        res.append((got, want))
    q.put((rank, res))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_candidate_sampling_matches_full_vocabulary(world):
    """Top-k rows sampled from the exchanged per-rank candidates give exactly the tokens of the sampler over the
    whole vocabulary (ties, top-p cuts, soft-cap included)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cand_run, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        for cand, want in got[r]:
            assert cand == want, (r, cand, want)


def _argmax_run(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from nanovllm_b200.layers.embedding import ParallelLMHead
    from nanovllm_b200.parallel import state as ps
    ps.init_tp("gloo")
    V, H, T = 301, 8, 6
    head = ParallelLMHead(torch.zeros(V, H), V)
    g = torch.Generator().manual_seed(0)
    full = torch.randn(T, V, generator=g).bfloat16()
    full[1, 7] = full[1, 290] = 50.0           # tie across ranks: the lower id wins
    full[2, 100] = full[2, 101] = 40.0         # tie inside one slice
    full[3, :] = -5.0                          # all equal: id 0
    per = head.weight.shape[0]
    mine = torch.full((T, per), 1e4).bfloat16()  # padding columns past the vocabulary must be ignored
    mine[:, :head.ncols] = full[:, head.vstart:head.vstart + head.ncols]
    got = head.argmax(mine, 0.0).tolist()
    capped = head.argmax(mine, 3.0).tolist()     # soft-capped values tie more often; still lowest id
    q.put((rank, got, capped, torch.argmax(full.float(), 1).tolist(),
           torch.argmax(3.0 * torch.tanh(full.float() / 3.0), 1).tolist()))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_distributed_argmax_is_exact(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_argmax_run, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict((r, rest) for r, *rest in (q.get(timeout=240) for _ in procs))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r, (toks, capped, want, want_capped) in got.items():
        assert toks == want, (r, toks, want)
        assert capped == want_capped, (r, capped, want_capped)


def _lfm2_run(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from nanovllm_b200.config import EngineConfig
    from nanovllm_b200.llm import LLM
    from nanovllm_b200.models.registry import init_random_weights
    from nanovllm_b200.parallel import state as ps
    from nanovllm_b200.sampling_params import SamplingParams
    from tests.test_models_cpu import lfm2_tiny
    ps.init_tp("gloo")
    hf = lfm2_tiny()
    llm = LLM((hf, init_random_weights(hf, 3)), EngineConfig(max_num_seqs=4, max_model_len=512, num_kvcache_blocks=8,
                                                             max_num_batched_tokens=64), device="cpu")
    conv = next(L.conv for L in llm.model.layers if L.is_conv)
    outs = llm.generate_token_ids([list(range(5, 90)), [7, 8, 9]],
                                  SamplingParams(max_tokens=5, ignore_eos=True, temperature=0.8, seed=11))
    q.put((rank, [o.token_ids for o in outs], conv.H, tuple(conv.conv_w.shape)))
    dist.barrier()
    dist.destroy_process_group()


def test_lfm2_conv_layers_shard_channels_under_tp2():
    """LFM2's short-conv layers are channel-parallel under TP (in_proj thirds column-sharded, conv weight and
    recurrent state per channel slice, out_proj row-parallel): TP=2 reproduces the TP=1 tokens through chunked
    prefill (64-token budget) and decode."""
    from nanovllm_b200.config import EngineConfig
    from nanovllm_b200.llm import LLM
    from nanovllm_b200.models.registry import init_random_weights
    from nanovllm_b200.sampling_params import SamplingParams
    from tests.test_models_cpu import lfm2_tiny
    hf = lfm2_tiny()
    ref = LLM((hf, init_random_weights(hf, 3)), EngineConfig(max_num_seqs=4, max_model_len=512, num_kvcache_blocks=8,
                                                             max_num_batched_tokens=64), device="cpu")
    want = [o.token_ids for o in ref.generate_token_ids(
        [list(range(5, 90)), [7, 8, 9]], SamplingParams(max_tokens=5, ignore_eos=True, temperature=0.8, seed=11))]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_lfm2_run, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {r: rest for r, *rest in (q.get(timeout=240) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got[0][0] == got[1][0] == want
    assert got[0][1] == hf.hidden_size // 2 and got[0][2][0] == hf.hidden_size // 2


def _dp_run(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from nanovllm_b200.models.bert import BertEncoder
    from nanovllm_b200.models.registry import init_random_weights
    from nanovllm_b200.parallel import state as ps
    from nanovllm_b200.parallel.dp import DataParallelEmbedder
    from tests.test_models_cpu import bert_tiny
    ps.init_tp("gloo")
    hf = bert_tiny()
    enc = BertEncoder(hf, init_random_weights(hf, 1), "cpu", torch.float32)
    g = torch.Generator().manual_seed(4)
    batch = [torch.randint(0, hf.vocab_size, (int(n),), generator=g).tolist()
             for n in torch.randint(2, 100, (13,), generator=g)]
    dp = DataParallelEmbedder(enc)
    mine, _ = dp.shard(batch)
    q.put((rank, dp.embed_ids(batch).numpy(), sum(len(batch[i]) for i in mine)))
    dist.barrier()
    dist.destroy_process_group()


def test_bert_data_parallel_embeddings_match_single_process():
    """BERT DP across 3 gloo ranks: token-balanced deal, replicas encode their share, one all-gather restores the
    input order -- every rank returns the single-process embeddings."""
    from nanovllm_b200.models.bert import BertEncoder
    from nanovllm_b200.models.registry import init_random_weights
    from nanovllm_b200.parallel.dp import deal_by_tokens
    from tests.test_models_cpu import bert_tiny
    hf = bert_tiny()
    g = torch.Generator().manual_seed(4)
    batch = [torch.randint(0, hf.vocab_size, (int(n),), generator=g).tolist()
             for n in torch.randint(2, 100, (13,), generator=g)]
    want = BertEncoder(hf, init_random_weights(hf, 1), "cpu", torch.float32).embed_ids(batch)
    plan = deal_by_tokens([len(s) for s in batch], 3)
    assert sorted(i for p in plan for i in p) == list(range(len(batch)))
    loads = [sum(len(batch[i]) for i in p) for p in plan]
    assert max(loads) - min(loads) <= max(len(s) for s in batch)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dp_run, args=(r, 3, port, q)) for r in range(3)]
    for p in procs:
        p.start()
    got = {r: (torch.from_numpy(e), n) for r, e, n in (q.get(timeout=240) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r, (emb, _) in got.items():
        assert torch.allclose(emb, want, atol=1e-5), (r, (emb - want).abs().max())
