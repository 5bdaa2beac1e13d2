"""Engine on the GPU: CUDA path vs the CPU oracle, CUDA-graph decode vs eager decode, seeded determinism."""
import pytest
import torch

from nanovllm_b200 import ops
from nanovllm_b200.config import EngineConfig, HfConfig
from nanovllm_b200.engine.sequence import Sequence
from nanovllm_b200.llm import LLM
from nanovllm_b200.models.registry import init_random_weights
from nanovllm_b200.sampling_params import SamplingParams

pytestmark = pytest.mark.gpu


def tiny(**kw):
    d = dict(vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=8,
             num_key_value_heads=2, head_dim=128, max_position_embeddings=4096, model_type="qwen3",
             tie_word_embeddings=False)
    d.update(kw)
    return HfConfig(**d)


def build(hf, device, eager=False, seed=0):
    w = init_random_weights(hf, seed)
    cfg = EngineConfig(max_num_seqs=8, max_model_len=2048, num_kvcache_blocks=24, max_num_batched_tokens=1024,
                       enforce_eager=eager, stop_on_degenerate=False)
    return LLM((hf, w), cfg, device=device)


def prefill_logits(llm, ids):
    s = Sequence(ids, SamplingParams(max_tokens=1), 256)
    bm = llm.scheduler.block_manager
    bm.allocate(s, 0)
    s.num_scheduled_tokens = len(ids)
    out = llm.runner.forward_logits([s], True)[0].float().cpu()
    bm.deallocate(s)
    return out


def test_gpu_prefill_logits_match_cpu_oracle():
    hf = tiny()
    ids = list(range(3, 300))
    a = prefill_logits(build(hf, "cpu"), ids)
    b = prefill_logits(build(hf, "cuda", eager=True), ids)
    assert torch.allclose(a, b, atol=0.05, rtol=0.05), (a - b).abs().max()


def test_graph_decode_matches_eager_decode():
    hf = tiny()
    sp = SamplingParams(max_tokens=12, ignore_eos=True).deterministic()
    prompts = [list(range(5, 60)), list(range(100, 400)), [7]]
    a = build(hf, "cuda", eager=True).generate_token_ids(prompts, sp)
    b = build(hf, "cuda", eager=False).generate_token_ids(prompts, sp)
    assert [o.token_ids for o in a] == [o.token_ids for o in b]
    ops.check_device_errors()


def test_gpu_seeded_sampling_reproducible():
    hf = tiny()
    llm = build(hf, "cuda")
    sp = SamplingParams(max_tokens=10, ignore_eos=True, temperature=0.8, top_p=0.9, top_k=50, seed=123)
    x = llm.generate_token_ids([[1, 2, 3, 4]], sp)[0].token_ids
    y = llm.generate_token_ids([[9, 9, 9], [1, 2, 3, 4]], [sp, sp])[1].token_ids
    assert x == y


def test_gpu_greedy_matches_cpu_first_tokens():
    hf = tiny()
    sp = SamplingParams(max_tokens=3, ignore_eos=True).deterministic()
    p = [list(range(11, 140))]
    a = build(hf, "cpu").generate_token_ids(p, sp)[0].token_ids
    b = build(hf, "cuda").generate_token_ids(p, sp)[0].token_ids
    assert a[0] == b[0]
