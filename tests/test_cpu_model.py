"""End-to-end engine on the CPU oracle path: tiny random Qwen3 / Llama models (reference analogue: the
…WhenWeightsPresent generation cases of CoreUnitTest, here with random-init weights)."""
import torch

from nanovllm_b200 import ops
from nanovllm_b200.config import EngineConfig, HfConfig
from nanovllm_b200.engine.context import StepContext, set_context
from nanovllm_b200.llm import LLM
from nanovllm_b200.models.registry import init_random_weights
from nanovllm_b200.sampling_params import SamplingParams


def tiny(model_type="qwen3", **kw):
    d = dict(vocab_size=300, hidden_size=128, intermediate_size=256, num_hidden_layers=2, num_attention_heads=4,
             num_key_value_heads=2, head_dim=64, max_position_embeddings=2048, model_type=model_type,
             tie_word_embeddings=True)
    d.update(kw)
    return HfConfig(**d)


def make_llm(hf, seed=0, **cfg):
    c = dict(max_num_seqs=4, max_model_len=1024, num_kvcache_blocks=16, max_num_batched_tokens=512)
    c.update(cfg)
    return LLM((hf, init_random_weights(hf, seed)), EngineConfig(**c), device="cpu")


def full_forward_logits(llm, ids):
    """Logits of the last position computed by one dense prefill (fresh engine state)."""
    from nanovllm_b200.engine.sequence import Sequence
    s = Sequence(ids, SamplingParams(max_tokens=1), 256)
    llm.runner.model  # noqa
    bm = llm.scheduler.block_manager
    bm.allocate(s, 0)
    s.num_scheduled_tokens = len(ids)
    logits = llm.runner.forward_logits([s], True)
    bm.deallocate(s)
    return logits[0].float()


def test_greedy_generation_runs_and_is_deterministic():
    hf = tiny()
    llm = make_llm(hf)
    sp = SamplingParams(max_tokens=6, ignore_eos=True).deterministic()
    a = llm.generate_token_ids([[1, 2, 3, 4], [5, 6]], sp)
    b = llm.generate_token_ids([[1, 2, 3, 4], [5, 6]], sp)
    assert [o.token_ids for o in a] == [o.token_ids for o in b]
    assert all(len(o.token_ids) == 6 for o in a)


def test_decode_with_kv_cache_matches_full_prefill():
    """The token chosen after k decode steps equals the argmax of a dense prefill over the same prefix."""
    hf = tiny()
    llm = make_llm(hf, stop_on_degenerate=False)
    prompt = [3, 14, 15, 92, 65, 35]
    out = llm.generate_token_ids([prompt], SamplingParams(max_tokens=5, ignore_eos=True).deterministic())[0]
    seq = prompt + out.token_ids
    for k in range(1, 5):
        logits = full_forward_logits(llm, seq[:len(prompt) + k])
        assert int(torch.argmax(logits)) == seq[len(prompt) + k]


def test_chunked_prefill_matches_single_shot():
    hf = tiny()
    prompt = list(range(1, 400))
    sp = SamplingParams(max_tokens=4, ignore_eos=True).deterministic()
    a = make_llm(hf, max_num_batched_tokens=128).generate_token_ids([prompt], sp)[0].token_ids
    b = make_llm(hf, max_num_batched_tokens=1024).generate_token_ids([prompt], sp)[0].token_ids
    assert a == b


def test_prefix_cache_hit_gives_same_tokens():
    hf = tiny()
    llm = make_llm(hf)
    prompt = list(range(7, 7 + 600))
    sp = SamplingParams(max_tokens=3, ignore_eos=True).deterministic()
    a = llm.generate_token_ids([prompt], sp)[0].token_ids
    hits0 = llm.scheduler.block_manager.prefix_hit_blocks
    b = llm.generate_token_ids([prompt], sp)[0].token_ids
    assert llm.scheduler.block_manager.prefix_hit_blocks > hits0
    assert a == b


def test_seeded_sampling_reproducible_and_batch_independent():
    hf = tiny()
    llm = make_llm(hf)
    sp = SamplingParams(max_tokens=6, ignore_eos=True, temperature=0.9, top_k=40, top_p=0.9, seed=11)
    solo = llm.generate_token_ids([[1, 2, 3]], sp)[0].token_ids
    batched = llm.generate_token_ids([[9, 9], [1, 2, 3]], [sp, sp])[1].token_ids
    assert solo == batched


def test_llama_variant_and_timeout_cancel():
    import pytest
    from nanovllm_b200.exceptions import GenerationCancelledException
    hf = tiny("llama")
    llm = make_llm(hf)
    llm.cancel()  # cancel before start is cleared by generate
    llm.generate_token_ids([[1, 2]], SamplingParams(max_tokens=2).deterministic())
    calls = []

    def on_token(i, sid, tok):
        calls.append(tok)
        llm.cancel()

    with pytest.raises(GenerationCancelledException):
        llm.generate_token_ids([[1, 2]], SamplingParams(max_tokens=50, ignore_eos=True).deterministic(),
                               on_token=on_token)
    assert calls and llm.scheduler.is_finished()


def test_prompt_too_long_rejected():
    import pytest
    llm = make_llm(tiny(), max_model_len=64)
    with pytest.raises(ValueError):
        llm.generate_token_ids([list(range(64))])
