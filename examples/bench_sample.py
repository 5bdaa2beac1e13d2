"""Throughput smoke test in the shape of the reference's ``Bench`` sample: N sequences of random prompt ids
(16-128), 8-64 new tokens each, T=0.6, ignore_eos; prints tokens/s.

    python examples/bench_sample.py [--model PATH] [--seqs 8] [--seed 0]

Without ``--model`` it runs a random-init Qwen3-0.6B-shaped model (no download needed).
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))  # run from a checkout
import argparse
import random
import time

from nanovllm_b200.config import EngineConfig, HfConfig
from nanovllm_b200.llm import LLM
from nanovllm_b200.sampling_params import SamplingParams


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default=None)
    ap.add_argument("--seqs", type=int, default=8)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args()
    if a.model:
        from nanovllm_b200.api.factory import LlmModelFactory
        model = LlmModelFactory.make(a.model)
        vocab = model.hf_config.vocab_size
    else:
        from nanovllm_b200.models.registry import init_random_weights
        hf = HfConfig(vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                      num_attention_heads=16, num_key_value_heads=8, head_dim=128, max_position_embeddings=40960,
                      model_type="qwen3", tie_word_embeddings=True)
        model = (hf, init_random_weights(hf, a.seed))
        vocab = hf.vocab_size
    llm = LLM(model, EngineConfig(max_model_len=512, max_num_seqs=max(8, a.seqs)), warmup=True)
    rng = random.Random(a.seed)
    prompts = [[rng.randrange(vocab) for _ in range(rng.randint(16, 128))] for _ in range(a.seqs)]
    sps = [SamplingParams(temperature=0.6, max_tokens=rng.randint(8, 64), ignore_eos=True, seed=a.seed + i)
           for i in range(a.seqs)]
    t0 = time.perf_counter()
    outs = llm.generate_token_ids(prompts, sps)
    dt = time.perf_counter() - t0
    n = sum(len(o.token_ids) for o in outs)
    print(f"{a.seqs} seqs, {n} new tokens in {dt:.3f}s: {n / dt:.1f} tok/s "
          f"(p50 TTFT {llm.last_stats.p50_ttft() * 1e3:.1f} ms)")
    llm.close()


if __name__ == "__main__":
    main()
