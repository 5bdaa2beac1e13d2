"""Smallest end-to-end uses: generate text from a chat model and embed sentences with an encoder.

    python examples/hello.py --model /path/to/Qwen3-0.6B [--embed /path/to/bge-small.gguf]
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))  # run from a checkout
import argparse

from nanovllm_b200.api.factory import LlmModelFactory
from nanovllm_b200.llm import LLM
from nanovllm_b200.sampling_params import SamplingParams

ap = argparse.ArgumentParser()
ap.add_argument("--model", required=True)
ap.add_argument("--embed", default=None)
a = ap.parse_args()

llm = LLM(LlmModelFactory.make(a.model))
print(llm.chat_once("Name three primary colours.", sampling=SamplingParams(max_tokens=64).deterministic()))
for out in llm.generate(["The capital of France is", "1, 2, 3,"], SamplingParams(max_tokens=16)):
    print(repr(out.text))
llm.close()

if a.embed:
    enc = LlmModelFactory.make(a.embed)
    v = enc.embed(["a cat sits on the mat", "a kitten rests on a rug", "stock prices fell"])
    print("cosine(cat, kitten) =", float(v[0] @ v[1]), " cosine(cat, stocks) =", float(v[0] @ v[2]))
