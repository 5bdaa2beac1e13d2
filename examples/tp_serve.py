"""Tensor-parallel serving with one front door: one process per GPU, rank 0 takes the prompts and streams the
answers, every other rank follows rank 0's step plans (``LLM.serve_worker``) -- no rank but 0 needs the requests.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 --master-port 29500 examples/tp_serve.py [MODEL] [PROMPT ...]

Without a model path a tiny random Qwen3 is built (the same on every rank), so the output is fluent nonsense.
"""
import sys
import time

import demo_models  # noqa: F401
from demo_models import chat_model

from nanovllm_b200.api.factory import LlmModelFactory
from nanovllm_b200.llm import LLM
from nanovllm_b200.parallel import state as ps
from nanovllm_b200.sampling_params import SamplingParams

PROMPTS = ["The capital of France is", "Once upon a time", "1, 2, 3,"]


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    ps.init_tp()
    rank = ps.tp_rank()
    path = chat_model(argv[0] if argv else None)
    prompts = argv[1:] or PROMPTS
    t0 = time.perf_counter()
    llm = LLM.builder(LlmModelFactory.make(path)).max_model_len(256).max_num_seqs(4).front_door("rank0").build()
    try:
        if llm.is_worker:
            steps = llm.serve_worker()
            print(f"rank {rank}: followed {steps} steps of rank 0")
        else:
            outs = llm.generate(prompts, SamplingParams(temperature=0.7, top_k=20, max_tokens=12, seed=3))
            for p, o in zip(prompts, outs):
                print(f"{p!r} -> {o.text!r}")
            print(f"rank 0 of {ps.tp_size()}: {len(outs)} answers, Time taken: "
                  f"{(time.perf_counter() - t0) * 1000:.0f} ms")
            llm.close()  # tells the workers to stop
    finally:
        ps.destroy()
    return 0


if __name__ == "__main__":
    sys.exit(main())
