"""Continue a seed text token by token and print every sampled token as it streams (the reference's
NextTokenHelloWorld, on this engine).

    python examples/next_token_hello.py [MODEL] [SEED TEXT]
"""
import sys
import time

import demo_models  # noqa: F401
from demo_models import chat_model

from nanovllm_b200.api.factory import LlmModelFactory
from nanovllm_b200.llm import LLM
from nanovllm_b200.sampling_params import SamplingParams

SEED = "The capital of France is"
NEXT = 8


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    path = chat_model(argv[0] if argv else None)
    seed = argv[1] if len(argv) > 1 else SEED
    t0 = time.perf_counter()
    model = LlmModelFactory.make(path)
    llm = LLM.builder(model).max_model_len(256).max_num_seqs(1).build()
    tok = llm.tokenizer
    ids = tok.encode(seed)
    print(f"seed: {seed}\nprompt tokens: {ids}\nnext {NEXT} tokens:")
    out = llm.generate_token_ids([ids], SamplingParams(temperature=0.2, max_tokens=NEXT, seed=7),
                                 on_token=lambda i, sid, t: print(f"  {t}\t{tok.decode([t])!r}"))[0]
    text = tok.decode(out.token_ids)
    print(f"continuation: {text!r}\nfull text: {seed + text!r}")
    print(f"Time taken: {(time.perf_counter() - t0) * 1000:.0f} ms")
    llm.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
