"""Retrieval-augmented answers with an advisor: a BM25 index over a small document folder, an advisor that
collects facts before every turn, and the retrieved passages printed with their scores (the reference's
AdvisorRagHelloWorld, on this engine).

    python examples/advisor_rag_hello.py [MODEL] [DOCUMENT FOLDER]
"""
import sys
import time

import demo_models  # noqa: F401
from demo_models import chat_model, corpus_folder

from nanovllm_b200.api.factory import LlmModelFactory
from nanovllm_b200.chat import LlmListeners
from nanovllm_b200.chat.session import LlmAdvisor
from nanovllm_b200.llm import LLM
from nanovllm_b200.rag import RagFactory, RagLoadOptions

QUESTIONS = ("What are the names of the Grimm brothers?", "Who was the Grimm brothers' father?")


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    path = chat_model(argv[0] if argv else None)
    docs = argv[1] if len(argv) > 1 else corpus_folder()
    t0 = time.perf_counter()
    model = LlmModelFactory.make(path)
    llm = LLM.builder(model).max_model_len(2048).max_num_seqs(4).system_prompt("") \
        .advisors(LlmAdvisor("Alex", "Find facts and shortly present them.")).build()
    corpus = RagFactory.make(docs, RagLoadOptions.for_tiny_models())
    print(f"BM25 chunks: {corpus.size()}")
    rag = llm.rag(corpus, 128, isolate_generation=True).top_k(2).max_context(900)
    rag.chat.listener = LlmListeners.to_print_streams()  # thinking -> stderr, answer -> stdout
    for q in QUESTIONS:
        print(f"\nQ: {q}")
        r = rag.send(q)
        print(f"\nA: {r.answer}")
        for hit in rag.last_hits:
            print(f"  {hit.score:.3f}  {hit.chunk.source}")
    print(f"Time taken: {(time.perf_counter() - t0) * 1000:.0f} ms")
    llm.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
