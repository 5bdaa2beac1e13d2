"""Shaping a corpus before indexing with RAG tuners: keep only markdown files, strip headings markup and
normalise whitespace, then answer questions from the tuned index (the reference's RagTunerHelloWorld, on this
engine).

    python examples/rag_tuner_hello.py [MODEL] [DOCUMENT FOLDER]
"""
import re
import sys
import time

import demo_models  # noqa: F401
from demo_models import chat_model, corpus_folder

from nanovllm_b200.api.factory import LlmModelFactory
from nanovllm_b200.llm import LLM
from nanovllm_b200.rag import RagFactory
from nanovllm_b200.rag.corpus import RagTuner


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    path = chat_model(argv[0] if argv else None)
    docs = argv[1] if len(argv) > 1 else corpus_folder()
    t0 = time.perf_counter()
    index = (RagFactory.builder().for_tiny_models()
             .add_processor(RagTuner.allowing(lambda r: r.file_name().endswith(".md")),      # filter
                            RagTuner.preprocessing(lambda t: re.sub(r"^#+\s*", "", t, flags=re.M)),
                            RagTuner.preprocessing(lambda t: re.sub(r"[ \t]+", " ", t)))     # pipeline
             .add_folder(docs).build())
    print(f"BM25 chunks after tuning: {index.size()}")
    model = LlmModelFactory.make(path)
    llm = LLM.builder(model).max_model_len(2048).max_num_seqs(2).system_prompt("").deterministic().build()
    rag = llm.rag(index, 96).top_k(3).max_context(1800)
    for q in ("When was the collection of tales first published?", "Where did the father work?"):
        r = rag.send(q)
        print(f"\nQ: {q}\nA: {r.answer}")
        for hit in rag.last_hits:
            print(f"  {hit.score:.3f}  {hit.chunk.source}")
    print(f"Time taken: {(time.perf_counter() - t0) * 1000:.0f} ms")
    llm.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
