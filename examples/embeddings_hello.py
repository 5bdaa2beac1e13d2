"""Sentence embeddings: load a BERT-family model, embed a sentence twice, a related and an unrelated one, and
print the cosine similarities (the reference's EmbeddingsHelloWorld, on this engine).

    python examples/embeddings_hello.py [MODEL (.gguf / ONNX folder)] [TEXT]
"""
import sys
import time

import demo_models  # noqa: F401  (puts the checkout on sys.path)
from demo_models import embedding_model

from nanovllm_b200.api.factory import LlmModelFactory

TEXT = "The capital of France is Paris."
RELATED = "Paris is the capital city of France."
UNRELATED = "A completely different sentence about astronomy."


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    path = embedding_model(argv[0] if argv else None)
    text = argv[1] if len(argv) > 1 else TEXT
    t0 = time.perf_counter()
    model = LlmModelFactory.make(path)
    print(f"architecture={model.architecture_name} embedding={model.is_embedding()} "
          f"modalities={model.modalities()}")
    v = model.embed(text)
    same, related, other = model.embed(text), model.embed(RELATED), model.embed(UNRELATED)
    print(f"text: {text}\ndim={v.numel()}  L2={float(v.norm()):.4f}")
    print("preview: " + ", ".join(f"{float(x):.4f}" for x in v[:8]))
    cos = lambda a, b: float((a * b).sum())  # noqa: E731 (unit vectors)
    print(f"cos(same)={cos(v, same):.4f}\ncos(related)={cos(v, related):.4f}  {RELATED}")
    print(f"cos(unrelated)={cos(v, other):.4f}  {UNRELATED}")
    print(f"Time taken: {(time.perf_counter() - t0) * 1000:.0f} ms")
    model.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
