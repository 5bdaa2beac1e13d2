"""Checkpoints for the example programs: a user passes a real model path; without one the examples build a tiny
random-init checkpoint in a temporary folder (no network here, and the examples stay runnable and testable).
Random weights produce fluent-looking nonsense: the point is the API, not the answer."""
from __future__ import annotations

import os
import sys
import tempfile

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))  # run from a checkout

GRIMM = ("# The Brothers Grimm\n\nJacob Grimm (1785-1863) and Wilhelm Grimm (1786-1859) were German scholars who "
         "collected folk tales. Their father was Philipp Wilhelm Grimm, a jurist in Hanau. Their collection "
         "Children's and Household Tales was first published in 1812.\n")
PARIS = "Paris is the capital of France. It lies on the Seine river and has about two million inhabitants.\n"


def chat_model(path: str = None) -> str:
    """A chat checkpoint folder: ``path`` itself, or a tiny random Qwen3 with a byte-level BPE tokenizer."""
    if path:
        return path
    from nanovllm_b200.config import HfConfig
    from nanovllm_b200.models.registry import init_random_weights
    from nanovllm_b200.models.writers import byte_level_tokenizer_json, write_hf_folder
    hf = HfConfig(vocab_size=320, hidden_size=128, intermediate_size=256, num_hidden_layers=2, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=32, max_position_embeddings=4096, model_type="qwen3",
                  architectures=["Qwen3ForCausalLM"], tie_word_embeddings=True)
    d = os.path.join(tempfile.mkdtemp(prefix="nvb_demo_"), "tiny-qwen3")
    return write_hf_folder(d, hf, init_random_weights(hf, 0), tokenizer_json=byte_level_tokenizer_json(320))


def embedding_model(path: str = None) -> str:
    """An embedding checkpoint: ``path`` itself, or a tiny random BERT stored as GGUF with a WordPiece vocab."""
    if path:
        return path
    from nanovllm_b200.config import HfConfig
    from nanovllm_b200.models.registry import init_random_weights
    from nanovllm_b200.models.writers import write_gguf_model
    hf = HfConfig(vocab_size=300, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                  num_key_value_heads=4, head_dim=16, max_position_embeddings=256, model_type="bert",
                  layer_norm_eps=1e-12)
    p = os.path.join(tempfile.mkdtemp(prefix="nvb_demo_"), "tiny-bert.gguf")
    return write_gguf_model(p, hf, init_random_weights(hf, 1), "F16", tokenizer_model="bert")


def corpus_folder() -> str:
    """A small document folder (markdown + text) for the retrieval examples."""
    d = tempfile.mkdtemp(prefix="nvb_corpus_")
    with open(os.path.join(d, "grimm.md"), "w") as f:
        f.write(GRIMM)
    with open(os.path.join(d, "paris.txt"), "w") as f:
        f.write(PARIS)
    return d
