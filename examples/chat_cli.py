"""Interactive terminal chat over any supported checkpoint, optionally grounded on a document folder (RAG).

    python examples/chat_cli.py --model /path/to/Qwen3-0.6B [--rag docs/] [--embed /path/to/bge.gguf]
                                [--system "You are terse."] [--think] [--tp 1]

Commands inside the session: /clear (forget the dialog), /rag on|off, /exit.  Thinking text is printed dimmed
on stderr, the answer on stdout (the listener decides; see chat.listeners.LlmListeners.to_print_streams).
Mirrors the reference's sample terminal app (nano-vllm-java-samples/.../Example.java) on this engine.
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))  # run from a checkout
import argparse
import sys

from nanovllm_b200.api.factory import LlmModelFactory
from nanovllm_b200.chat import ChatSession, LlmListeners
from nanovllm_b200.config import EngineConfig
from nanovllm_b200.llm import LLM
from nanovllm_b200.rag import RagFactory, RagLoadOptions, RagSession
from nanovllm_b200.sampling_params import SamplingParams


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", required=True, help="HF folder, .gguf file or ONNX folder")
    ap.add_argument("--rag", default=None, help="folder or file of documents to ground answers on")
    ap.add_argument("--embed", default=None, help="embedding model (BERT family) for hybrid retrieval")
    ap.add_argument("--system", default="")
    ap.add_argument("--think", action="store_true", help="let the model think before answering")
    ap.add_argument("--max-tokens", type=int, default=512)
    ap.add_argument("--temperature", type=float, default=0.6)
    a = ap.parse_args()

    listener = LlmListeners.to_system()
    model = LlmModelFactory.make(a.model, {"listener": listener})
    llm = LLM(model, EngineConfig(max_num_seqs=4))
    sp = SamplingParams(temperature=a.temperature, max_tokens=a.max_tokens)
    chat = ChatSession(llm, system_prompt=a.system, sampling=sp, enable_thinking=a.think, listener=listener)
    rag = None
    if a.rag:
        encoder = LlmModelFactory.make(a.embed) if a.embed else None
        index = RagFactory.make(a.rag, RagLoadOptions.for_tiny_models(), listener, encoder)
        rag = RagSession(llm, index, chat=chat, sampling=sp)
    use_rag = rag is not None
    print(f"model: {model}  (/exit, /clear, /rag on|off)", file=sys.stderr)
    while True:
        try:
            line = input("\n> ").strip()
        except (EOFError, KeyboardInterrupt):
            break
        if not line:
            continue
        if line == "/exit":
            break
        if line == "/clear":
            (rag or chat).clear()
            continue
        if line.startswith("/rag"):
            use_rag = rag is not None and line.endswith("on")
            print(f"rag {'on' if use_rag else 'off'}", file=sys.stderr)
            continue
        reply = rag.send(line) if use_rag else chat.send(line)
        if reply.stats is not None:
            print(f"\n[{reply.stats}]", file=sys.stderr)
    llm.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
