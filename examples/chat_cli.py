"""Interactive terminal app: chat over any supported checkpoint (optionally grounded on documents and helped by
advisors), or an embedding REPL when the checkpoint is an embedding model.  The reference's sample terminal app
(nano-vllm-java-samples/.../Example.java) on this engine.

    python examples/chat_cli.py --model PATH [--rag-mode none|bm25|dense|hybrid] [--docs FOLDER]
                                [--embed EMBEDDING_MODEL] [--advisors N] [--system TEXT] [--think] [--debug]

Without --model a tiny random checkpoint is built (fluent nonsense, but every path of the app runs).
Commands: /exit, /clear (forget the dialog), /rag on|off.  Thinking goes to stderr, answers to stdout; --debug
prints every prompt sent to the model.  With an embedding model each line is embedded and compared (cosine)
with the previous line.
"""
import argparse
import sys

import demo_models  # noqa: F401  (puts the checkout on sys.path)
from demo_models import chat_model, corpus_folder, embedding_model

from nanovllm_b200.api.factory import LlmModelFactory
from nanovllm_b200.chat import ChatSession, LlmListeners
from nanovllm_b200.chat.session import LlmAdvisor
from nanovllm_b200.config import EngineConfig
from nanovllm_b200.llm import LLM
from nanovllm_b200.rag import RagFactory, RagLoadOptions, RagSession
from nanovllm_b200.rag.dense import DenseRagIndex
from nanovllm_b200.sampling_params import SamplingParams

ADVISOR_ROLES = [("Facts", "List the facts the question depends on, one per line."),
                 ("Skeptic", "Name one thing the answer could get wrong, in one sentence."),
                 ("Editor", "Suggest the shortest clear form for the answer.")]


def _lines(prompt: str, script):
    """Input lines: a scripted list (tests) or the terminal."""
    if script is not None:
        yield from script
        return
    while True:
        try:
            yield input(prompt)
        except (EOFError, KeyboardInterrupt):
            return


def embed_repl(model, script=None) -> int:
    print(f"embedding model {model.architecture_name}; type sentences (/exit)", file=sys.stderr)
    prev = None
    for line in _lines("\nembed> ", script):
        line = line.strip()
        if line == "/exit":
            break
        if not line:
            continue
        v = model.embed(line)
        msg = f"dim={v.numel()} preview=[{', '.join(f'{float(x):.3f}' for x in v[:4])}, ...]"
        if prev is not None:
            msg += f"  cos(previous)={float((v * prev).sum()):.4f}"
        print(msg)
        prev = v
    return 0


def main(argv=None, script=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default=None, help="HF folder, .gguf file or ONNX folder")
    ap.add_argument("--rag-mode", choices=["none", "bm25", "dense", "hybrid"], default="none")
    ap.add_argument("--docs", default=None, help="folder or file of documents for retrieval")
    ap.add_argument("--embed", default=None, help="embedding model (BERT family) for dense / hybrid retrieval")
    ap.add_argument("--advisors", type=int, default=0, help=f"advisors run before each turn (0..{len(ADVISOR_ROLES)})")
    ap.add_argument("--system", default="")
    ap.add_argument("--think", action="store_true", help="let the model think before answering")
    ap.add_argument("--debug", action="store_true", help="print the prompts sent to the model")
    ap.add_argument("--max-tokens", type=int, default=512)
    ap.add_argument("--temperature", type=float, default=0.6)
    a = ap.parse_args(argv)

    listener = LlmListeners.to_print_streams()
    model = LlmModelFactory.make(chat_model(a.model), {"listener": LlmListeners.silent()})
    if model.is_embedding():
        return embed_repl(model, script)
    llm = LLM(model, EngineConfig(max_num_seqs=4, max_model_len=4096))
    sp = SamplingParams(temperature=a.temperature, max_tokens=a.max_tokens)
    advisors = [LlmAdvisor(n, p) for n, p in ADVISOR_ROLES[:max(0, min(a.advisors, len(ADVISOR_ROLES)))]]
    chat = ChatSession(llm, system_prompt=a.system, sampling=sp, enable_thinking=a.think, listener=listener,
                       advisors=advisors, emit_debug_prompts=a.debug)
    rag = None
    if a.rag_mode != "none":
        docs = a.docs or corpus_folder()
        lexical = RagFactory.make(docs, RagLoadOptions.for_tiny_models())
        if a.rag_mode == "bm25":
            index = lexical
        else:
            encoder = LlmModelFactory.make(embedding_model(a.embed))
            index = DenseRagIndex.of(lexical, encoder) if a.rag_mode == "dense" \
                else RagFactory.with_embeddings(lexical, encoder)
        rag = RagSession(llm, index, chat=chat, sampling=sp)
    use_rag = rag is not None
    print(f"model: {model}  rag={a.rag_mode} advisors={len(advisors)}  (/exit, /clear, /rag on|off)", file=sys.stderr)
    for line in _lines("\n> ", script):
        line = line.strip()
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
        print()
        if reply.stats is not None:
            print(f"[{reply.stats}]", file=sys.stderr)
    llm.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
