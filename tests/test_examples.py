"""Every example program runs end to end on the CPU with the tiny random checkpoints it builds itself (the
reference's samples module: HelloWorld, EmbeddingsHelloWorld, NextTokenHelloWorld, LogTriageHelloWorld,
AdvisorRagHelloWorld, RagTunerHelloWorld)."""
import importlib
import os
import sys

import pytest

EXAMPLES = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "examples")


@pytest.mark.parametrize("name", ["embeddings_hello", "next_token_hello", "log_triage_hello", "advisor_rag_hello",
                                  "rag_tuner_hello"])
def test_example_runs(name, capsys, monkeypatch):
    monkeypatch.syspath_prepend(EXAMPLES)
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "")  # examples pick the GPU when present; keep this test on CPU
    mod = importlib.import_module(name)
    assert mod.main([]) == 0
    out = capsys.readouterr().out
    assert "Time taken" in out or "[timing] total" in out
    if name == "embeddings_hello":
        assert "cos(same)=1.0000" in out
    if name in ("advisor_rag_hello", "rag_tuner_hello"):
        assert "chunks" in out


@pytest.mark.parametrize("args", [["--rag-mode", "hybrid", "--advisors", "2", "--debug"], ["--rag-mode", "bm25"],
                                  ["--rag-mode", "dense"], []])
def test_terminal_app_chat_modes(args, capsys, monkeypatch):
    monkeypatch.syspath_prepend(EXAMPLES)
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "")
    app = importlib.import_module("chat_cli")
    assert app.main(args + ["--max-tokens", "8"], script=["Who collected the tales?", "/rag off", "/clear",
                                                           "And Paris?", "/exit"]) == 0


def test_terminal_app_embedding_repl(capsys, monkeypatch):
    monkeypatch.syspath_prepend(EXAMPLES)
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "")
    app = importlib.import_module("chat_cli")
    from demo_models import embedding_model
    assert app.main(["--model", embedding_model()], script=["a first sentence", "a first sentence", "/exit"]) == 0
    out = capsys.readouterr().out
    assert "cos(previous)=1.0000" in out
