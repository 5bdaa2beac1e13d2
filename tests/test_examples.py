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
