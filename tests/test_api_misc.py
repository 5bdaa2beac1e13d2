"""Model file sources, capped JSON parsing and the load progress bar."""
import os

import pytest

from nanovllm_b200.api.factory import LlmModelFactory
from nanovllm_b200.api.sources import ModelFileId, ModelFileSources
from nanovllm_b200.chat.listeners import LlmListeners, LlmTextKind
from nanovllm_b200.exceptions import ModelLoadException
from nanovllm_b200.utils import json_limits
from nanovllm_b200.utils.progress import LoadProgress


def test_json_caps():
    assert json_limits.loads('{"a": [1, {"b": 2}]}') == {"a": [1, {"b": 2}]}
    assert json_limits.max_depth('{"s": "[[[[", "x": [[1]]}') == 3
    with pytest.raises(ModelLoadException):
        json_limits.loads("[" * 70 + "]" * 70)
    with pytest.raises(ModelLoadException):
        json_limits.loads('{"a": 1}', size_cap=3)
    with pytest.raises(ModelLoadException):
        json_limits.loads('{"a": }')


def test_load_progress_reports_through_listener():
    listener, events = LlmListeners.collecting()
    p = LoadProgress("weights", 4, listener)
    for i in range(4):
        p.step(f"tensor {i}")
    p.finish("4 tensors")
    p.finish("again")  # idempotent
    prog = [e for e in events if e.kind == LlmTextKind.STATUS_PROGRESS]
    assert len(prog) == 5 and "100%" in prog[-1].text and "(4/4)" in prog[-1].text
    infos = [e for e in events if e.kind == LlmTextKind.STATUS_INFO]
    assert len(infos) == 1 and "done in" in infos[0].text


def test_sources_bytes_and_path_load_the_same_model(tmp_path):
    from test_cpu_model import tiny
    from nanovllm_b200.models.registry import init_random_weights
    from nanovllm_b200.models.writers import byte_level_tokenizer_json, write_hf_folder
    hf = tiny(vocab_size=300)
    d = write_hf_folder(str(tmp_path / "m"), hf, init_random_weights(hf, 0), byte_level_tokenizer_json(300))
    src = ModelFileSources.from_path(d)
    assert src.open(ModelFileId.CONFIG) is not None and src.open(ModelFileId.MODEL_ONNX) is None
    mem = ModelFileSources.from_bytes({n: open(os.path.join(d, n), "rb").read() for n in os.listdir(d)})
    a = LlmModelFactory.make(src, device="cpu")
    b = LlmModelFactory.make(mem, device="cpu")
    assert a.hf_config.hidden_size == b.hf_config.hidden_size
    assert set(a.weights) == set(b.weights)
    assert mem._dir is None  # spooled folder removed after the load
