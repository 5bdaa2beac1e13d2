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


def _tiny_qwen():
    from nanovllm_b200.config import HfConfig
    from nanovllm_b200.models.registry import init_random_weights
    hf = HfConfig(vocab_size=300, hidden_size=128, intermediate_size=256, num_hidden_layers=1, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=32, max_position_embeddings=512, model_type="qwen3")
    return hf, init_random_weights(hf, 1)


def test_builder_knobs_of_the_reference_builder(monkeypatch):
    """LLM.java:1499-1870 builder knobs: system prompt / advisors overrides, KV memory share, CPU workers,
    unpacking, warm-up switches."""
    import torch
    from nanovllm_b200.chat import session
    from nanovllm_b200.llm import LLM
    threads = torch.get_num_threads()
    try:
        b = (LLM.builder(_tiny_qwen()).device("cpu").num_kvcache_blocks(8).max_model_len(256).kv_heap_fraction(0.5)
             .disable_multi_cpu().system_prompt("be brief").no_system_prompt().advisors(object()).no_advisors()
             .warmup().skip_warmup().advisor_note_filter(lambda s: "keep" in s))
        llm = b.build()
        assert llm.cfg.gpu_memory_utilization == 0.5
        assert torch.get_num_threads() == 1
        assert llm.system_prompt == "" and llm.advisors == [] and llm.advisor_mixer is None
        seen = {}
        monkeypatch.setattr(session.AdvisorRunner, "enrich",
                            staticmethod(lambda *a, **kw: seen.update(kw) or "enriched"))
        assert llm.run_advisors("hello") == "enriched"
        assert seen["note_filter"]("keep this") and not seen["note_filter"]("drop")
        llm2 = LLM.builder(_tiny_qwen()).device("cpu").num_kvcache_blocks(8).max_model_len(256) \
            .system_prompt("x").default_system_prompt().build()
        assert llm2.system_prompt == ""
    finally:
        torch.set_num_threads(threads)
    with pytest.raises(ValueError):
        LLM.builder(_tiny_qwen()).cpu_threads(0)
    with pytest.raises(ValueError):
        LLM.builder(_tiny_qwen()).device("cpu").kv_heap_fraction(0.0).build()
    with pytest.raises(TypeError):
        LLM.builder(_tiny_qwen()).advisor_note_filter("not callable")


def test_model_chat_specials_option_and_engine_accessors():
    from nanovllm_b200.api.model import LlmModel
    from nanovllm_b200.chat.markup import ChatSpecials
    from nanovllm_b200.llm import LLM
    hf, w = _tiny_qwen()
    m = LlmModel(hf, w, options={"chat_specials": ["<|x|>"]})
    assert m.chat_specials().markers == ("<|x|>",)
    assert LlmModel(hf, w).chat_specials() == ChatSpecials.default()
    llm = LLM.builder(m).device("cpu").num_kvcache_blocks(8).max_model_len(256).build()
    assert llm.chat_specials().markers == ("<|x|>",) and not llm.is_closed()
    assert m.input_modalities() == ["text"] and m.output_modalities() == ["text"] and m.path == ""
    llm.close()
    assert llm.is_closed()
