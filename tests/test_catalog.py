"""Binding a checkpoint from its headers alone (the reference's ContainerCatalog / ModelBindingTest): the
architecture, the config and the tensor inventory come out of GGUF, safetensors and ONNX containers while every
payload accessor is disabled; an incomplete checkpoint is rejected before loading."""
import json

import pytest
import torch

from nanovllm_b200.config import HfConfig
from nanovllm_b200.exceptions import ModelLoadException
from nanovllm_b200.loaders import catalog as C
from nanovllm_b200.loaders import model_support as MS
from nanovllm_b200.models.registry import init_random_weights
from nanovllm_b200.models.writers import write_gguf_model, write_hf_folder
from tests.test_models_cpu import bert_tiny, gemma3_tiny, lfm2_tiny


def _qwen3_tiny():
    return HfConfig(vocab_size=300, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                    num_attention_heads=4, num_key_value_heads=2, head_dim=32, max_position_embeddings=512,
                    model_type="qwen3", architectures=["Qwen3ForCausalLM"], tie_word_embeddings=False)


@pytest.fixture
def no_payloads(monkeypatch):
    """Every call that would read tensor bytes raises: binding must not need them."""
    from nanovllm_b200.loaders import gguf, onnx, safetensors

    def boom(*a, **k):
        raise AssertionError("a payload was read while binding")
    for cls, names in ((gguf.GgufFile, ("get", "packed")), (safetensors.SafetensorsFile, ("get", "raw"))):
        for n in names:
            if hasattr(cls, n):
                monkeypatch.setattr(cls, n, boom)
    monkeypatch.setattr(onnx, "_tensor_to_torch", boom)


def test_bind_safetensors_and_gguf_without_payloads(tmp_path, no_payloads):
    hf = _qwen3_tiny()
    w = init_random_weights(hf, 0)
    st = C.ContainerCatalog.bind(write_hf_folder(str(tmp_path / "q3"), hf, w, shards=2))
    assert (st.container, st.architecture) == ("safetensors", MS.QWEN3)
    assert st.hf.hidden_size == 128 and st.names() == sorted(w)
    assert st.shape("model.layers.1.mlp.down_proj.weight") == (128, 256)
    assert st.missing() == [] and st.mismatched() == []
    gg = C.ContainerCatalog.bind(write_gguf_model(str(tmp_path / "q3.gguf"), hf, w, "Q8_0"))
    assert (gg.container, gg.architecture) == ("gguf", MS.QWEN3)
    assert gg.tensors["model.layers.0.self_attn.q_proj.weight"].dtype == "Q8_0"
    assert gg.require_complete() is gg
    lf = lfm2_tiny()
    lc = C.ContainerCatalog.bind(write_gguf_model(str(tmp_path / "lfm2.gguf"), lf, init_random_weights(lf, 3),
                                                  "Q4_K", big_type="Q6_K", random_packed=True))
    assert lc.architecture == MS.LFM2 and lc.hf.is_conv_layer(0) and not lc.hf.is_conv_layer(1)
    assert lc.tensors["blk.0.ffn_down.weight"].dtype == "Q6_K" and lc.missing() == []
    g3 = gemma3_tiny()
    gc = C.ContainerCatalog.bind(write_hf_folder(str(tmp_path / "g3"), g3, init_random_weights(g3, 2)))
    assert gc.architecture == MS.GEMMA3 and gc.missing() == []


def test_bind_onnx_bert_without_payloads(tmp_path, no_payloads):
    from nanovllm_b200.loaders.onnx import write_onnx
    hf = bert_tiny()
    w = init_random_weights(hf, 1)
    rev = {"token_embd.weight": "embeddings.word_embeddings.weight",
           "position_embd.weight": "embeddings.position_embeddings.weight",
           "token_types.weight": "embeddings.token_type_embeddings.weight",
           "token_embd_norm.weight": "embeddings.LayerNorm.weight", "token_embd_norm.bias": "embeddings.LayerNorm.bias"}
    sub = {"attn_q": "attention.self.query", "attn_k": "attention.self.key", "attn_v": "attention.self.value",
           "attn_output": "attention.output.dense", "attn_output_norm": "attention.output.LayerNorm",
           "ffn_up": "intermediate.dense", "ffn_down": "output.dense", "layer_output_norm": "output.LayerNorm"}
    onnx_w, mm = {}, {}
    for k, v in w.items():
        if k in rev:
            onnx_w[rev[k]] = v.float()
            continue
        _, i, part, kind = k.split(".")
        if kind == "weight" and "norm" not in part:
            anon = f"onnx::MatMul_{len(mm) + 100}"
            onnx_w[anon] = v.float().t().contiguous()
            mm[anon] = f"/encoder/layer.{i}/{sub[part].replace('.', '/')}/MatMul"
        else:
            onnx_w[f"encoder.layer.{i}.{sub[part]}.{kind}"] = v.float()
    d = tmp_path / "bert_onnx"
    d.mkdir()
    write_onnx(str(d / "model.onnx"), onnx_w, mm)
    (d / "config.json").write_text(json.dumps(hf.to_dict()))
    cat = C.ContainerCatalog.bind(str(d))
    assert (cat.container, cat.architecture) == ("onnx", MS.BERT)
    # MatMul operands behind anonymous initializers come out under their layer names, as [out, in]
    assert cat.shape("blk.0.ffn_up.weight") == (hf.intermediate_size, hf.hidden_size)
    assert cat.missing() == [] and cat.mismatched() == []


def test_incomplete_or_wrong_checkpoint_rejected_at_bind(tmp_path):
    hf = _qwen3_tiny()
    w = init_random_weights(hf, 0)
    del w["model.layers.1.self_attn.k_proj.weight"]
    w["model.layers.0.mlp.up_proj.weight"] = torch.zeros(255, 128, dtype=torch.bfloat16)
    cat = C.ContainerCatalog.bind(write_hf_folder(str(tmp_path / "bad"), hf, w))
    assert cat.missing() == ["model.layers.1.self_attn.k_proj.weight"]
    assert cat.mismatched() == [("model.layers.0.mlp.up_proj.weight", (256, 128), (255, 128))]
    with pytest.raises(ModelLoadException):
        cat.require_complete()
    with pytest.raises(ModelLoadException):
        C.ContainerCatalog.bind(str(tmp_path / "nothing-here"))


def test_factory_exposes_the_catalog(tmp_path):
    from nanovllm_b200.api.factory import LlmModelFactory
    hf = _qwen3_tiny()
    cat = LlmModelFactory.catalog(write_hf_folder(str(tmp_path / "q"), hf, init_random_weights(hf, 0)))
    assert cat.architecture == MS.QWEN3 and cat.require_complete().hf.num_hidden_layers == 2
