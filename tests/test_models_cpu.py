"""Model families and loaders on the CPU oracle path: Gemma3 (sliding / global, sandwich norms), LFM2 (short-conv
state across chunked prefill and decode), BERT embeddings, and LlmModelFactory round trips through HF safetensors
folders, GGUF files (Q8_0 / F16 / random K-quant blocks) and ONNX initializer files (reference analogues:
ModelBindingTest, BertEmbeddingTest, the Lfm2 / Gemma load tests, GgufUnitTest's ShortConv identity)."""
import math
import os

import pytest
import torch

from nanovllm_b200.api.factory import LlmModelFactory
from nanovllm_b200.config import EngineConfig, HfConfig
from nanovllm_b200.engine.sequence import Sequence
from nanovllm_b200.exceptions import UnsupportedModelException
from nanovllm_b200.llm import LLM
from nanovllm_b200.models.registry import init_random_weights
from nanovllm_b200.models.writers import write_gguf_model, write_hf_folder
from nanovllm_b200.sampling_params import SamplingParams

GREEDY = SamplingParams(max_tokens=5, ignore_eos=True).deterministic()


def _cfg(**kw):
    c = dict(max_num_seqs=4, max_model_len=1024, num_kvcache_blocks=12, max_num_batched_tokens=512,
             stop_on_degenerate=False)
    c.update(kw)
    return EngineConfig(**c)


def _prefill_logits(llm, ids):
    s = Sequence(ids, SamplingParams(max_tokens=1), 256)
    bm = llm.scheduler.block_manager
    bm.allocate(s, 0)
    s.num_scheduled_tokens = len(ids)
    out = llm.runner.forward_logits([s], True)[0].float()
    bm.deallocate(s)
    llm.runner.release_state(s)
    return out


def gemma3_tiny():
    return HfConfig(vocab_size=300, hidden_size=128, intermediate_size=256, num_hidden_layers=3, num_attention_heads=2,
                    num_key_value_heads=1, head_dim=64, max_position_embeddings=2048, model_type="gemma3_text",
                    architectures=["Gemma3ForCausalLM"], sliding_window=16, query_pre_attn_scalar=64,
                    rope_local_base_freq=10000.0, rope_theta=1e6, tie_word_embeddings=True,
                    layer_types=["sliding_attention", "sliding_attention", "full_attention"])


def lfm2_tiny():
    return HfConfig(vocab_size=300, hidden_size=128, intermediate_size=256, num_hidden_layers=4, num_attention_heads=2,
                    num_key_value_heads=2, head_dim=64, max_position_embeddings=2048, model_type="lfm2",
                    layer_types=["conv", "full_attention", "conv", "full_attention"], layer_kv_heads=[0, 2, 0, 2],
                    conv_l_cache=3, rope_theta=1e6)


def bert_tiny():
    return HfConfig(vocab_size=300, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                    num_key_value_heads=4, head_dim=16, max_position_embeddings=128, model_type="bert",
                    layer_norm_eps=1e-12)


def _decode_consistency(llm, prompt, steps=4):
    out = llm.generate_token_ids([prompt], SamplingParams(max_tokens=steps + 1, ignore_eos=True).deterministic())[0]
    seq = prompt + out.token_ids
    for k in range(1, steps + 1):
        logits = _prefill_logits(llm, seq[:len(prompt) + k])
        assert int(torch.argmax(logits)) == seq[len(prompt) + k], k


def test_gemma3_decode_matches_prefill_with_sliding_window():
    hf = gemma3_tiny()
    llm = LLM((hf, init_random_weights(hf, 2)), _cfg(), device="cpu")
    _decode_consistency(llm, list(range(3, 40)))  # prompt longer than the window


def test_lfm2_conv_state_across_chunks_and_decode():
    hf = lfm2_tiny()
    w = init_random_weights(hf, 3)
    prompt = list(range(5, 305))
    a = LLM((hf, w), _cfg(max_num_batched_tokens=128), device="cpu").generate_token_ids([prompt], GREEDY)[0]
    b = LLM((hf, w), _cfg(max_num_batched_tokens=1024), device="cpu").generate_token_ids([prompt], GREEDY)[0]
    assert a.token_ids == b.token_ids  # chunked prefill carries the conv state correctly
    llm = LLM((hf, w), _cfg(), device="cpu")
    assert not llm.scheduler.block_manager.prefix_caching
    _decode_consistency(llm, list(range(9, 50)))


def test_bert_embedding_matches_direct_math():
    from nanovllm_b200.models.bert import BertEncoder
    hf = bert_tiny()
    w = init_random_weights(hf, 1)
    for k in list(w):
        if k.endswith(".bias"):
            w[k] = torch.randn_like(w[k].float()).mul(0.02).bfloat16()
    enc = BertEncoder(hf, w, torch.device("cpu"))
    ids = [[2, 7, 9, 11, 3], [2, 5, 3]]
    got = enc.embed_ids(ids)

    def ln(x, g, b):
        m = x.mean(-1, keepdim=True)
        v = ((x - m) ** 2).mean(-1, keepdim=True)
        return (x - m) / torch.sqrt(v + 1e-12) * g + b

    f = {k: v.float() for k, v in w.items()}
    for n, s in enumerate(ids):
        x = f["token_embd.weight"][s] + f["position_embd.weight"][:len(s)] + f["token_types.weight"][0]
        x = ln(x, f["token_embd_norm.weight"], f["token_embd_norm.bias"])
        for i in range(hf.num_hidden_layers):
            p = f"blk.{i}."
            q = x @ f[p + "attn_q.weight"].t() + f[p + "attn_q.bias"]
            k = x @ f[p + "attn_k.weight"].t() + f[p + "attn_k.bias"]
            v = x @ f[p + "attn_v.weight"].t() + f[p + "attn_v.bias"]
            hd = 16
            q, k, v = (t.view(len(s), 4, hd).transpose(0, 1) for t in (q, k, v))
            a = torch.softmax(q @ k.transpose(1, 2) / math.sqrt(hd), -1) @ v
            a = a.transpose(0, 1).reshape(len(s), -1) @ f[p + "attn_output.weight"].t() + f[p + "attn_output.bias"]
            x = ln(x + a, f[p + "attn_output_norm.weight"], f[p + "attn_output_norm.bias"])
            h = x @ f[p + "ffn_up.weight"].t() + f[p + "ffn_up.bias"]
            h = 0.5 * h * (1 + torch.tanh(0.7978845608 * (h + 0.044715 * h ** 3)))
            h = h @ f[p + "ffn_down.weight"].t() + f[p + "ffn_down.bias"]
            x = ln(x + h, f[p + "layer_output_norm.weight"], f[p + "layer_output_norm.bias"])
        e = x.mean(0)
        e = e / e.norm()
        assert torch.nn.functional.cosine_similarity(e, got[n], dim=0) > 0.999
        assert abs(float(got[n].norm()) - 1.0) < 1e-3


def test_factory_hf_folder_generate_text(tmp_path):
    hf = HfConfig(vocab_size=300, hidden_size=128, intermediate_size=256, num_hidden_layers=2, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=32, max_position_embeddings=2048, model_type="qwen3",
                  architectures=["Qwen3ForCausalLM"], tie_word_embeddings=False)
    w = init_random_weights(hf, 0)
    d = write_hf_folder(str(tmp_path / "q3"), hf, w, shards=2)
    m = LlmModelFactory.make(d, device="cpu")
    assert m.is_causal() and m.architecture_name == "Qwen3ForCausalLM" and m.container == "hf-safetensors"
    llm = LLM(m, _cfg(), device="cpu")
    out = llm.generate(["the then"], GREEDY)[0]
    assert len(out.token_ids) == 5 and isinstance(out.text, str)
    direct = LLM((hf, w), _cfg(), device="cpu")
    ids = m.tokenizer.encode("the then")
    assert torch.equal(_prefill_logits(llm, ids), _prefill_logits(direct, ids))


def test_factory_gguf_qwen3_q8_0_close_to_dense(tmp_path):
    hf = HfConfig(vocab_size=300, hidden_size=128, intermediate_size=256, num_hidden_layers=2, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=32, max_position_embeddings=2048, model_type="qwen3",
                  architectures=["Qwen3ForCausalLM"], tie_word_embeddings=False)
    w = init_random_weights(hf, 0)
    p = write_gguf_model(str(tmp_path / "q3.gguf"), hf, w, "Q8_0")
    m = LlmModelFactory.make(p, device="cpu")
    assert m.container == "gguf" and m.has_packed_weights()
    ids = list(range(3, 60))
    a = _prefill_logits(LLM(m, _cfg(), device="cpu"), ids)
    b = _prefill_logits(LLM((hf, w), _cfg(), device="cpu"), ids)
    assert torch.nn.functional.cosine_similarity(a, b, dim=0) > 0.99


def test_unpacked_engine_over_packed_gguf_model(tmp_path, monkeypatch):
    """An engine built with unpack_parameters over a model whose GGUF projections stay packed gets dense bf16
    copies (the model keeps its blocks) and the packed engine's logits within bf16 rounding."""
    from nanovllm_b200.ops.quant import GgufPacked
    hf = HfConfig(vocab_size=300, hidden_size=128, intermediate_size=256, num_hidden_layers=2, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=32, max_position_embeddings=2048, model_type="qwen3",
                  architectures=["Qwen3ForCausalLM"], tie_word_embeddings=False)
    p = write_gguf_model(str(tmp_path / "q3p.gguf"), hf, init_random_weights(hf, 0), "Q8_0")
    monkeypatch.setenv("NVB_GGUF_PACKED", "force")
    m = LlmModelFactory.make(p, device="cpu")
    n_packed = sum(isinstance(v, GgufPacked) for v in m.weights.values())
    assert n_packed > 0
    ids = list(range(3, 60))
    packed = LLM(m, _cfg(), device="cpu")
    assert all(isinstance(L.down.weight, GgufPacked) for L in packed.model.layers)
    a = _prefill_logits(packed, ids)
    llm = LLM(m, _cfg(), device="cpu", unpack_parameters=True)
    assert sum(isinstance(v, GgufPacked) for v in m.weights.values()) == n_packed
    assert all(isinstance(L.down.weight, torch.Tensor) for L in llm.model.layers)
    b = _prefill_logits(llm, ids)
    assert torch.nn.functional.cosine_similarity(a, b, dim=0) > 0.999


def test_factory_open_builder_unpacks_at_load(tmp_path, monkeypatch):
    """LlmModelFactory.open(path) builder knobs (LlmModelFactory.java:817-870): unpack_parameters expands the GGUF
    blocks during the load, listen / chat_specials / think_tags land in the model options."""
    from nanovllm_b200.chat.listeners import LlmListeners
    from nanovllm_b200.chat.markup import ChatSpecials, ThinkTags
    from nanovllm_b200.ops.quant import GgufPacked
    hf = HfConfig(vocab_size=300, hidden_size=128, intermediate_size=256, num_hidden_layers=2, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=32, max_position_embeddings=2048, model_type="qwen3",
                  architectures=["Qwen3ForCausalLM"], tie_word_embeddings=False)
    p = write_gguf_model(str(tmp_path / "q3o.gguf"), hf, init_random_weights(hf, 0), "Q8_0")
    monkeypatch.setenv("NVB_GGUF_PACKED", "force")
    listener, events = LlmListeners.collecting()
    packed = LlmModelFactory.open(p).device("cpu").build()
    assert any(isinstance(v, GgufPacked) for v in packed.weights.values())
    m = (LlmModelFactory.open(p).device("cpu").unpack_parameters().listen(listener)
         .chat_specials(ChatSpecials(("<x>",))).think_tags(ThinkTags("<t>", "</t>")).build())
    assert not any(isinstance(v, GgufPacked) for v in m.weights.values())
    assert m.chat_specials().markers == ("<x>",) and m.think_tags().open == "<t>" and events
    ids = list(range(3, 40))
    a = _prefill_logits(LLM(packed, _cfg(), device="cpu"), ids)
    b = _prefill_logits(LLM(m, _cfg(), device="cpu"), ids)
    assert torch.nn.functional.cosine_similarity(a, b, dim=0) > 0.999


def test_factory_gguf_lfm2_q4_k_m(tmp_path):
    hf = lfm2_tiny()
    w = init_random_weights(hf, 3)
    p = write_gguf_model(str(tmp_path / "lfm2.gguf"), hf, w, "Q4_K", big_type="Q6_K", random_packed=True)
    m = LlmModelFactory.make(p, device="cpu")
    assert m.hf_config.layer_types == hf.layer_types and m.hf_config.conv_l_cache == 3
    out = LLM(m, _cfg(), device="cpu").generate_token_ids([list(range(3, 90))], GREEDY)[0]
    assert len(out.token_ids) == 5


def test_factory_bert_gguf_and_onnx_agree(tmp_path):
    from nanovllm_b200.loaders.onnx import write_onnx
    hf = bert_tiny()
    w = init_random_weights(hf, 1)
    g = LlmModelFactory.make(write_gguf_model(str(tmp_path / "bert.gguf"), hf, w, "F16", tokenizer_model="bert"),
                             device="cpu")
    assert g.is_embedding()
    e1 = g.embed("abc de")
    # ONNX export naming (HF BERT names; MatMul weights stored [in, out] behind anonymous initializers)
    onnx_w, mm = {}, {}
    rev = {"token_embd.weight": "embeddings.word_embeddings.weight",
           "position_embd.weight": "embeddings.position_embeddings.weight",
           "token_types.weight": "embeddings.token_type_embeddings.weight",
           "token_embd_norm.weight": "embeddings.LayerNorm.weight", "token_embd_norm.bias": "embeddings.LayerNorm.bias"}
    sub = {"attn_q": "attention.self.query", "attn_k": "attention.self.key", "attn_v": "attention.self.value",
           "attn_output": "attention.output.dense", "attn_output_norm": "attention.output.LayerNorm",
           "ffn_up": "intermediate.dense", "ffn_down": "output.dense", "layer_output_norm": "output.LayerNorm"}
    for k, v in w.items():
        if k in rev:
            onnx_w[rev[k]] = v.float()
            continue
        _, i, part, kind = k.split(".")
        name = f"encoder.layer.{i}.{sub[part]}.{kind}"
        if kind == "weight" and "norm" not in part:
            anon = f"onnx::MatMul_{len(mm) + 100}"
            onnx_w[anon] = v.float().t().contiguous()
            mm[anon] = f"/encoder/layer.{i}/{sub[part].replace('.', '/')}/MatMul"
        else:
            onnx_w[name] = v.float()
    d = tmp_path / "bert_onnx"
    d.mkdir()
    write_onnx(str(d / "model.onnx"), onnx_w, mm)
    import json
    (d / "config.json").write_text(json.dumps(hf.to_dict()))
    (d / "tokenizer.json").write_text(json.dumps({
        "model": {"type": "WordPiece", "vocab": {t: i for i, t in enumerate(g.tokenizer.id_to_token)},
                  "unk_token": "[UNK]"}, "normalizer": {"type": "BertNormalizer", "lowercase": True},
        "pre_tokenizer": {"type": "BertPreTokenizer"}, "added_tokens": []}))
    o = LlmModelFactory.make(str(d), device="cpu")
    assert o.container == "onnx"
    e2 = o.embed("abc de")
    assert torch.nn.functional.cosine_similarity(e1, e2, dim=0) > 0.999


def test_model_support_rejections(tmp_path):
    from nanovllm_b200.loaders import model_support as MS
    for mt, arch in (("qwen2", "Qwen2ForCausalLM"), ("mixtral", "MixtralForCausalLM"), ("gemma2", "Gemma2ForCausalLM"),
                     ("qwen3_moe", "Qwen3MoeForCausalLM")):
        with pytest.raises(UnsupportedModelException) as e:
            MS.resolve(HfConfig(model_type=mt, architectures=[arch]))
        assert "Supported by this library" in str(e.value)
    with pytest.raises(UnsupportedModelException):
        MS.check_source(MS.Selection("gemma3", False), MS.SRC_GGUF)
    with pytest.raises(UnsupportedModelException):
        MS.check_source(MS.Selection("bert", True), MS.SRC_HF_SAFETENSORS)
    with pytest.raises(UnsupportedModelException):
        MS.check_source(MS.Selection("lfm2", False), MS.SRC_HF_SAFETENSORS)
    assert MS.resolve(HfConfig(model_type="qwen3", architectures=["Qwen3ForCausalLM"])).architecture == "qwen3"
    with pytest.raises(ValueError):
        LLM(LlmModelFactory.make(write_gguf_model(str(tmp_path / "b.gguf"), bert_tiny(),
                                                  init_random_weights(bert_tiny(), 1), "F16",
                                                  tokenizer_model="bert"), device="cpu"), _cfg(), device="cpu")
