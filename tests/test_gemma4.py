"""Gemma4 (text, QAT): packing, loader round trip, SRQ, and the engine graph against a plain fp32 restatement."""
import math

import pytest
import torch

from nanovllm_b200.config import EngineConfig, HfConfig
from nanovllm_b200.llm import LLM
from nanovllm_b200.loaders.gemma4_qat import (QatWeight, infer_bits, infer_bits_from_width, load_gemma4_qat,
                                              packed_width, quantize, write_gemma4_qat_folder)
from nanovllm_b200.models.registry import init_random_weights
from nanovllm_b200.ops import reference_cpu as ref
from nanovllm_b200.sampling_params import SamplingParams


def gemma4_tiny(**kw):
    text = {"vocab_size": 300, "hidden_size": 128, "intermediate_size": 128, "num_hidden_layers": 6,
            "num_attention_heads": 4, "num_key_value_heads": 1, "head_dim": 64, "global_head_dim": 128,
            "hidden_size_per_layer_input": 32, "num_kv_shared_layers": 2,
            "layer_types": ["sliding_attention", "sliding_attention", "full_attention", "sliding_attention",
                            "sliding_attention", "full_attention"],
            "sliding_window": 16, "final_logit_softcapping": 30.0, "hidden_activation": "gelu_pytorch_tanh",
            "rope_parameters": {"sliding_attention": {"rope_theta": 10000.0},
                                "full_attention": {"rope_theta": 1000000.0, "partial_rotary_factor": 0.25}},
            "rms_norm_eps": 1e-6, "max_position_embeddings": 2048, "use_double_wide_mlp": True,
            "tie_word_embeddings": True}
    text.update(kw)
    return HfConfig.parse({"model_type": "gemma4", "architectures": ["Gemma4ForConditionalGeneration"],
                           "text_config": text})


# ------------------------------------------------------------------------------------------------- packing
def test_qat_pack_layout_and_bits():
    assert packed_width(10, 2) == 3 and packed_width(10, 4) == 5 and packed_width(10, 8) == 10
    assert infer_bits_from_width(5, 10) == 4 and infer_bits_from_width(3, 10) == 2
    # 4-bit: low nibble first, value - 8; 2-bit: crumbs low to high, value - 2
    w4 = QatWeight("a", torch.tensor([[0x1F, 0x80]], dtype=torch.uint8), torch.tensor([[2.0]]), 1, 4, 4, 1)
    assert w4.dequantize(torch.float32).tolist() == [[14.0, -14.0, -16.0, 0.0]]
    w2 = QatWeight("b", torch.tensor([[0b11100100]], dtype=torch.uint8), torch.tensor([[1.0, 10.0]]), 1, 4, 2, 2)
    assert w2.dequantize(torch.float32).tolist() == [[-2.0, -1.0, 0.0, 10.0]]
    w8 = QatWeight("c", torch.tensor([[-3, 5]], dtype=torch.int8), torch.tensor([[0.5]]), 1, 2, 8, 1)
    assert w8.dequantize(torch.float32).tolist() == [[-1.5, 2.5]]
    hf = gemma4_tiny()
    assert infer_bits("model.embed_tokens.weight", "U8", hf) == 2
    assert infer_bits("model.embed_tokens_per_layer.weight", "U8", hf) == 4
    assert infer_bits("model.layers.5.mlp.down_proj.weight", "U8", hf) == 2  # KV-shared layer MLP
    assert infer_bits("model.layers.1.mlp.down_proj.weight", "U8", hf) == 4
    assert infer_bits("model.layers.1.mlp.down_proj.weight", "I8", hf) == 8
    g = torch.Generator().manual_seed(0)
    dense = torch.randn(16, 64, generator=g)
    for bits in (2, 4, 8):
        q = quantize("x", dense, bits, 4)
        err = (q.dequantize(torch.float32) - dense).abs().max() / dense.abs().max()
        assert err < {2: 1.0, 4: 0.2, 8: 0.01}[bits]
        assert torch.equal(q.dequantize_row(3), q.dequantize(torch.float32)[3])


def test_srq_matches_definition():
    x = torch.tensor([[0.26, -0.74, 100.0, -100.0, 0.25]], dtype=torch.bfloat16)
    y = ref.srq(x, 0.5)
    # round half up of v / s, clamped to [-128, 127]
    assert y.float().tolist() == [[0.5, -0.5, 63.5, -64.0, 0.5]]


# ------------------------------------------------------------------------------------------------- graph
def _rms(x, w, eps):
    x = x.float()
    y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return y * w.float() if w is not None else y


def _gelu(x):
    return 0.5 * x * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x ** 3)))


def _rope(x, pos, hd, base, partial=1.0):
    half = hd // 2
    inv = 1.0 / (base ** (torch.arange(half, dtype=torch.float64) * 2.0 / hd))
    if partial < 1.0:
        inv[int(partial * hd / 2):] = 0.0
    ang = pos[:, None].double() * inv[None, :]
    c, s = torch.cos(ang).float()[:, None, :], torch.sin(ang).float()[:, None, :]
    a, b = x[..., :half], x[..., half:]
    return torch.cat([a * c - b * s, b * c + a * s], -1)


def reference_logits(hf: HfConfig, w, ids):
    """Plain fp32 Gemma4 forward over one sequence (no cache) -> logits [T, V] with the final softcap."""
    g4, H, eps = hf.gemma4, hf.hidden_size, hf.rms_norm_eps
    P, L, T = g4.hidden_size_per_layer_input, hf.num_hidden_layers, len(ids)
    f = {k: v.float() for k, v in w.items()}
    ids_t = torch.tensor(ids)
    pos = torch.arange(T)
    h = f["model.embed_tokens.weight"][ids_t] * math.sqrt(H)
    tok = f["model.embed_tokens_per_layer.weight"][ids_t] * math.sqrt(P)
    proj = (h @ f["model.per_layer_model_projection.weight"].t()) / math.sqrt(H)
    proj = _rms(proj.reshape(T, L, P), f["model.per_layer_projection_norm.weight"], eps).reshape(T, L * P)
    ple = (proj + tok) / math.sqrt(2.0)
    nq, nkv = hf.num_attention_heads, hf.num_key_value_heads
    kv = {}
    for i in range(L):
        p = f"model.layers.{i}."
        hd = hf.layer_head_dim(i)
        sliding = hf.is_sliding_layer(i)
        x = _rms(h, f[p + "input_layernorm.weight"], eps)
        q = (x @ f[p + "self_attn.q_proj.weight"].t()).reshape(T, nq, hd)
        q = _rms(q, f[p + "self_attn.q_norm.weight"], eps)
        base = hf.rope_local_base_freq if sliding else hf.rope_theta
        part = 1.0 if sliding else g4.full_partial_rotary_factor
        q = _rope(q, pos, hd, base, part)
        if hf.is_kv_shared_layer(i):
            k, v = kv[hf.kv_producer_layer(i)]
        else:
            k = _rms((x @ f[p + "self_attn.k_proj.weight"].t()).reshape(T, nkv, hd), f[p + "self_attn.k_norm.weight"], eps)
            k = _rope(k, pos, hd, base, part)
            v = _rms((x @ f[p + "self_attn.v_proj.weight"].t()).reshape(T, nkv, hd), None, eps)
            kv[i] = (k, v)
        G = nq // nkv
        kk, vv = k.repeat_interleave(G, 1), v.repeat_interleave(G, 1)
        s = torch.einsum("qhd,khd->hqk", q, kk)  # scale 1.0
        mask = torch.ones(T, T, dtype=torch.bool).tril()
        if sliding:
            mask &= (pos[:, None] - pos[None, :]) < hf.sliding_window
        s = s.masked_fill(~mask, float("-inf"))
        o = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), vv).reshape(T, nq * hd)
        a = o @ f[p + "self_attn.o_proj.weight"].t()
        h = h + _rms(a, f[p + "post_attention_layernorm.weight"], eps)
        x = _rms(h, f[p + "pre_feedforward_layernorm.weight"], eps)
        m = (_gelu(x @ f[p + "mlp.gate_proj.weight"].t()) * (x @ f[p + "mlp.up_proj.weight"].t())) @ \
            f[p + "mlp.down_proj.weight"].t()
        h = h + _rms(m, f[p + "post_feedforward_layernorm.weight"], eps)
        gte = _gelu(h @ f[p + "per_layer_input_gate.weight"].t()) * ple[:, i * P:(i + 1) * P]
        h = h + _rms(gte @ f[p + "per_layer_projection.weight"].t(), f[p + "post_per_layer_input_norm.weight"], eps)
        h = h * f[p + "layer_scalar"].reshape(-1)[0]
    h = _rms(h, f["model.norm.weight"], eps)
    logits = h @ f["model.embed_tokens.weight"].t()
    c = g4.final_logit_softcapping
    return torch.tanh(logits / c) * c


def _cfg(**kw):
    c = dict(max_num_seqs=4, max_model_len=512, num_kvcache_blocks=8, max_num_batched_tokens=512,
             stop_on_degenerate=False)
    c.update(kw)
    return EngineConfig(**c)


def _engine_logits(llm, ids):
    from test_models_cpu import _prefill_logits
    return _prefill_logits(llm, ids)


def test_gemma4_graph_matches_fp32_restatement_cpu():
    hf = gemma4_tiny()
    w = init_random_weights(hf, 5)
    ids = list(range(3, 43))
    want = reference_logits(hf, w, ids)[-1]
    llm = LLM((hf, w), _cfg(), device="cpu")
    got = _engine_logits(llm, ids)
    c = hf.gemma4.final_logit_softcapping
    got = torch.tanh(got.float() / c) * c
    assert torch.nn.functional.cosine_similarity(got, want, dim=0) > 0.995
    assert (got - want).abs().max() < 0.25


def test_gemma4_decode_with_shared_kv_matches_prefill_cpu():
    hf = gemma4_tiny()
    w = init_random_weights(hf, 6)
    prompt = list(range(10, 50))
    sp = SamplingParams(max_tokens=6, ignore_eos=True).deterministic()
    out = LLM((hf, w), _cfg(), device="cpu").generate_token_ids([prompt], sp)[0].token_ids
    # teacher-forced: every generated token is the argmax of the full-sequence restatement
    seq = list(prompt)
    for t in out:
        assert int(reference_logits(hf, w, seq)[-1].argmax()) == t
        seq.append(t)


def test_gemma4_qat_folder_round_trip(tmp_path):
    from nanovllm_b200.api.factory import LlmModelFactory
    from nanovllm_b200.models.writers import byte_level_tokenizer_json
    hf = gemma4_tiny()
    dense = init_random_weights(hf, 7)
    srq = {"model.layers.1.mlp.down_proj.weight": (0.02, 0.05)}
    d = write_gemma4_qat_folder(str(tmp_path / "g4"), hf, dense, scale_cols=4, srq=srq,
                                tokenizer_json=byte_level_tokenizer_json(300))
    loaded = load_gemma4_qat(d, hf)
    q = loaded["model.layers.2.self_attn.q_proj.weight"]
    assert isinstance(q, QatWeight) and q.bits == 4 and q.scale_cols == 4
    assert loaded["model.embed_tokens.weight"].bits == 2
    assert loaded["model.layers.4.mlp.gate_proj.weight"].bits == 2
    dq = loaded["model.layers.1.mlp.down_proj.weight"]
    assert (dq.in_scale, dq.out_scale) == pytest.approx((0.02, 0.05))
    assert torch.equal(q.dequantize(torch.float32),
                       quantize("x", dense["model.layers.2.self_attn.q_proj.weight"], 4, 4).dequantize(torch.float32))
    model = LlmModelFactory.make(d, device="cpu")
    assert model.architecture_name in ("gemma4", "Gemma4ForCausalLM") or "gemma4" in model.architecture_name.lower()
    llm = LLM(model, _cfg(), device="cpu")
    toks = llm.generate_token_ids([list(range(5, 25))], SamplingParams(max_tokens=4, ignore_eos=True).deterministic())
    assert len(toks[0].token_ids) == 4


def test_gemma4_qat_projections_run_packed(tmp_path, monkeypatch):
    """QAT int4 / int2 / int8 projections become GGUF Q4_0 / Q8_0 blocks for the dequant-fused GEMM (no bf16
    expansion): same logits as the expanded path within the fp16 rounding of the block scales."""
    from nanovllm_b200.api.factory import LlmModelFactory
    from nanovllm_b200.models.gemma4 import QatLinearGroup
    from nanovllm_b200.models.writers import byte_level_tokenizer_json
    hf = gemma4_tiny(hidden_size=256, intermediate_size=256)
    dense = init_random_weights(hf, 8)
    d = write_gemma4_qat_folder(str(tmp_path / "g4p"), hf, dense, scale_cols=4,
                                tokenizer_json=byte_level_tokenizer_json(300))
    ids = list(range(5, 37))
    monkeypatch.setenv("NVB_GGUF_PACKED", "0")
    want = _engine_logits(LLM(LlmModelFactory.make(d, device="cpu"), _cfg(), device="cpu"), ids).float()
    monkeypatch.setenv("NVB_GGUF_PACKED", "force")
    llm = LLM(LlmModelFactory.make(d, device="cpu"), _cfg(), device="cpu")
    groups = [g for L in llm.model.layers for g in (L.qkv, L.o_proj, L.gate_up, L.down)]
    packed = [g for g in groups if not isinstance(getattr(g, "w", None), torch.Tensor) and hasattr(g, "w")]
    assert packed, "no projection took the packed path"
    assert all(isinstance(g, QatLinearGroup) for g in groups)
    got = _engine_logits(llm, ids).float()
    assert torch.nn.functional.cosine_similarity(got, want, dim=0) > 0.999
    assert (got - want).abs().max() < 0.05


def test_allow_unpack_parameters_expands_packed_projections(tmp_path, monkeypatch):
    """``allow_unpack_parameters`` (LLM.java:1819-1835): an engine over a packed model expands its projections to
    bf16 (the shared model keeps its packed tensors) and gives the packed engine's logits within bf16 rounding."""
    from nanovllm_b200.api.factory import LlmModelFactory
    from nanovllm_b200.models.writers import byte_level_tokenizer_json
    hf = gemma4_tiny(hidden_size=256, intermediate_size=256)
    d = write_gemma4_qat_folder(str(tmp_path / "g4u"), hf, init_random_weights(hf, 8), scale_cols=4,
                                tokenizer_json=byte_level_tokenizer_json(300))
    ids = list(range(5, 37))
    monkeypatch.setenv("NVB_GGUF_PACKED", "force")
    model = LlmModelFactory.make(d, device="cpu")
    packed = LLM(model, _cfg(), device="cpu")
    groups = [g for L in packed.model.layers for g in (L.qkv, L.o_proj, L.gate_up, L.down)]
    assert any(not isinstance(w, torch.Tensor) for g in groups for w in (getattr(g, "ws", None) or [g.w]))
    want = _engine_logits(packed, ids).float()
    llm = LLM.builder(model).device("cpu").max_model_len(_cfg().max_model_len).allow_unpack_parameters().build()
    groups = [g for L in llm.model.layers for g in (L.qkv, L.o_proj, L.gate_up, L.down)]
    assert all(isinstance(w, torch.Tensor) for g in groups for w in (getattr(g, "ws", None) or [g.w]))
    got = _engine_logits(llm, ids).float()
    assert torch.nn.functional.cosine_similarity(got, want, dim=0) > 0.999


@pytest.mark.gpu
def test_gemma4_qat_packed_gemm_on_gpu(tmp_path, monkeypatch):
    """On the GPU the converted QAT projections run the dequant-fused tcgen05 GEMM (decode) and the dequant +
    dense GEMM (prefill); tokens and logits agree with the bf16-expanded engine."""
    from nanovllm_b200 import ops
    from nanovllm_b200.api.factory import LlmModelFactory
    from nanovllm_b200.models.writers import byte_level_tokenizer_json
    hf = gemma4_tiny(hidden_size=256, intermediate_size=256)
    d = write_gemma4_qat_folder(str(tmp_path / "g4g"), hf, init_random_weights(hf, 8), scale_cols=4,
                                tokenizer_json=byte_level_tokenizer_json(300))
    ids = list(range(5, 37))
    dev = torch.device("cuda", 0)
    monkeypatch.setenv("NVB_GGUF_PACKED", "0")
    dense = LLM(LlmModelFactory.make(d, device="cpu"), _cfg(), device=dev)
    want = _engine_logits(dense, ids).float().cpu()
    dense.close()
    monkeypatch.setenv("NVB_GGUF_PACKED", "1")
    llm = LLM(LlmModelFactory.make(d, device="cpu"), _cfg(), device=dev)
    got = _engine_logits(llm, ids).float().cpu()
    torch.cuda.synchronize()
    ops.check_device_errors()
    assert torch.nn.functional.cosine_similarity(got, want, dim=0) > 0.999
    out = llm.generate_token_ids([ids], SamplingParams(max_tokens=4, ignore_eos=True).deterministic())
    assert len(out[0].token_ids) == 4
