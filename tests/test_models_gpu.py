"""Gemma3 / LFM2 / BERT on the sm_100a kernels against the CPU oracle path, and the short-conv kernel itself."""
import pytest
import torch

from nanovllm_b200 import ops
from nanovllm_b200.config import EngineConfig
from nanovllm_b200.llm import LLM
from nanovllm_b200.models.registry import init_random_weights
from nanovllm_b200.ops import reference_cpu as ref
from nanovllm_b200.sampling_params import SamplingParams

from test_gemma4 import gemma4_tiny
from test_models_cpu import _prefill_logits, bert_tiny, gemma3_tiny, lfm2_tiny

pytestmark = pytest.mark.gpu


def _cfg(**kw):
    c = dict(max_num_seqs=4, max_model_len=1024, num_kvcache_blocks=12, max_num_batched_tokens=512,
             stop_on_degenerate=False)
    c.update(kw)
    return EngineConfig(**c)


def test_shortconv_kernel_matches_oracle():
    g = torch.Generator().manual_seed(0)
    H, L = 256, 3
    T = 37
    proj = torch.randn(T, 3 * H, generator=g).bfloat16()
    w = torch.randn(H, L, generator=g)
    cu = torch.tensor([0, 20, 21, 37], dtype=torch.int32)
    rows = torch.tensor([3, 1, 2])
    fresh = torch.tensor([True, False, True])
    state = torch.randn(5, 2 * (L - 1) * H, generator=g)
    st_cpu = state.clone()
    want = ref.shortconv(proj, w, cu, rows, fresh, st_cpu, (L - 1) * H)
    st_gpu = state.cuda()
    got = ops.shortconv(proj.cuda(), w.cuda(), cu.cuda(), rows.cuda(), fresh.cuda(), st_gpu, (L - 1) * H)
    assert torch.allclose(got.float().cpu(), want.float(), atol=2e-2, rtol=2e-2)
    assert torch.allclose(st_gpu.cpu(), st_cpu, atol=1e-5)


@pytest.mark.parametrize("make", [gemma3_tiny, lfm2_tiny, gemma4_tiny])
def test_causal_family_gpu_matches_cpu(make):
    hf = make()
    w = init_random_weights(hf, 7)
    ids = list(range(3, 120))
    a = _prefill_logits(LLM((hf, w), _cfg(), device="cpu"), ids)
    b = _prefill_logits(LLM((hf, w), _cfg(enforce_eager=True), device="cuda"), ids).cpu()
    assert torch.nn.functional.cosine_similarity(a, b, dim=0) > 0.999
    assert (a - b).abs().max() < 0.1


def test_lfm2_gpu_graph_decode_and_chunked_prefill():
    hf = lfm2_tiny()
    w = init_random_weights(hf, 3)
    prompt = list(range(5, 305))
    sp = SamplingParams(max_tokens=8, ignore_eos=True).deterministic()
    a = LLM((hf, w), _cfg(max_num_batched_tokens=128), device="cuda").generate_token_ids([prompt, [7, 8]], sp)
    b = LLM((hf, w), _cfg(max_num_batched_tokens=1024, enforce_eager=True), device="cuda").generate_token_ids(
        [prompt, [7, 8]], sp)
    assert [o.token_ids for o in a] == [o.token_ids for o in b]
    ops.check_device_errors()


def test_bert_gpu_matches_cpu():
    from nanovllm_b200.models.bert import BertEncoder
    hf = bert_tiny()
    w = init_random_weights(hf, 1)
    ids = [[2] + list(range(10, 10 + n)) + [3] for n in (5, 40, 100)]
    a = BertEncoder(hf, w, torch.device("cpu")).embed_ids(ids)
    b = BertEncoder(hf, w, torch.device("cuda")).embed_ids(ids)
    assert torch.nn.functional.cosine_similarity(a, b, dim=1).min() > 0.999


def test_gemma4_elementwise_kernels_match_oracle():
    g = torch.Generator().manual_seed(3)
    T, H, L, P = 37, 256, 5, 64
    x = torch.randn(T, H, generator=g).bfloat16()
    res = torch.randn(T, H, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(H, generator=g)).bfloat16()
    want = ref.rms_norm_post_add(x, res.clone(), w, 1e-6, 0, 0.75)
    got = ops.rms_norm_post_add_(x.cuda(), res.cuda(), w.cuda(), 1e-6, 0, 0.75)
    assert torch.allclose(got.float().cpu(), want.float(), atol=3e-2, rtol=2e-2)
    proj = torch.randn(T, L * P, generator=g).bfloat16()
    tok = torch.randn(T, L * P, generator=g).bfloat16()
    pw = (1 + 0.1 * torch.randn(P, generator=g)).bfloat16()
    want = ref.ple_combine(proj, tok, pw, 1e-6, 0.0625, 0.7071)
    got = ops.ple_combine(proj.cuda(), tok.cuda(), pw.cuda(), 1e-6, 0.0625, 0.7071)
    assert torch.allclose(got.float().cpu(), want.float(), atol=3e-2, rtol=2e-2)
    wide = torch.randn(T, 3 * P, generator=g).bfloat16()
    gate = torch.randn(T, P, generator=g).bfloat16()
    want = ref.gate_act_mul(gate, wide[:, P:2 * P])
    got = ops.gate_act_mul(gate.cuda(), wide.cuda()[:, P:2 * P])
    assert torch.allclose(got.float().cpu(), want.float(), atol=2e-2, rtol=2e-2)
    y = (4 * torch.randn(T, 2 * P, generator=g)).bfloat16()
    want = y.clone()
    want[:, :P] = ref.srq(y[:, :P], 0.05)
    yc = y.cuda()
    ops.srq_(yc[:, :P], 0.05)
    assert torch.equal(yc.cpu(), want)
