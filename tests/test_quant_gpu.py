"""Dequant-fused GEMM for packed GGUF weights (csrc/qgemm.cu) against fp32 torch references."""
import numpy as np
import pytest
import torch

from nanovllm_b200.loaders import dequant as DQ
from nanovllm_b200.loaders.gguf import pack_random_blocks
from nanovllm_b200.ops.quant import FUSED_TYPES, GgufPacked

pytestmark = pytest.mark.gpu
TYPES = sorted(FUSED_TYPES)


def _packed(t, N, K, seed=0):
    raw = torch.from_numpy(np.frombuffer(pack_random_blocks(t, (N, K), seed), dtype=np.uint8).copy())
    return GgufPacked(raw.cuda(), t, N, K)


def _check_errors():
    from nanovllm_b200 import ops
    ops.check_device_errors(torch.device("cuda", torch.cuda.current_device()))


@pytest.mark.parametrize("t", TYPES)
def test_device_dequant_matches_torch_decoder(t):
    N, K = 300, 768
    w = _packed(t, N, K, seed=1)
    want = DQ.dequantize(w.raw.reshape(-1).cpu(), t, N * K).reshape(N, K)
    got = w.dense_cuda().float().cpu()
    ref = want.bfloat16().float()
    # same fp32 formula, one rounding to bf16 (a fused multiply-add may move a tie by one ulp)
    assert ((got - ref).abs() <= ref.abs() * 2 ** -7 + 1e-9).all(), (got - ref).abs().max()
    _check_errors()


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("M", [1, 16, 100, 128])
def test_fused_decode_gemm_matches_fp32(t, M):
    N, K = 300, 1024
    w = _packed(t, N, K, seed=2)
    dense = DQ.dequantize(w.raw.reshape(-1).cpu(), t, N * K).reshape(N, K).bfloat16().float()
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(M)).bfloat16()
    want = x.float() @ dense.t()
    y = w.linear(x.cuda()).float().cpu()
    scale = want.abs().max().item()
    assert torch.allclose(y, want, atol=2e-2 * scale, rtol=2e-2), (t, M, (y - want).abs().max().item(), scale)
    _check_errors()


@pytest.mark.parametrize("M", [8, 64, 200, 256])
def test_fused_decode_gemm_shapes_and_split_partials(M):
    from nanovllm_b200 import ops
    t, N, K = 12, 1024, 4096
    w = _packed(t, N, K, seed=3)
    dense = w.dense_cuda()
    x = torch.randn(M, K, device="cuda").bfloat16()
    want = x.float() @ dense.float().t()
    y = w.linear(x)
    scale = want.abs().max().item()
    assert torch.allclose(y.float(), want, atol=2e-2 * scale, rtol=2e-2)
    p = w.linear(x, partial_ok=True)
    s = ops.materialize(p).float() if isinstance(p, ops.SplitK) else p.float()
    assert torch.allclose(s, want, atol=2e-2 * scale, rtol=2e-2)
    # prefill-sized M dequantizes and runs the tensor-core GEMM
    xl = torch.randn(300, K, device="cuda").bfloat16()
    assert torch.allclose(w.linear(xl).float(), xl.float() @ dense.float().t(), atol=3e-2 * scale, rtol=3e-2)
    _check_errors()


def test_fused_gemm_in_cuda_graph():
    t, N, K = 40, 512, 2048
    w = _packed(t, N, K, seed=4)
    x = torch.randn(16, K, device="cuda").bfloat16()
    w.linear(x)  # repack before capture
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            y = w.linear(x)
    torch.cuda.current_stream().wait_stream(s)
    x.copy_(torch.randn(16, K, device="cuda").bfloat16())
    g.replay()
    torch.cuda.synchronize()
    want = x.float() @ w.dense_cuda().float().t()
    assert torch.allclose(y.float(), want, atol=2e-2 * want.abs().max().item(), rtol=2e-2)
    _check_errors()


def test_gguf_model_packed_on_gpu_matches_dequantized(tmp_path, monkeypatch):
    from nanovllm_b200.api.factory import LlmModelFactory
    from nanovllm_b200.config import EngineConfig, HfConfig
    from nanovllm_b200.engine.sequence import Sequence
    from nanovllm_b200.llm import LLM
    from nanovllm_b200.models.registry import init_random_weights
    from nanovllm_b200.models.writers import write_gguf_model
    from nanovllm_b200.sampling_params import SamplingParams

    hf = HfConfig(vocab_size=512, hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=8,
                  num_key_value_heads=2, head_dim=64, max_position_embeddings=2048, model_type="qwen3",
                  architectures=["Qwen3ForCausalLM"], tie_word_embeddings=False)
    p = write_gguf_model(str(tmp_path / "q.gguf"), hf, init_random_weights(hf, 0), "Q4_K", big_type="Q6_K",
                         random_packed=True)

    def run(mode):
        monkeypatch.setenv("NVB_GGUF_PACKED", mode)
        m = LlmModelFactory.make(p, device="cuda")
        llm = LLM(m, EngineConfig(max_num_seqs=4, max_model_len=512, num_kvcache_blocks=8,
                                  max_num_batched_tokens=256, stop_on_degenerate=False), device=torch.device("cuda", 0))
        s = Sequence(list(range(3, 60)), SamplingParams(max_tokens=1), 256)
        bm = llm.scheduler.block_manager
        bm.allocate(s, 0)
        s.num_scheduled_tokens = len(s.token_ids)
        logits = llm.runner.forward_logits([s], True)[0].float().cpu()
        bm.deallocate(s)
        toks = llm.generate_token_ids([list(range(5, 40))], SamplingParams(max_tokens=6, ignore_eos=True).deterministic())
        return logits, toks[0].token_ids, {type(v).__name__ for v in m.weights.values()}

    a, ta, ka = run("1")
    b, tb, kb = run("0")
    assert "GgufPacked" in ka and "GgufPacked" not in kb
    assert torch.allclose(a, b, atol=3e-2, rtol=3e-2), (a - b).abs().max()
    assert len(ta) == 6 and len(tb) == 6
    _check_errors()
