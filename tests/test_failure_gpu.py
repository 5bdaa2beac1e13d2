"""Failure detection on one GPU without faulting it: a bounded peer-flag wait that nothing ever satisfies gives up
after its limit, the kernel returns, the host sees the error code, and the context stays usable.

The fused all-reduce kernel is launched as rank 0 of a two-rank group whose "peer" buffers are private local
allocations that no kernel signals (no second process, no peer mapping), with a 5 ms wait limit."""
import time

import pytest
import torch

from nanovllm_b200 import ops
from nanovllm_b200.exceptions import DeviceWaitTimeout

pytestmark = pytest.mark.gpu


def test_peer_flag_wait_times_out_and_reports_on_the_host():
    C = ops._cuda_ext()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    T, H = 4, 1024
    sig = [torch.zeros(2 * 1024 * 8, dtype=torch.int32, device=dev) for _ in range(2)]
    inp = [torch.randn(T, H, device=dev).bfloat16() for _ in range(2)]
    out = [torch.zeros(T, H, device=dev, dtype=torch.bfloat16) for _ in range(2)]
    counters = torch.zeros(1024, dtype=torch.int32, device=dev)
    ops.error_word(dev).zero_()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    C.tp_allreduce_norm([t.data_ptr() for t in inp], [0, 0], [t.data_ptr() for t in out],
                        [t.data_ptr() for t in sig], 0, T, H, None, 1e-6, 3, counters, ops.error_word(dev), 148, 1,
                        wait_ns=5_000_000)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert elapsed < 1.0, f"the bounded wait should give up after ~5 ms, took {elapsed:.3f} s"
    assert int(ops.error_word(dev).item()) == 2  # kErrFlagTimeout
    with pytest.raises(DeviceWaitTimeout):
        ops.check_device_errors(dev)
    assert int(ops.error_word(dev).item()) == 0, "check_device_errors clears the word"
    # the context is still usable: a normal kernel runs and matches the CPU oracle
    x = torch.randn(8, H, generator=torch.Generator().manual_seed(0)).bfloat16()
    w = torch.ones(H, dtype=torch.bfloat16)
    y, _ = ops.rms_norm(x.to(dev), w.to(dev), 1e-6)
    want, _ = ops.ref.rms_norm(x, w, 1e-6, 0)
    assert (y.float().cpu() - want.float()).abs().max().item() < 2e-2


def test_engine_step_raises_when_a_kernel_reports_an_error():
    """The model runner copies the error word next to the sampled tokens every step and raises."""
    from nanovllm_b200.config import EngineConfig, HfConfig
    from nanovllm_b200.llm import LLM
    from nanovllm_b200.models.registry import init_random_weights
    from nanovllm_b200.sampling_params import SamplingParams
    dev = torch.device("cuda", 0)
    hf = HfConfig(vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=1,
                  num_attention_heads=4, num_key_value_heads=2, head_dim=64, max_position_embeddings=1024,
                  model_type="qwen3", tie_word_embeddings=True)
    llm = LLM((hf, init_random_weights(hf, 0)), EngineConfig(max_num_seqs=2, max_model_len=512, num_kvcache_blocks=8,
                                                              max_num_batched_tokens=512), device=dev)
    llm.add_request([1, 2, 3], SamplingParams(max_tokens=4, ignore_eos=True).deterministic())
    llm.step()
    ops.error_word(dev).fill_(2)  # as if a bounded wait had given up during the next step
    with pytest.raises(DeviceWaitTimeout):
        llm.step()
    assert int(ops.error_word(dev).item()) == 0
    llm.close()
