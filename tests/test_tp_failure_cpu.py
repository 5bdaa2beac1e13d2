"""Failure propagation across tensor-parallel ranks, on gloo CPU ranks (no GPU is involved).

Three ranks run the sharded tiny Qwen3 engine.  At its third step rank 1 either raises (a host-side failure,
as when a device wait gave up and the runner raised DeviceWaitTimeout) or exits without a word.  Every rank
must end promptly: the failing rank with its own error, the others with ``TensorParallelAbort`` naming rank 1
(learned through the rendezvous store) or, when rank 1 vanished silently, with the collective's error."""
import datetime
import os
import socket
import time

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=6))
    from nanovllm_b200.config import EngineConfig, HfConfig
    from nanovllm_b200.llm import LLM
    from nanovllm_b200.models.registry import init_random_weights
    from nanovllm_b200.parallel import state as ps
    from nanovllm_b200.sampling_params import SamplingParams
    ps.init_tp("gloo")
    hf = HfConfig(vocab_size=300, hidden_size=96, intermediate_size=192, num_hidden_layers=1, num_attention_heads=6,
                  num_key_value_heads=3, head_dim=32, max_position_embeddings=512, model_type="qwen3",
                  tie_word_embeddings=False)
    llm = LLM((hf, init_random_weights(hf, 0)), EngineConfig(max_num_seqs=2, max_model_len=256, num_kvcache_blocks=4,
                                                             max_num_batched_tokens=256), device="cpu")
    real_run = llm.runner.run
    calls = [0]

    def flaky_run(seqs, is_prefill):
        calls[0] += 1
        if rank == 1 and calls[0] == 3:
            if mode == "exit":
                os._exit(3)  # vanish between steps, nothing in flight
            raise RuntimeError("injected failure on rank 1")
        return real_run(seqs, is_prefill)

    llm.runner.run = flaky_run
    t0 = time.perf_counter()
    try:
        llm.generate_token_ids([[1, 2, 3, 4]], SamplingParams(max_tokens=20, ignore_eos=True).deterministic())
        q.put((rank, "finished", "", time.perf_counter() - t0))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, type(e).__name__, str(e), time.perf_counter() - t0))
    q.close()
    q.join_thread()  # flush the queue's feeder thread before the hard exit
    os._exit(0)  # skip the collective teardown: a peer is gone


@pytest.mark.parametrize("mode", ["raise", "exit"])
def test_a_failing_rank_stops_every_rank(mode):
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    expect = world if mode == "raise" else world - 1
    got = {}
    for _ in range(expect):
        r, kind, msg, dt = q.get(timeout=120)
        got[r] = (kind, msg, dt)
    for p in procs:
        p.join(timeout=30)
    for r in got:
        assert got[r][0] != "finished", f"rank {r} kept generating after rank 1 failed"
        assert got[r][2] < 60, f"rank {r} took {got[r][2]:.1f}s to stop"
    if mode == "raise":
        assert got[1][0] == "RuntimeError" and "injected" in got[1][1]
        for r in (0, 2):
            assert got[r][0] == "TensorParallelAbort", got[r]
            assert "rank 1" in got[r][1]
    else:
        assert 1 not in got
        assert procs[1].exitcode == 3
