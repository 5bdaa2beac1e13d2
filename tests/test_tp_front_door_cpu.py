"""Front-door tensor parallelism (rank 0 takes the requests and broadcasts step plans, the other ranks follow):
plan encoding round trip against the scheduler's own sequences (chunked prefill, prefix reuse, preemption, finish),
divergence detection, and gloo ranks that reproduce the single-process tokens, end on rank 0's close and learn of
a rank-0 failure while idle."""
import os
import random
import socket
import time

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from nanovllm_b200.config import EngineConfig
from nanovllm_b200.engine.plan import PlanReceiver, PlanSender
from nanovllm_b200.engine.scheduler import Scheduler
from nanovllm_b200.engine.sequence import Sequence
from nanovllm_b200.exceptions import TensorParallelAbort
from nanovllm_b200.sampling_params import SamplingParams


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _mirror_equal(m, s):
    assert m.seq_id == s.seq_id
    assert m.token_ids == s.token_ids and m.num_tokens == s.num_tokens and m.last_token == s.last_token
    assert m.block_table == s.block_table and m.bt_gen == s.bt_gen
    assert (m.num_cached_tokens, m.num_scheduled_tokens) == (s.num_cached_tokens, s.num_scheduled_tokens)
    assert (m.temperature, m.top_k, m.top_p, m.seed) == (s.temperature, s.top_k, s.top_p, s.seed)


def test_plan_round_trip_follows_the_scheduler():
    """Every step's mirrors equal rank 0's sequences, through chunked prefill, prefix-cache hits, preemption
    (pages released and reallocated: the whole table is resent) and finished sequences (dropped)."""
    rng = random.Random(7)
    cfg = EngineConfig(max_num_seqs=6, max_model_len=1024, max_num_batched_tokens=700, kvcache_block_size=256)
    released = []
    sch = Scheduler(cfg, num_blocks=7, on_release=lambda s: released.append(s))
    tx = PlanSender(None)
    rx_released = []
    rx = PlanReceiver(None, 256, release=lambda m: rx_released.append(m.seq_id))
    sch.on_release = lambda s: (released.append(s), tx.note_release(s))
    shared = [rng.randrange(500) for _ in range(256)]
    for i in range(6):
        sp = SamplingParams(max_tokens=rng.randint(150, 500), temperature=0.5 + i / 10, top_k=i, seed=i or None,
                            ignore_eos=True)
        sch.add(Sequence(shared + [rng.randrange(500) for _ in range(rng.randint(10, 400))], sp, 256))
    steps = 0
    while not sch.is_finished():
        seqs, pre = sch.schedule()
        kind, is_prefill, mirrors = rx.apply(tx.encode(seqs, pre))
        assert is_prefill == pre and len(mirrors) == len(seqs)
        for m, s in zip(mirrors, seqs):
            _mirror_equal(m, s)
        toks = [rng.randrange(500) for _ in seqs]
        rx.note_sampled(mirrors, toks)
        sch.postprocess(seqs, toks, pre)
        steps += 1
    rx.apply(tx.encode([], False))  # the last releases reach the receiver with the next plan
    assert sch.num_preemptions > 0, "the pool is meant to be small enough to preempt"
    assert not rx.mirrors and not rx.expect
    assert sorted(rx_released) == sorted(s.seq_id for s in released)
    assert steps > 10


def test_worker_reports_divergent_tokens():
    cfg = EngineConfig(max_num_seqs=2, max_model_len=512, max_num_batched_tokens=512)
    sch = Scheduler(cfg, num_blocks=4)
    tx, rx = PlanSender(None), PlanReceiver(None, 256)
    sch.add(Sequence(list(range(10)), SamplingParams(max_tokens=5, ignore_eos=True), 256))
    seqs, pre = sch.schedule()
    _, _, mirrors = rx.apply(tx.encode(seqs, pre))
    rx.note_sampled(mirrors, [41])   # this rank sampled 41 ...
    sch.postprocess(seqs, [42], pre)  # ... rank 0 sampled 42
    seqs, pre = sch.schedule()
    with pytest.raises(TensorParallelAbort, match="diverged"):
        rx.apply(tx.encode(seqs, pre))


def _tiny():
    from nanovllm_b200.config import HfConfig
    return HfConfig(vocab_size=302, hidden_size=128, intermediate_size=256, num_hidden_layers=2, num_attention_heads=4,
                    num_key_value_heads=2, head_dim=64, max_position_embeddings=1024, model_type="qwen3",
                    tie_word_embeddings=False)


PROMPTS = [[1, 2, 3, 4, 5], list(range(20, 90)), list(range(100, 340)), list(range(7, 250))]


def _cfg():
    # 5 pages for 4 sequences that each grow past one page: decode preempts, preempted sequences recompute
    return EngineConfig(max_num_seqs=4, max_model_len=512, num_kvcache_blocks=5, max_num_batched_tokens=300,
                        front_door="rank0")


def _sp():
    return SamplingParams(max_tokens=24, ignore_eos=True, temperature=0.8, top_k=20, seed=5)


def _front_door_run(rank, world, port, q, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    from nanovllm_b200.llm import LLM
    from nanovllm_b200.models.registry import init_random_weights
    from nanovllm_b200.parallel import state as ps
    ps.init_tp("gloo", timeout_s=60)
    hf = _tiny()
    cfg = _cfg()
    if mode == "spmd":
        cfg.front_door = "spmd"
    llm = LLM((hf, init_random_weights(hf, 0)), cfg, device="cpu")
    try:
        if mode == "spmd":  # every rank takes the same requests
            outs = llm.generate_token_ids(PROMPTS, _sp())
            q.put((rank, [o.token_ids for o in outs], llm.scheduler.num_preemptions))
        elif rank == 0:
            if mode == "fail":
                seq = llm.add_request(PROMPTS[1], _sp())
                llm.step()
                time.sleep(1.0)  # the worker is now waiting for the next plan
                ps.signal_abort("injected failure on rank 0")
                q.put((rank, "signalled", None))
                return
            if mode == "online":
                seqs = [llm.add_request(p, _sp()) for p in PROMPTS]
                n = 0
                while llm.has_unfinished():
                    llm.step()
                    n += 1
                    if n == 6:
                        llm.abort(seqs[2])  # released on rank 0; the worker drops its mirror with the next plan
                q.put((rank, [s.completion_token_ids for s in seqs], n))
            else:
                outs = llm.generate_token_ids(PROMPTS, _sp())
                q.put((rank, [o.token_ids for o in outs], llm.scheduler.num_preemptions))
            llm.close()
        else:
            t0 = time.perf_counter()
            try:
                steps = llm.serve_worker()
                q.put((rank, "done", steps))
            except TensorParallelAbort as e:
                q.put((rank, "aborted", (str(e), time.perf_counter() - t0)))
    finally:
        ps.destroy()


def _spawn(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_front_door_run, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        r, a, b = q.get(timeout=240)
        got[r] = (a, b)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return got


@pytest.mark.parametrize("world", [2, 4])
def test_front_door_ranks_reproduce_spmd_tokens(world):
    """Only rank 0 gets the requests; the workers follow its plans (with preemption and recompute) and every
    token equals the SPMD engine's at the same world size, where every rank schedules for itself.  (Against one
    process the sharded fp32 sums may flip a sampled token near a cut-off over this many steps; the TP=1
    comparison is test_tp_cpu.py's.)"""
    spmd = _spawn(world, "spmd")
    assert all(spmd[r] == spmd[0] for r in range(world))
    got = _spawn(world, "generate")
    toks, preemptions = got[0]
    assert preemptions > 0
    assert (toks, preemptions) == spmd[0]
    for r in range(1, world):
        assert got[r][0] == "done" and got[r][1] > 0


def test_front_door_online_api_with_abort():
    got = _spawn(2, "online")
    (toks, steps), (state, wsteps) = got[0], got[1]
    assert state == "done" and wsteps == steps
    assert len(toks[2]) < 24 and all(len(t) == 24 for i, t in enumerate(toks) if i != 2)


def test_idle_worker_learns_of_rank0_failure():
    """A worker waiting for the next plan leaves with TensorParallelAbort soon after rank 0 signals a failure
    (the control group's own timeout is days)."""
    got = _spawn(2, "fail")
    state, info = got[1]
    assert state == "aborted"
    reason, elapsed = info
    assert "injected failure" in reason and elapsed < 30


def _example_run(rank, world, port, q):
    import io
    import contextlib
    import sys as _sys
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      CUDA_VISIBLE_DEVICES="")
    examples = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "examples")
    _sys.path.insert(0, examples)
    import tp_serve
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        rc = tp_serve.main([])
    q.put((rank, rc, buf.getvalue()))


def test_tp_serve_example_runs_on_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_example_run, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        r, rc, out = q.get(timeout=240)
        got[r] = (rc, out)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got[0][0] == 0 and "3 answers" in got[0][1] and "Time taken" in got[0][1]
    assert got[1][0] == 0 and "followed" in got[1][1]
