"""Scheduler / block manager / sequence semantics (reference: engine/Scheduler.java, BlockManager.java,
Sequence.java and the corresponding cases of CoreUnitTest: blockManagerPrefixCache, detectsDegenerateTokenRepetition)."""
import pytest

from nanovllm_b200.config import EngineConfig
from nanovllm_b200.engine.block_manager import BlockManager, compute_hash
from nanovllm_b200.engine.scheduler import Scheduler
from nanovllm_b200.engine.sequence import Sequence, SequenceStatus
from nanovllm_b200.sampling_params import SamplingParams


def seq(n, start=0, bs=256, **kw):
    return Sequence(list(range(start, start + n)), SamplingParams(**kw) if kw else None, bs)


def test_block_math():
    s = seq(513)
    assert s.num_blocks == 3 and s.last_block_num_tokens == 1
    assert s.block(1) == list(range(256, 512))


def test_block_size_must_be_multiple_of_256():
    with pytest.raises(ValueError):
        EngineConfig(kvcache_block_size=128)


def test_prefix_cache_reuses_full_blocks_only():
    bm = BlockManager(16, 256)
    a = seq(600)
    assert bm.can_allocate(a) == 0
    bm.allocate(a, 0)
    a.num_scheduled_tokens = 600
    bm.hash_blocks(a)  # publishes blocks 0 and 1 (full), not the partial third
    b = seq(600)
    cached = bm.can_allocate(b)
    assert cached == 2
    bm.allocate(b, cached)
    assert b.block_table[:2] == a.block_table[:2]
    assert b.block_table[2] != a.block_table[2]
    assert b.num_cached_tokens == 512
    assert bm.blocks[a.block_table[0]].ref_count == 2
    bm.deallocate(a)
    assert bm.blocks[b.block_table[0]].ref_count == 1
    bm.deallocate(b)
    assert bm.num_free_blocks == 16


def test_last_block_never_cached():
    bm = BlockManager(8, 256)
    a = seq(512)
    bm.allocate(a, 0)
    a.num_scheduled_tokens = 512
    bm.hash_blocks(a)
    b = seq(512)
    assert bm.can_allocate(b) == 1  # the second (last) block is not a hit even though it is full


def test_hash_chain_depends_on_prefix():
    assert compute_hash([1, 2, 3]) != compute_hash([1, 2, 3], prefix=5)


def test_may_append_allocates_on_new_page():
    bm = BlockManager(4, 256)
    s = seq(256)
    bm.allocate(s, 0)
    assert len(s.block_table) == 1
    s.append_token(7)  # len 257 -> 257 % 256 == 1
    assert bm.can_append(s)
    bm.may_append(s)
    assert len(s.block_table) == 2


def test_scheduler_prefill_first_then_decode():
    cfg = EngineConfig(max_num_seqs=4, max_num_batched_tokens=1000, max_model_len=2048)
    sch = Scheduler(cfg, 32)
    a, b = seq(100), seq(50)
    sch.add(a)
    sch.add(b)
    batch, pre = sch.schedule()
    assert pre and batch == [a, b]
    sch.postprocess(batch, [1, 2], True)
    assert a.completion_token_ids == [1] and b.completion_token_ids == [2]
    batch, pre = sch.schedule()
    assert not pre and batch == [a, b]


def test_chunked_prefill_keeps_head_waiting():
    cfg = EngineConfig(max_num_seqs=4, max_num_batched_tokens=300, max_model_len=4096)
    sch = Scheduler(cfg, 32)
    a = seq(700)
    sch.add(a)
    batch, pre = sch.schedule()
    assert pre and a.num_scheduled_tokens == 300 and a.status == SequenceStatus.WAITING
    sch.postprocess(batch, [9], True)
    assert a.num_completion_tokens == 0 and a.num_cached_tokens == 300  # mid-prompt token discarded
    batch, _ = sch.schedule()
    assert a.num_scheduled_tokens == 300
    sch.postprocess(batch, [9], True)
    batch, _ = sch.schedule()
    assert a.num_scheduled_tokens == 100 and a.status == SequenceStatus.RUNNING
    sch.postprocess(batch, [5], True)
    assert a.completion_token_ids == [5]


def test_second_prompt_not_chunked_when_budget_short():
    cfg = EngineConfig(max_num_seqs=4, max_num_batched_tokens=300, max_model_len=4096)
    sch = Scheduler(cfg, 32)
    a, b = seq(200), seq(200, start=1000)
    sch.add(a)
    sch.add(b)
    batch, _ = sch.schedule()
    assert batch == [a]


def test_preemption_takes_running_tail():
    cfg = EngineConfig(max_num_seqs=4, max_num_batched_tokens=4096, max_model_len=4096)
    sch = Scheduler(cfg, 2)
    a, b = seq(256), seq(256, start=500)
    sch.add(a)
    sch.add(b)
    batch, pre = sch.schedule()
    assert pre and len(batch) == 2
    sch.postprocess(batch, [1, 1], True)  # both now need a second page for the next decode token
    batch, pre = sch.schedule()
    assert not pre
    assert batch == [a] and b.status == SequenceStatus.WAITING and sch.waiting[0] is b
    assert sch.num_preemptions == 1 and not b.block_table


def test_stop_rules():
    cfg = EngineConfig(max_num_seqs=4, max_num_batched_tokens=4096, max_model_len=4096, eos=3)
    sch = Scheduler(cfg, 8)
    a = seq(10, max_tokens=5)
    b = seq(10, start=50, max_tokens=5, ignore_eos=True)
    sch.add(a)
    sch.add(b)
    batch, pre = sch.schedule()
    fin = sch.postprocess(batch, [3, 3], True)
    assert fin == [a] and a.is_finished and not b.is_finished
    for _ in range(4):
        batch, _ = sch.schedule()
        fin = sch.postprocess(batch, [3], False)
    assert b.is_finished and b.num_completion_tokens == 5


def test_degenerate_repetition():
    s = seq(4)
    for _ in range(31):
        s.append_token(7)
    assert not s.has_degenerate_repetition()
    s.append_token(7)
    assert s.has_degenerate_repetition()
    p = seq(4)
    for i in range(32):
        p.append_token(100 + (i % 16))
    assert p.has_degenerate_repetition()  # two identical halves of period 16
    r = seq(4)
    for i in range(40):
        r.append_token(100 + (i % 20))
    assert not r.has_degenerate_repetition()  # period 20 is not probed and < 48 tokens for the n-gram rule
    for i in range(40, 60):
        r.append_token(100 + (i % 20))
    assert r.has_degenerate_repetition()  # a 12-gram now occurs 3 times in the window
    q = seq(4)
    for i in range(64):
        q.append_token(i)
    assert not q.has_degenerate_repetition()


def _degenerate_by_definition(ids, prompt):
    """The stop rule written out directly: recounts every window from scratch."""
    comp = len(ids) - prompt
    if comp < 32:
        return False
    streak = 0
    for t in reversed(ids[prompt:]):
        if t != ids[-1]:
            break
        streak += 1
    if streak >= 32:
        return True
    for period in range(16, min(64, comp // 2) + 1, 8):
        start = len(ids) - 2 * period
        if start >= prompt and ids[start:start + period] == ids[start + period:]:
            return True
    if comp < 48:
        return False
    window = min(comp, 128)
    counts = {}
    for s in range(len(ids) - window, len(ids) - 12 + 1):
        key = tuple(ids[s:s + 12])
        counts[key] = counts.get(key, 0) + 1
        if counts[key] >= 3:
            return True
    return False


@pytest.mark.parametrize("alphabet,check_every", [(2, 1), (3, 1), (5, 1), (3, 7), (40, 1), (1000, 3)])
def test_incremental_repetition_check_matches_definition(alphabet, check_every):
    """The sliding n-gram counts give the same answer as a full recount after every appended token, also when the
    check skips steps (the counts then catch up over several tokens at once) and past the 128-token window."""
    import random
    rng = random.Random(alphabet * 31 + check_every)
    for trial in range(6):
        s = seq(5 + trial)
        prompt = s.num_prompt_tokens
        for i in range(400):
            if rng.random() < 0.3 and s.num_completion_tokens > 12:
                s.append_token(s.token_ids[-12 + rng.randrange(12)])  # copy a recent token: repeats appear
            else:
                s.append_token(1000 + rng.randrange(alphabet))
            if i % check_every == 0:
                assert s.has_degenerate_repetition() == _degenerate_by_definition(s.token_ids, prompt), (trial, i)


def test_sampling_params_validation():
    with pytest.raises(ValueError):
        SamplingParams(temperature=0.0)
    with pytest.raises(ValueError):
        SamplingParams(top_p=0.0)
    with pytest.raises(ValueError):
        SamplingParams(max_tokens=0)
    sp = SamplingParams.builder().temperature(0.7).top_k(5).seed(3).build()
    assert sp.deterministic().top_k == 1 and sp.deterministic().top_p == 1.0
    d = SamplingParams()
    assert (d.temperature, d.top_p, d.top_k, d.max_tokens) == (0.6, 0.95, 0, 256)


def test_abort_and_clear_release_blocks():
    cfg = EngineConfig(max_num_seqs=4, max_num_batched_tokens=4096, max_model_len=4096)
    released = []
    sch = Scheduler(cfg, 8, on_release=released.append)
    a, b = seq(300), seq(20, start=900)
    sch.add(a)
    sch.add(b)
    sch.schedule()
    assert sch.abort(a.seq_id) and a in released
    sch.clear()
    assert sch.block_manager.num_free_blocks == 8 and sch.is_finished()


def test_scheduler_caps_live_sequences_for_recurrent_state():
    """With a state arena of N rows no (N+1)-th sequence is admitted until one finishes."""
    from nanovllm_b200.config import EngineConfig
    from nanovllm_b200.engine.scheduler import Scheduler
    from nanovllm_b200.engine.sequence import Sequence
    from nanovllm_b200.sampling_params import SamplingParams
    cfg = EngineConfig(max_num_seqs=2, max_model_len=1024, kvcache_block_size=256, max_num_batched_tokens=4096)
    sch = Scheduler(cfg, 64, max_live_seqs=3)
    seqs = [Sequence(list(range(10)), SamplingParams(max_tokens=4, ignore_eos=True), 256) for _ in range(5)]
    for s in seqs:
        sch.add(s)
    first, pf = sch.schedule()
    second, pf2 = sch.schedule()
    assert pf and pf2 and len(first) == 2 and len(second) == 1  # the batch cap, then the live cap
    assert len(sch.running) == 3 and len(sch.waiting) == 2


def test_nvtx_ranges_are_off_by_default_and_harmless_on_cpu():
    from nanovllm_b200.utils import trace
    assert not trace.enabled()
    trace.set_enabled(True)
    try:
        with trace.nvtx("x"):  # no CUDA here: a no-op, not an error
            pass
    finally:
        trace.set_enabled(False)


def test_decode_block_rows_are_written_incrementally():
    """The graph-replay block-table rows keep their contents across steps: unchanged sequences only append new
    blocks, a reordered batch or a released-and-reallocated table rewrites the row."""
    import numpy as np
    from nanovllm_b200.engine.model_runner import write_block_rows
    from nanovllm_b200.engine.sequence import Sequence
    a, b = Sequence([1, 2, 3]), Sequence([4, 5])
    a.block_table[:] = [7, 8]
    b.block_table[:] = [3]
    btn = np.full((4, 6), -1, dtype=np.int32)
    rows = [None] * 4
    write_block_rows(btn, rows, [a, b])
    assert btn[0, :2].tolist() == [7, 8] and btn[1, :1].tolist() == [3]
    a.block_table.append(9)
    btn[0, :2] = -5  # untouched prefix must not be rewritten
    write_block_rows(btn, rows, [a, b])
    assert btn[0, :3].tolist() == [-5, -5, 9]
    write_block_rows(btn, rows, [b, a])  # reordered: both rows rewritten
    assert btn[0, :1].tolist() == [3] and btn[1, :3].tolist() == [7, 8, 9]
    b.block_table.clear()
    b.bt_gen += 1  # what the block manager does on release
    b.block_table[:] = [11, 12]
    write_block_rows(btn, rows, [b, a])
    assert btn[0, :2].tolist() == [11, 12]


def test_prefill_and_decode_staging_match_block_tables():
    """Step staging: flat ids, positions and KV slots of the scheduled (uncached) tokens of a chunked, partly
    prefix-cached prefill batch, and the decode rows, agree with a per-token computation from the block tables."""
    import random
    import torch
    from nanovllm_b200.engine import model_runner as mr
    cfg = EngineConfig(max_num_seqs=8, max_model_len=4096, max_num_batched_tokens=1500)
    sch = Scheduler(cfg, num_blocks=64)
    rng = random.Random(3)
    shared = [rng.randrange(1000) for _ in range(512)]
    for n in (700, 300, 1100, 40):
        sch.add(Sequence(shared + [rng.randrange(1000) for _ in range(n)], SamplingParams(max_tokens=4), 256))
    r = mr.ModelRunner.__new__(mr.ModelRunner)
    r.cfg, r.is_cuda, r.block_size, r.max_blocks_per_seq = cfg, False, 256, 16
    r.state_arena, r.device, r.last_h2d_bytes, r.step_events, r._started = None, torch.device("cpu"), 0, None, False
    r._staging()
    steps = 0
    while not sch.is_finished():
        seqs, pre = sch.schedule()
        if pre:
            ids, pos, ctx = r.prepare_prefill(seqs)
            want_ids, want_pos, want_slots = [], [], []
            for s in seqs:
                a = s.num_cached_tokens
                for p in range(a, a + s.num_scheduled_tokens):
                    want_ids.append(s.token_ids[p])
                    want_pos.append(p)
                    want_slots.append(s.block_table[p // 256] * 256 + p % 256)
            assert ids.tolist() == want_ids and pos.tolist() == want_pos
            assert ctx.slot_mapping.tolist() == want_slots
        else:
            ids, pos, ctx = r.prepare_decode(seqs)
            assert ids.tolist() == [s.last_token for s in seqs]
            assert pos.tolist() == [len(s) - 1 for s in seqs]
            assert ctx.context_lens.tolist() == [len(s) for s in seqs]
            assert ctx.slot_mapping.tolist() == [s.block_table[(len(s) - 1) // 256] * 256 + (len(s) - 1) % 256
                                                 for s in seqs]
        sch.postprocess(seqs, [rng.randrange(1000) for _ in seqs], pre)
        steps += 1
    assert steps > 4


def test_sampling_knobs_stay_on_device_while_the_batch_is_unchanged():
    import torch
    from nanovllm_b200.engine import model_runner as mr
    cfg = EngineConfig(max_num_seqs=8, max_model_len=512)
    r = mr.ModelRunner.__new__(mr.ModelRunner)
    r.cfg, r.is_cuda, r.block_size, r.max_blocks_per_seq = cfg, False, 256, 2
    r.device, r.last_h2d_bytes, r.step_events, r._started = torch.device("cpu"), 0, None, False
    r._staging()
    a = Sequence([1, 2, 3], SamplingParams(temperature=0.5, top_k=3, top_p=0.9, seed=11))
    b = Sequence([4, 5], SamplingParams(temperature=0.9, top_k=0, top_p=0.5))
    t1 = r._sampling_tensors([a, b])
    a.append_token(7)
    t2 = r._sampling_tensors([a, b])
    assert all(x is y for x, y in zip(t1[:5], t2[:5]))  # knobs not staged again
    assert t2[5].tolist() == [4, 2]
    t3 = r._sampling_tensors([b, a])  # another order: restaged
    assert t3[0].tolist() == pytest.approx([0.9, 0.5]) and t3[1].tolist() == [0, 3]
    assert t3[3].tolist()[1] == 11 and t3[4].tolist() == [b.seq_id, 0] and t3[5].tolist() == [2, 4]


def test_step_input_checks_pass_a_real_run_and_catch_violations():
    """Debug-mode step checks (engine/checks.py): a full engine run with chunked prefill, prefix sharing and
    preemption passes them; bad ids, slots, block-table entries and page races are reported, not executed."""
    import numpy as np
    from nanovllm_b200.config import HfConfig
    from nanovllm_b200.engine.checks import check_step
    from nanovllm_b200.exceptions import StepInputError
    from nanovllm_b200.llm import LLM
    from nanovllm_b200.models.registry import init_random_weights
    hf = HfConfig(vocab_size=300, hidden_size=64, intermediate_size=128, num_hidden_layers=1, num_attention_heads=2,
                  num_key_value_heads=1, head_dim=32, max_position_embeddings=1024, model_type="qwen3")
    cfg = EngineConfig(max_num_seqs=4, max_model_len=1024, num_kvcache_blocks=5, max_num_batched_tokens=300,
                       check_inputs=True)
    llm = LLM((hf, init_random_weights(hf, 0)), cfg, device="cpu")
    shared = list(range(1, 257))
    prompts = [shared + [7] * 30, shared + [8] * 200, list(range(40, 290)), [3] * 20]
    outs = llm.generate_token_ids(prompts, SamplingParams(max_tokens=40, ignore_eos=True, seed=1))
    assert all(len(o.token_ids) == 40 for o in outs) and llm.scheduler.num_preemptions > 0

    base = dict(ids=np.array([5, 6]), pos=np.array([256, 3]), slots=np.array([256 * 2 + 0, 256 * 3 + 3]),
                block_tables=np.array([[1, 2], [3, 0]]), context_lens=np.array([257, 4]),
                seq_of_token=np.array([0, 1]), vocab=300, max_pos=1024, num_blocks=5, block_size=256)
    check_step(**base)
    cases = [("ids", np.array([5, 300]), "token id"), ("slots", np.array([256 * 2, 256 * 5]), "slot"),
             ("block_tables", np.array([[1, 7], [3, 0]]), "block-table entry"),
             ("slots", np.array([256 * 2 + 1, 256 * 3 + 3]), "not the block table's slot"),
             ("context_lens", np.array([600, 4]), "pages")]
    for key, val, msg in cases:
        with pytest.raises(StepInputError, match=msg):
            check_step(**{**base, key: val})
    # two tokens of one step on one slot, and a page written by one sequence while another's table holds it
    with pytest.raises(StepInputError, match="more than one token"):
        check_step(**{**base, "pos": np.array([3, 3]), "slots": np.array([256 * 3 + 3, 256 * 3 + 3]),
                      "block_tables": np.array([[3, 0], [3, 0]]), "context_lens": np.array([4, 4])})
    with pytest.raises(StepInputError, match="copy-on-write"):
        check_step(**{**base, "block_tables": np.array([[1, 2], [3, 2]]), "context_lens": np.array([257, 300])})


def test_host_bench_runs():
    from nanovllm_b200.utils.host_bench import run
    res = run(batch=8, steps=5, warmup=60)
    assert res["total"] > 0 and set(res) >= {"schedule", "postprocess"}


def test_decode_fast_path_schedules_like_the_preempting_loop():
    """The one-pass decode batch and the pop / re-push loop give the same batches, pages and preemptions over a
    random request stream with a pool small enough to preempt."""
    import random

    def trace(fast):
        rng = random.Random(21)
        cfg = EngineConfig(max_num_seqs=5, max_model_len=2048, max_num_batched_tokens=600)
        sch = Scheduler(cfg, num_blocks=8)
        sch.decode_fast_path = fast
        for i in range(9):
            sch.add(Sequence([rng.randrange(100) for _ in range(rng.randint(5, 500))],
                             SamplingParams(max_tokens=rng.randint(5, 400), ignore_eos=True), 256))
        out = []
        while not sch.is_finished():
            seqs, pre = sch.schedule()
            out.append((pre, [(s.seq_id - base, tuple(s.block_table)) for s in seqs]))
            sch.postprocess(seqs, [rng.randrange(100) for _ in seqs], pre)
        return out, sch.num_preemptions

    from nanovllm_b200.engine import sequence as _sq
    base = next(_sq._SEQ_COUNTER) + 1
    slow = trace(False)
    base = next(_sq._SEQ_COUNTER) + 1
    fast = trace(True)
    assert slow[1] > 0 and fast == slow
