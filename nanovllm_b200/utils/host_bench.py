"""Host-side cost of one decode step, without a model: scheduling, staging (decode rows, block-table rows,
sampling knobs) and post-processing (append, stop rules incl. the degenerate-repetition detector) for a batch of
running sequences, timed with perf_counter.  The device forward is not run; this is the part of a step the GPU
waits for in a synchronous engine loop.

    python -m nanovllm_b200.utils.host_bench --batch 128 --steps 200 [--no-degenerate]
"""
from __future__ import annotations

import argparse
import random
import time

import torch

from ..config import EngineConfig
from ..engine import model_runner as mr
from ..engine.scheduler import Scheduler
from ..engine.sequence import Sequence
from ..sampling_params import SamplingParams


def run(batch: int = 128, steps: int = 200, warmup: int = 150, degenerate: bool = True, seed: int = 0) -> dict:
    rng = random.Random(seed)
    cfg = EngineConfig(max_num_seqs=batch, max_model_len=9216, max_num_batched_tokens=16384,
                       stop_on_degenerate=degenerate)
    sched = Scheduler(cfg, num_blocks=batch * 40, stop_token_ids=[-5])
    for _ in range(batch):
        n = rng.randint(512, 8192)
        sched.add(Sequence([rng.randrange(150000) for _ in range(n)],
                           SamplingParams(temperature=0.8, top_k=50, max_tokens=100000, ignore_eos=True)))
    while sched.waiting:  # admit everything (prefill without a model)
        seqs, pre = sched.schedule()
        sched.postprocess(seqs, [1] * len(seqs), pre)
    r = mr.ModelRunner.__new__(mr.ModelRunner)
    r.cfg, r.is_cuda, r.block_size, r.max_blocks_per_seq = cfg, False, cfg.kvcache_block_size, 36
    r.state_arena, r.device, r.last_h2d_bytes, r.step_events, r._started = None, torch.device("cpu"), 0, None, False
    r._staging()
    names = ("schedule", "decode rows", "block-table rows", "sampling knobs", "postprocess")
    tot = dict.fromkeys(names, 0.0)

    def step(acc):
        t = [time.perf_counter()]
        seqs, pre = sched.schedule()
        t.append(time.perf_counter())
        r._fill_decode_rows(seqs, len(seqs))
        t.append(time.perf_counter())
        mr.write_block_rows(r.n_bt[:len(seqs) * 36].reshape(len(seqs), 36), r._bt_rows, seqs)
        t.append(time.perf_counter())
        r._sampling_tensors(seqs)
        t.append(time.perf_counter())
        toks = [rng.randrange(150000) for _ in seqs]
        t0 = time.perf_counter()
        sched.postprocess(seqs, toks, pre)
        t.append(time.perf_counter() - t0 + t[-1])
        if acc is not None:
            for k, a, b in zip(names, t, t[1:]):
                acc[k] += b - a

    for _ in range(warmup):  # completions pass the detector's 48-token gate
        step(None)
    for _ in range(steps):
        step(tot)
    out = {k: v / steps * 1e6 for k, v in tot.items()}
    out["total"] = sum(out.values())
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=128)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--no-degenerate", action="store_true")
    a = ap.parse_args(argv)
    res = run(a.batch, a.steps, degenerate=not a.no_degenerate)
    print(f"host work per decode step, {a.batch} sequences (us): " +
          ", ".join(f"{k} {v:.1f}" for k, v in res.items()))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
