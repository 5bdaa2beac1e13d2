"""Model runner: KV arena, step preparation, CUDA graphs per decode batch bucket, sampling.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/engine/Transformer.java (ctor + KV arena
113-143 and 295-314, ``step`` = prepare -> forward -> logits -> sample 168-195, ``preparePrefill`` 342-424 builds
flat ids / positions / cu_seqlens / slot mapping of uncached tokens / block tables, ``prepareDecode`` 433-457
builds last token, position len-1, slot, context lengths and -1-padded block tables).

B200 design:
* the KV arena is one zero-initialised bf16 allocation per (kv heads, head dim) class, laid out
  [layers, 2, num_blocks, kv_heads, block_size, head_dim] so a 64-token tile of one head is one contiguous
  TMA box; the block count comes from free device memory (``gpu_memory_utilization``) instead of the JVM heap;
* step metadata is written into pinned host staging buffers and copied with one async H2D per field; the
  sampling knobs stay on the device while a decode batch keeps its sequences, and graph-replay block-table rows
  are only appended to;
* decode runs as a replay of a CUDA graph captured per batch bucket (1, 2, 4, 8, 16, 32, ...); padded rows get
  slot -1 (no KV write) and context length 0 (no attention work);
* the sampler keys Philox by (request seed, position) when the request has a seed, else by
  (engine seed + sequence id, position), so reruns are bit-identical regardless of batch composition.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from .. import ops
from ..config import EngineConfig, HfConfig
from ..parallel import state as ps
from ..utils.trace import nvtx
from .context import StepContext, set_context
from .sequence import Sequence


def write_block_rows(btn, rows: List[Optional[tuple]], seqs: List[Sequence]) -> None:
    """Decode block-table rows in place (numpy view of pinned memory).  The rows persist across steps: a row
    whose sequence and block-table generation are unchanged only gets its newly appended blocks, any other row
    is rewritten; entries past a row's context are never read by the attention kernel, so nothing is cleared
    (padding rows have context 0).  ``rows[i]`` records (seq id, generation, blocks written) for row i."""
    for i, s in enumerate(seqs):
        bt_list = s.block_table
        nb = len(bt_list)
        st = rows[i]
        if st is not None and st[0] == s.seq_id and st[1] == s.bt_gen and st[2] <= nb:
            if st[2] < nb:
                btn[i, st[2]:nb] = bt_list[st[2]:]
        elif nb:
            btn[i, :nb] = bt_list
        rows[i] = (s.seq_id, s.bt_gen, nb)


def _bucket_sizes(max_bs: int) -> List[int]:
    out = [b for b in (1, 2, 4, 8) if b <= max_bs]
    out += list(range(16, max_bs + 1, 16))
    if max_bs not in out:
        out.append(max_bs)
    return sorted(set(out))


class ModelRunner:
    def __init__(self, model, hf: HfConfig, cfg: EngineConfig, device: torch.device):
        self.model = model
        self.hf = hf
        self.cfg = cfg
        self.device = device
        self.is_cuda = device.type == "cuda"
        self.block_size = cfg.kvcache_block_size
        self.max_blocks_per_seq = (cfg.max_model_len + self.block_size - 1) // self.block_size
        self.graphs: Dict[int, torch.cuda.CUDAGraph] = {}
        self.graph_pool = None
        self.graph_bufs = None
        self.num_blocks = 0
        self.kv_arenas: List[torch.Tensor] = []
        self.state_arena: Optional[torch.Tensor] = None
        self.state_capacity: Optional[int] = None  # live sequences the recurrent-state arena can hold
        self.state_rows: Dict[int, int] = {}
        self.free_state_rows: List[int] = []
        self.final_softcap = getattr(model, "final_softcap", 0.0)
        if self.is_cuda and ps.tp_size() > 1:
            # symmetric buffers for the fused all-reduce + RMSNorm kernels (collective: same point on all ranks)
            from ..parallel import sp, symm
            symm.init_workspace(max(cfg.max_num_batched_tokens, cfg.max_num_seqs), hf.hidden_size, device)
            # sequence-parallel buffers for the fused decode path (GEMM + reduce-scatter, all-gather + norm + GEMM)
            sp.init_workspace(min(cfg.max_num_seqs, sp.MAX_ROWS), hf.hidden_size, device)
        self._allocate_kv()
        self._allocate_state()
        self._attn_scratch = None
        self.step_events = None      # optional (start, end) CUDA events bracketing one step's GPU work
        self._started = False
        self.last_h2d_bytes = 0
        self.graph_launches: Dict[int, int] = {}
        self._staging()
        if self.is_cuda and not cfg.enforce_eager:
            self.capture_graphs()

    # ------------------------------------------------------------------ memory
    def _kv_bytes_per_block(self) -> int:
        return sum(2 * self.block_size * nkv * hd * 2 for _, nkv, hd in self.model.kv_specs())

    def _allocate_kv(self) -> None:
        specs = self.model.kv_specs()
        bpb = max(1, self._kv_bytes_per_block())
        if self.cfg.num_kvcache_blocks > 0:
            nb = self.cfg.num_kvcache_blocks
        elif self.is_cuda:
            free, total = torch.cuda.mem_get_info(self.device)
            used = total - free
            reserve = self._activation_reserve()
            budget = int(total * self.cfg.gpu_memory_utilization) - used - reserve
            cap = max(32, budget // bpb)
            per_seq = self.max_blocks_per_seq
            nb = int(min(max(self.cfg.max_num_seqs * per_seq, 128), cap))
            if ps.tp_size() > 1:
                # every rank must schedule with the same pool size (ranks run the scheduler in lock-step)
                t = torch.tensor([nb], dtype=torch.int64, device=self.device)
                torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN, group=ps.tp_group())
                nb = int(t.item())
        else:
            nb = int(min(max(self.cfg.max_num_seqs * self.max_blocks_per_seq, 128), max(32, (2 << 30) // bpb)))
        self.num_blocks = nb
        groups: Dict[Tuple[int, int], List[int]] = {}
        for layer, nkv, hd in specs:
            groups.setdefault((nkv, hd), []).append(layer)
        caches = {}
        for (nkv, hd), layers in groups.items():
            arena = torch.zeros(len(layers), 2, nb, nkv, self.block_size, hd, dtype=torch.bfloat16, device=self.device)
            self.kv_arenas.append(arena)
            for j, layer in enumerate(layers):
                caches[layer] = (arena[j, 0], arena[j, 1])
        self.model.bind_kv(caches)

    def _activation_reserve(self) -> int:
        hf = self.hf
        T = self.cfg.max_num_batched_tokens
        tp = ps.tp_size()
        width = (hf.num_attention_heads + 2 * hf.num_key_value_heads) * max(hf.head_dim, 1) // tp
        width += 3 * max(hf.intermediate_size, 1) // tp + 6 * hf.hidden_size
        act = 2 * T * width * 2
        logits = self.cfg.max_num_seqs * hf.vocab_size * 4
        return int(act + logits + (2 << 30))

    def _allocate_state(self) -> None:
        specs = self.model.state_specs()  # [(layer, row_width)]
        if not specs:
            return
        width = sum(w for _, w in specs)
        # live sequences can outnumber max_num_seqs (that caps each batch, not admission): keep twice as many rows;
        # the scheduler admits no new sequence while every row is taken (``state_capacity``)
        rows = 2 * self.cfg.max_num_seqs + 1
        self.state_capacity = rows - 1
        self.state_arena = torch.zeros(rows, width, dtype=torch.float32, device=self.device)
        self.free_state_rows = list(range(rows - 1, 0, -1))  # row 0 is a scratch row for padding
        self.model.bind_state(self.state_arena)

    def release_state(self, seq: Sequence) -> None:
        row = self.state_rows.pop(seq.seq_id, None)
        if row is not None:
            self.free_state_rows.append(row)

    def _state_row(self, seq: Sequence) -> Tuple[int, bool]:
        row = self.state_rows.get(seq.seq_id)
        if row is not None:
            return row, False
        row = self.free_state_rows.pop()
        self.state_rows[seq.seq_id] = row
        return row, True

    # ------------------------------------------------------------------ staging
    def _staging(self) -> None:
        pin = self.is_cuda
        T = max(self.cfg.max_num_batched_tokens, self.cfg.max_num_seqs)
        S = self.cfg.max_num_seqs

        def buf(n, dtype):
            t = torch.empty(n, dtype=dtype)
            return t.pin_memory() if pin else t

        self.h_ids = buf(T, torch.int64)
        self.h_pos = buf(T, torch.int64)
        self.h_slots = buf(T, torch.int32)
        self.h_cu_q = buf(S + 1, torch.int32)
        self.h_cu_k = buf(S + 1, torch.int32)
        self.h_ctx = buf(S, torch.int32)
        self.h_last = buf(S, torch.int64)
        self.h_bt = buf(S * self.max_blocks_per_seq, torch.int32)
        self.h_rows = buf(S, torch.int64)
        self.h_fresh = buf(S, torch.bool)
        self.h_temps = buf(S, torch.float32)
        self.h_topk = buf(S, torch.int32)
        self.h_topp = buf(S, torch.float32)
        self.h_seeds = buf(S, torch.int64)
        self.h_sids = buf(S, torch.int64)
        self.h_steps = buf(S, torch.int32)
        self._err_host = buf(1, torch.int32)
        self._bt_rows: List[Optional[tuple]] = [None] * S  # (seq id, block-table generation, blocks written)
        self._samp_key: Optional[List[int]] = None  # seq ids whose sampling knobs are on the device, in row order
        self._samp_dev: tuple = ()
        # numpy views share the pinned memory: element writes from Python stay cheap
        for name in ("ids", "pos", "slots", "cu_q", "cu_k", "ctx", "last", "bt", "rows", "fresh", "temps", "topk",
                     "topp", "seeds", "sids", "steps"):
            setattr(self, "n_" + name, getattr(self, "h_" + name).numpy())

    def _begin_gpu(self) -> None:
        if self.step_events is not None and not self._started:
            self.step_events[0].record()
            self._started = True

    def _h2d(self, host: torch.Tensor, n: int) -> torch.Tensor:
        self._begin_gpu()
        self.last_h2d_bytes += n * host.element_size()
        return host[:n].to(self.device, non_blocking=True)

    def _fill_block_tables(self, seqs: List[Sequence]) -> int:
        self._bt_rows = [None] * len(self._bt_rows)  # h_bt is rewritten here with another row width
        width = max(1, max(len(s.block_table) for s in seqs))
        bt = self.n_bt[:len(seqs) * width].reshape(len(seqs), width)
        bt.fill(0)
        for i, s in enumerate(seqs):
            if s.block_table:
                bt[i, :len(s.block_table)] = s.block_table
        return width

    def prepare_prefill(self, seqs: List[Sequence]):
        ids = []
        cu_q, cu_k = [0], [0]
        max_q = max_k = 0
        counts = []
        bs = self.block_size
        off = 0
        for s in seqs:
            start = s.num_cached_tokens
            end = start + s.num_scheduled_tokens
            ids.extend(s.token_ids[start:end])
            qlen, klen = end - start, end
            # positions and KV slots as numpy ranges (a prefill step stages up to max_num_batched_tokens of each)
            p = np.arange(start, end, dtype=np.int64)
            self.n_pos[off:off + qlen] = p
            self.n_slots[off:off + qlen] = np.asarray(s.block_table, dtype=np.int64)[p // bs] * bs + p % bs
            off += qlen
            cu_q.append(cu_q[-1] + qlen)
            cu_k.append(cu_k[-1] + klen)
            max_q, max_k = max(max_q, qlen), max(max_k, klen)
            counts.append(qlen)
        T, S = len(ids), len(seqs)
        self.n_ids[:T] = ids
        self.n_cu_q[:S + 1] = cu_q
        self.n_cu_k[:S + 1] = cu_k
        self.n_last[:S] = cu_q[1:]
        self.n_last[:S] -= 1
        width = self._fill_block_tables(seqs)
        if self.cfg.check_inputs:
            self._check(seqs, T, S, self.n_bt[:S * width].reshape(S, width),
                        np.diff(np.asarray(cu_k, dtype=np.int64)), np.repeat(np.arange(S), counts))
        ctx = StepContext(is_prefill=True, num_seqs=S, num_tokens=T,
                          slot_mapping=self._h2d(self.h_slots, T),
                          block_tables=self._h2d(self.h_bt, S * width).view(S, width),
                          cu_seqlens_q=self._h2d(self.h_cu_q, S + 1), cu_seqlens_k=self._h2d(self.h_cu_k, S + 1),
                          max_seqlen_q=max_q, max_seqlen_k=max_k, last_token_idx=self._h2d(self.h_last, S),
                          seq_token_counts=counts)
        self._prepare_state(seqs, ctx)
        return self._h2d(self.h_ids, T), self._h2d(self.h_pos, T), ctx

    def _prepare_state(self, seqs: List[Sequence], ctx: StepContext, pad_to: int = 0) -> None:
        if self.state_arena is None:
            return
        n = len(seqs)
        for i, s in enumerate(seqs):
            row, fresh = self._state_row(s)
            self.n_rows[i] = row
            self.n_fresh[i] = fresh or (ctx.is_prefill and s.num_cached_tokens == 0)
        for i in range(n, max(n, pad_to)):
            self.n_rows[i] = 0
            self.n_fresh[i] = True
        m = max(n, pad_to)
        ctx.state_rows = self._h2d(self.h_rows, m)
        ctx.state_fresh = self._h2d(self.h_fresh, m)

    def prepare_decode(self, seqs: List[Sequence]):
        S = len(seqs)
        bs = self.block_size
        self._fill_decode_rows(seqs, S)
        width = self._fill_block_tables(seqs)
        if self.cfg.check_inputs:
            self._check(seqs, S, S, self.n_bt[:S * width].reshape(S, width), self.n_ctx[:S].astype(np.int64),
                        np.arange(S))
        ctx = StepContext(is_prefill=False, num_seqs=S, num_tokens=S,
                          slot_mapping=self._h2d(self.h_slots, S), context_lens=self._h2d(self.h_ctx, S),
                          block_tables=self._h2d(self.h_bt, S * width).view(S, width),
                          max_context_len=max(len(s) for s in seqs))
        self._prepare_state(seqs, ctx)
        return self._h2d(self.h_ids, S), self._h2d(self.h_pos, S), ctx

    def _fill_decode_rows(self, seqs: List[Sequence], pad_to: int) -> None:
        blk = self.block_size
        n = len(seqs)
        # one list per field and one slice store each: element-wise stores into numpy cost ~0.1 us apiece
        lens = [s.num_tokens for s in seqs]
        self.n_ids[:n] = [s.last_token for s in seqs]
        self.n_ctx[:n] = lens
        self.n_pos[:n] = self.n_ctx[:n]
        self.n_pos[:n] -= 1
        self.n_slots[:n] = [s.block_table[(m - 1) // blk] * blk + (m - 1) % blk for s, m in zip(seqs, lens)]
        if pad_to > n:
            self.n_ids[n:pad_to] = 0
            self.n_pos[n:pad_to] = 0
            self.n_slots[n:pad_to] = -1
            self.n_ctx[n:pad_to] = 0

    def _check(self, seqs: List[Sequence], T: int, S: int, bt, ctx_lens, seq_of_token) -> None:
        """Debug-mode range / consistency / race check of the staged step (engine/checks.py)."""
        from .checks import check_step
        rows = None
        if self.state_arena is not None:
            rows = np.asarray([self.state_rows.get(s.seq_id, 0) for s in seqs], dtype=np.int64)
        check_step(ids=self.n_ids[:T], pos=self.n_pos[:T], slots=self.n_slots[:T].astype(np.int64), block_tables=bt,
                   context_lens=ctx_lens, seq_of_token=seq_of_token, vocab=self.hf.vocab_size,
                   max_pos=self.cfg.max_model_len, num_blocks=self.num_blocks, block_size=self.block_size,
                   state_rows=rows, state_capacity=0 if self.state_arena is None else self.state_arena.shape[0])

    # ------------------------------------------------------------------ sampling
    def _sampling_tensors(self, seqs: List[Sequence]):
        """(temperature, top_k, top_p, seed, seed id, step) per row on the device.  Only the step changes while
        the batch keeps its sequences in the same order (every decode step between admissions and finishes):
        the other five stay on the device from the step that staged them."""
        n = len(seqs)
        self.n_steps[:n] = [s.num_tokens for s in seqs]
        steps = self._h2d(self.h_steps, n)
        key = [s.seq_id for s in seqs]
        if key != self._samp_key:
            base = self.cfg.seed * 1000003
            self.n_temps[:n] = [s.temperature for s in seqs]
            self.n_topk[:n] = [s.top_k for s in seqs]
            self.n_topp[:n] = [s.top_p for s in seqs]
            self.n_seeds[:n] = [(int(s.seed) if s.seed is not None else base + s.seq_id) & 0x7FFFFFFFFFFFFFFF
                                for s in seqs]
            self.n_sids[:n] = [0 if s.seed is not None else s.seq_id for s in seqs]
            self._samp_dev = tuple(self._h2d(h, n) for h in (self.h_temps, self.h_topk, self.h_topp, self.h_seeds,
                                                             self.h_sids))
            self._samp_key = key
        return self._samp_dev + (steps,)

    def sample(self, logits: torch.Tensor, seqs: List[Sequence]) -> torch.Tensor:
        n = len(seqs)
        head = getattr(self.model, "lm_head", None)
        if head is not None and getattr(head, "sharded", False):
            # vocab-parallel logits: greedy rows need only the distributed argmax (exact, no logit gather)
            if all(s.top_k == 1 for s in seqs):
                return head.argmax(logits[:n], self.final_softcap)
            if all(1 <= s.top_k <= head.CANDIDATE_K for s in seqs):
                # top-k rows: exchange each rank's top-k candidates instead of the [n, V] logits
                t = self._sampling_tensors(seqs)
                return head.sample_candidates(logits[:n], *t, kmax=max(s.top_k for s in seqs),
                                              softcap=self.final_softcap)
            logits = head.gather_full(logits[:n])
        t = self._sampling_tensors(seqs)
        return ops.sample(logits[:n], *t, softcap=self.final_softcap)

    # ------------------------------------------------------------------ execution
    def _decode_scratch(self, bs: int) -> Optional[torch.Tensor]:
        if not self.is_cuda:
            return None
        need = 0
        for _, nkv, hd in self.model.kv_specs():
            nq = nkv * max(1, self.hf.num_attention_heads // max(1, self.hf.num_key_value_heads))
            need = max(need, ops.decode_scratch_numel(bs, nq, nkv, hd, self.cfg.max_model_len))
        if need == 0:
            return None
        if self._attn_scratch is None or self._attn_scratch.numel() < need:
            self._attn_scratch = torch.empty(need, dtype=torch.float32, device=self.device)
        return self._attn_scratch

    @torch.inference_mode()
    def run(self, seqs: List[Sequence], is_prefill: bool) -> List[int]:
        self._started = False
        self.last_h2d_bytes = 0
        with nvtx("forward"):
            logits = self.forward_logits(seqs, is_prefill)
        with nvtx("sample"):
            toks = self.sample(logits, seqs)
        if self.is_cuda:
            # the device error word rides back with the sampled tokens (4 bytes on the same synchronisation): a
            # bounded wait that gave up during this step surfaces here instead of as silently wrong tokens
            self._err_host.copy_(ops.error_word(self.device), non_blocking=True)
        if self.step_events is not None:
            self.step_events[1].record()
        out = toks.tolist()
        if self.is_cuda and int(self._err_host[0]) != 0:
            ops.check_device_errors(self.device)
        return out

    @torch.inference_mode()
    def forward_logits(self, seqs: List[Sequence], is_prefill: bool) -> torch.Tensor:
        if is_prefill:
            ids, pos, ctx = self.prepare_prefill(seqs)
            set_context(ctx)
            logits = self.model.compute_logits(self.model.forward(ids, pos))
            set_context(None)
            return logits
        bs = len(seqs)
        if self.graphs and bs <= max(self.graphs):
            return self._replay(seqs)
        ids, pos, ctx = self.prepare_decode(seqs)
        ctx.max_context_len = self.cfg.max_model_len
        ctx.attn_scratch = self._decode_scratch(bs)
        set_context(ctx)
        logits = self.model.compute_logits(self.model.forward(ids, pos))
        set_context(None)
        return logits

    # ------------------------------------------------------------------ CUDA graphs
    def _graph_context(self, bs: int) -> StepContext:
        g = self.graph_bufs
        ctx = StepContext(is_prefill=False, num_seqs=bs, num_tokens=bs, slot_mapping=g["slots"][:bs],
                          context_lens=g["ctx"][:bs], block_tables=g["bt"][:bs],
                          max_context_len=self.cfg.max_model_len, attn_scratch=g["scratch"])
        if self.state_arena is not None:
            ctx.state_rows = g["rows"][:bs]
            ctx.state_fresh = g["fresh"][:bs]
        return ctx

    @torch.inference_mode()
    def capture_graphs(self) -> None:
        max_bs = min(self.cfg.max_num_seqs, self.cfg.cuda_graph_max_bs, 512)
        dev = self.device
        g = {
            "ids": torch.zeros(max_bs, dtype=torch.int64, device=dev),
            "pos": torch.zeros(max_bs, dtype=torch.int64, device=dev),
            "slots": torch.full((max_bs,), -1, dtype=torch.int32, device=dev),
            "ctx": torch.zeros(max_bs, dtype=torch.int32, device=dev),
            "bt": torch.zeros(max_bs, self.max_blocks_per_seq, dtype=torch.int32, device=dev),
            "rows": torch.zeros(max_bs, dtype=torch.int64, device=dev),
            "fresh": torch.ones(max_bs, dtype=torch.bool, device=dev),
        }
        g["scratch"] = self._decode_scratch(max_bs)
        self.graph_bufs = g
        self.graph_logits = {}
        # eager warm-up at the largest bucket sizes the GEMM workspace before capture
        set_context(self._graph_context(max_bs))
        self.model.compute_logits(self.model.forward(g["ids"][:max_bs], g["pos"][:max_bs]))
        torch.cuda.synchronize(dev)
        for bs in reversed(_bucket_sizes(max_bs)):
            graph = torch.cuda.CUDAGraph()
            set_context(self._graph_context(bs))
            self.model.compute_logits(self.model.forward(g["ids"][:bs], g["pos"][:bs]))  # warm this shape
            n0 = ops.launch_count()
            with torch.cuda.graph(graph, self.graph_pool):
                out = self.model.compute_logits(self.model.forward(g["ids"][:bs], g["pos"][:bs]))
            self.graph_launches[bs] = ops.launch_count() - n0
            if self.graph_pool is None:
                self.graph_pool = graph.pool()
            self.graphs[bs] = graph
            self.graph_logits[bs] = out
            torch.cuda.synchronize(dev)
        set_context(None)
        ops.check_device_errors(dev)

    def _replay(self, seqs: List[Sequence]) -> torch.Tensor:
        n = len(seqs)
        bs = next(b for b in sorted(self.graphs) if b >= n)
        g = self.graph_bufs
        self._fill_decode_rows(seqs, bs)
        width = self.max_blocks_per_seq
        btn = self.n_bt[:bs * width].reshape(bs, width)
        write_block_rows(btn, self._bt_rows, seqs)
        if self.cfg.check_inputs:
            self._check(seqs, n, n, btn[:n], self.n_ctx[:n].astype(np.int64), np.arange(n))
        bt = self.h_bt[:bs * width].view(bs, width)
        self._begin_gpu()
        self.last_h2d_bytes += bs * (8 + 8 + 4 + 4 + 4 * width)
        g["ids"][:bs].copy_(self.h_ids[:bs], non_blocking=True)
        g["pos"][:bs].copy_(self.h_pos[:bs], non_blocking=True)
        g["slots"][:bs].copy_(self.h_slots[:bs], non_blocking=True)
        g["ctx"][:bs].copy_(self.h_ctx[:bs], non_blocking=True)
        g["bt"][:bs].copy_(bt, non_blocking=True)
        if self.state_arena is not None:
            ctx = StepContext(is_prefill=False, num_seqs=n, num_tokens=n)
            self._prepare_state(seqs, ctx, pad_to=bs)
            g["rows"][:bs].copy_(ctx.state_rows)
            g["fresh"][:bs].copy_(ctx.state_fresh)
        self.graphs[bs].replay()
        ops.add_launches(self.graph_launches.get(bs, 0))
        return self.graph_logits[bs]

    def close(self) -> None:
        self.graphs.clear()
        self.graph_logits = {}
        self.graph_bufs = None
        self.kv_arenas.clear()
        self.state_arena = None
