"""``LLM``: the engine front door (builder, generate family, cancel, timeout, stats, listeners).

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/llm/LLM.java:
* Builder knobs (1443-1946): sampling defaults, deterministic, stop token ids, max_num_batched_tokens,
  max_num_seqs, max_model_len, KV block size / count, warmup; embedding models are rejected (1883-1886);
* one in-flight generate per engine (a lock, 178, 774-822); ``cancel()`` sets a flag that is checked between
  engine steps (370-372, 910-928) and raises GenerationCancelledException; a wall-clock deadline raises
  GenerationTimeoutException the same way; an interrupted generate clears the scheduler (826-834);
* prompts are clamped so max_tokens <= max_model_len - prompt length, and a prompt that fills the context is
  an error (865-874);
* warmup = one synthetic 64-token prefill + 16 decode steps (277-301).
New here: per-request TTFT / TPOT (``GenerationStats``), an online request API (``add_request`` / ``step`` /
``abort``) for Poisson serving, and TP=1/2/4/8 through torch.distributed: SPMD (every rank runs this engine on the
same requests) or one front door (rank 0 takes the requests and broadcasts step plans, ``serve_worker`` on the
other ranks follows them; ``engine/plan.py``).
"""
from __future__ import annotations

import os
import threading
import time
from dataclasses import dataclass, field
from typing import Callable, Dict, Iterable, List, Optional, Sequence as Seq, Union

import torch

from .config import EngineConfig, HfConfig
from .engine.model_runner import ModelRunner
from .engine.scheduler import Scheduler
from .engine.sequence import Sequence
from .exceptions import (GenerationCancelledException, GenerationTimeoutException, NanoLlvmException,
                         TensorParallelAbort)
from .parallel import state as ps
from .utils.trace import nvtx
from .sampling_params import SamplingParams


@dataclass
class GenerationStats:
    """Counts and timings of one generate call (GenerationStats.java:23-63) plus TTFT / TPOT."""
    prompt_tokens: int = 0
    completion_tokens: int = 0
    elapsed_s: float = 0.0
    ttft_s: List[float] = field(default_factory=list)
    tpot_s: List[float] = field(default_factory=list)
    prefill_steps: int = 0
    decode_steps: int = 0
    preemptions: int = 0

    @property
    def completion_tokens_per_second(self) -> float:
        return self.completion_tokens / self.elapsed_s if self.elapsed_s > 0 else 0.0

    @staticmethod
    def _pct(xs: List[float], q: float) -> float:
        if not xs:
            return float("nan")
        s = sorted(xs)
        return s[min(len(s) - 1, int(round(q * (len(s) - 1))))]

    def p50_ttft(self) -> float:
        return self._pct(self.ttft_s, 0.5)

    def p99_ttft(self) -> float:
        return self._pct(self.ttft_s, 0.99)

    def p50_tpot(self) -> float:
        return self._pct(self.tpot_s, 0.5)


@dataclass
class GenerationOutput:
    prompt_token_ids: List[int]
    token_ids: List[int]
    text: Optional[str] = None
    finish_reason: str = "stop"
    ttft_s: Optional[float] = None


class LLM:
    def __init__(self, model, cfg: Optional[EngineConfig] = None, sampling: Optional[SamplingParams] = None,
                 device: Optional[Union[str, torch.device]] = None, warmup: bool = False,
                 unpack_parameters: bool = False, cpu_threads: Optional[int] = None):
        """``model``: an ``LlmModel`` (from LlmModelFactory) or a (HfConfig, weights-dict) tuple.
        ``unpack_parameters``: expand packed GGUF projections to bf16 for this engine (the shared model keeps its
        packed tensors).  ``cpu_threads``: intra-op threads when the engine runs on the CPU device."""
        from .api.model import LlmModel
        if isinstance(model, LlmModel):
            if model.is_embedding():
                raise ValueError("embedding models cannot back an LLM engine (use LlmModel.embed)")
            hf, weights, tokenizer = model.hf_config, model.weights, model.tokenizer
        else:
            hf, weights = model
            tokenizer = None
        self.hf: HfConfig = hf
        self.tokenizer = tokenizer
        # keep the LlmModel handle (think tags, options, engine refcount); a bare (config, weights) tuple is not
        # kept: the graph holds this rank's (sharded) copies, and the full tensors can be freed by the caller
        self.model_handle = model if isinstance(model, LlmModel) else None
        self.cfg = cfg or EngineConfig()
        self.cfg.clamp_to_model(hf)
        self.default_sampling = sampling or SamplingParams()
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
        self.device = torch.device(device)
        if cpu_threads is not None and self.device.type == "cpu":
            torch.set_num_threads(int(cpu_threads))
        if isinstance(model, LlmModel) and model.options.get("unpack_parameters"):
            unpack_parameters = True  # the model was opened with unpack_parameters
        if unpack_parameters:
            from .ops.quant import GgufPacked
            weights = {k: (v.dequantize(torch.bfloat16).to(self.device) if isinstance(v, GgufPacked) else v)
                       for k, v in weights.items()}
        from .models.base import unpacked_parameters
        from .models.registry import causal_model_class
        cls = causal_model_class(hf)
        with unpacked_parameters(unpack_parameters):  # QAT integer weights expand at graph build
            self.model = cls(hf, weights, self.device, max_pos=self.cfg.max_model_len + 1)
        stop = list(self.cfg.stop_token_ids)
        if not stop and tokenizer is not None:
            stop = list(tokenizer.stop_token_ids())
        if not stop and self.cfg.eos >= 0:
            stop = [self.cfg.eos]
        if self.model.state_specs():
            self.cfg.enable_prefix_caching = False
        self.runner = ModelRunner(self.model, hf, self.cfg, self.device)
        self.scheduler = Scheduler(self.cfg, self.runner.num_blocks, stop, on_release=self.runner.release_state,
                                   max_live_seqs=self.runner.state_capacity)
        # TP with one front door: rank 0 schedules and broadcasts step plans, the other ranks follow them
        self._plan_tx = self._plan_rx = None
        if ps.tp_size() > 1 and self.cfg.front_door == "rank0":
            from .engine.plan import PlanReceiver, PlanSender
            group = ps.control_group()
            if ps.tp_rank() == 0:
                self._plan_tx = PlanSender(group)
                self.scheduler.on_release = self._release_and_note
            else:
                self._plan_rx = PlanReceiver(group, self.cfg.kvcache_block_size, release=self.runner.release_state)
        self._lock = threading.Lock()
        self._cancel = threading.Event()
        self._closed = False
        self.listeners: List[Callable] = []
        self.listener = None          # default LlmListener for chat sessions on this engine
        self.system_prompt = ""       # default system prompt for chat sessions (empty, as in the reference)
        self.advisors: List = []      # LlmAdvisor list run before every chat turn
        self.advisor_mixer = None
        self.advisor_note_filter = None  # keep-test for advisor notes (default: non-blank)
        self.think_tags = None
        if warmup and self._plan_rx is None:  # a front-door worker follows rank 0's warm-up through the plans
            self.warmup()

    # ------------------------------------------------------------------ builder
    class Builder:
        def __init__(self, model):
            self._model = model
            self._cfg = {}
            self._sampling = SamplingParams()
            self._device = None
            self._warmup = False
            self._unpack = False
            self._cpu_threads = None
            self._extra = {}

        def max_num_batched_tokens(self, v): self._cfg["max_num_batched_tokens"] = int(v); return self
        def max_num_seqs(self, v): self._cfg["max_num_seqs"] = int(v); return self
        def max_model_len(self, v): self._cfg["max_model_len"] = int(v); return self
        def kvcache_block_size(self, v): self._cfg["kvcache_block_size"] = int(v); return self
        def num_kvcache_blocks(self, v): self._cfg["num_kvcache_blocks"] = int(v); return self
        def gpu_memory_utilization(self, v): self._cfg["gpu_memory_utilization"] = float(v); return self

        def kv_heap_fraction(self, v):
            """The reference's share of the heap for the KV cache: here the share of device memory the engine may
            fill (weights, activations and KV pages), in (0, 1]."""
            return self.gpu_memory_utilization(v)

        def cpu_threads(self, v):
            """Intra-op threads when the engine runs on the CPU device (>= 1); CUDA engines run on streams."""
            if int(v) < 1:
                raise ValueError(f"cpu_threads must be >= 1, got {v}")
            self._cpu_threads = int(v)
            return self

        def all_cpu_threads(self): return self.cpu_threads(os.cpu_count() or 1)
        def disable_multi_cpu(self): return self.cpu_threads(1)

        def allow_unpack_parameters(self, v=True):
            """Expand packed GGUF projections to bf16 for this engine (more memory, the dense GEMM path)."""
            self._unpack = bool(v)
            return self
        def tensor_parallel_size(self, v): self._cfg["tensor_parallel_size"] = int(v); return self
        def front_door(self, v): self._cfg["front_door"] = str(v); return self
        def enforce_eager(self, v=True): self._cfg["enforce_eager"] = bool(v); return self
        def cuda_graph_max_bs(self, v): self._cfg["cuda_graph_max_bs"] = int(v); return self
        def stop_token_ids(self, ids): self._cfg["stop_token_ids"] = tuple(int(i) for i in ids); return self
        def stop_on_degenerate(self, v): self._cfg["stop_on_degenerate"] = bool(v); return self
        def seed(self, v): self._cfg["seed"] = int(v); return self
        def sampling(self, sp: SamplingParams): self._sampling = sp; return self
        def deterministic(self): self._sampling = self._sampling.deterministic(); return self
        def device(self, d): self._device = d; return self
        def warmup(self, v=True): self._warmup = bool(v); return self
        def skip_warmup(self): return self.warmup(False)
        # chat-level defaults picked up by ChatSession / RagSession (LLM.java builder knobs)
        def listen(self, listener): self._extra["listener"] = listener; return self
        def system_prompt(self, text: str): self._extra["system_prompt"] = text or ""; return self
        def no_system_prompt(self): return self.system_prompt("")
        def default_system_prompt(self): self._extra.pop("system_prompt", None); return self
        def advisors(self, *advisors): self._extra["advisors"] = list(advisors); return self
        def no_advisors(self): self._extra["advisors"] = []; self._extra["advisor_mixer"] = None; return self

        def advisor_note_filter(self, keep: Callable[[str], bool]):
            """Keep-test applied to each advisor's decoded note before mixing (default: non-blank)."""
            if not callable(keep):
                raise TypeError("advisor_note_filter needs a callable")
            self._extra["advisor_note_filter"] = keep
            return self
        def advisor_mixer(self, mixer): self._extra["advisor_mixer"] = mixer; return self
        def think_tags(self, tags): self._extra["think_tags"] = tags; return self

        def build(self) -> "LLM":
            llm = LLM(self._model, EngineConfig(**self._cfg), self._sampling, self._device, self._warmup,
                      unpack_parameters=self._unpack, cpu_threads=self._cpu_threads)
            for k, v in self._extra.items():
                setattr(llm, k, v)
            return llm

    @staticmethod
    def builder(model) -> "LLM.Builder":
        return LLM.Builder(model)

    # ------------------------------------------------------------------ lifecycle
    def warmup(self) -> None:
        ids = [[(i * 7919) % max(2, self.hf.vocab_size - 1) + 1 for i in range(64)]]
        self.generate_token_ids(ids, SamplingParams(max_tokens=16, ignore_eos=True).deterministic())

    def cancel(self) -> None:
        """Stop the running generate at the next step boundary (thread-safe)."""
        self._cancel.set()

    def close(self) -> None:
        if not self._closed:
            self.scheduler.clear()
            if self._plan_tx is not None and not ps.abort_requested():
                self._plan_tx.send_shutdown()  # ends every worker's serve_worker loop
            self.runner.close()
            self._closed = True

    def is_closed(self) -> bool:
        return self._closed

    def chat_specials(self):
        """The model's chat-markup markers (stripped from visible answers)."""
        from .chat.markup import ChatSpecials
        return self.model_handle.chat_specials() if self.model_handle is not None else ChatSpecials.default()

    def _release_and_note(self, seq: Sequence) -> None:
        self.runner.release_state(seq)
        self._plan_tx.note_release(seq)

    @property
    def is_worker(self) -> bool:
        """True on ranks > 0 of a front-door TP engine: they take no requests and run ``serve_worker``."""
        return self._plan_rx is not None

    def serve_worker(self) -> int:
        """Follow rank 0's step plans until it closes its engine (front-door TP, ranks > 0); returns the number of
        steps run.  Raises TensorParallelAbort when a peer failed or this rank's tokens diverged from rank 0's."""
        if self._plan_rx is None:
            raise NanoLlvmException("serve_worker runs on ranks > 0 of an engine built with front_door='rank0'")
        from .engine.plan import KIND_SHUTDOWN
        rx = self._plan_rx
        steps = 0
        try:
            while True:
                ps.check_abort()
                kind, is_prefill, seqs = rx.apply(rx.recv())
                if kind == KIND_SHUTDOWN:
                    return steps
                with nvtx("step:prefill" if is_prefill else "step:decode"):
                    toks = self.runner.run(seqs, is_prefill)
                rx.note_sampled(seqs, toks)
                steps += 1
        except BaseException as e:
            if ps.abort_requested() or ps.peer_aborted(wait_s=2.0 if isinstance(e, torch.distributed.DistError) else 0.0):
                if isinstance(e, TensorParallelAbort):
                    raise
                raise TensorParallelAbort(ps.abort_reason()) from e
            ps.signal_abort(f"{type(e).__name__}: {e}")
            raise
        finally:
            self._closed = True
            self.runner.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # ------------------------------------------------------------------ online API
    def add_request(self, prompt_token_ids: List[int], sampling: Optional[SamplingParams] = None,
                    tag=None) -> Sequence:
        if self._plan_rx is not None:
            raise NanoLlvmException(f"rank {ps.tp_rank()} is a front-door worker: requests go to rank 0, this rank "
                                    "runs serve_worker()")
        sp = self._fit_sampling(len(prompt_token_ids), sampling or self.default_sampling)
        seq = Sequence(prompt_token_ids, sp, self.cfg.kvcache_block_size, user_tag=tag)
        self.scheduler.add(seq)
        return seq

    def abort(self, seq: Sequence) -> bool:
        return self.scheduler.abort(seq.seq_id)

    def has_unfinished(self) -> bool:
        return not self.scheduler.is_finished()

    def step(self, appended_out: Optional[list] = None):
        ps.check_abort()  # a peer rank failed: stop before launching anything that would wait for it
        with nvtx("schedule"):
            try:
                seqs, is_prefill = self.scheduler.schedule()
            except BaseException as e:
                if self._plan_tx is not None:  # front door: the workers wait for a plan that will not come
                    ps.signal_abort(f"rank 0 could not schedule: {type(e).__name__}: {e}")
                raise
        try:
            if self._plan_tx is not None:
                with nvtx("plan"):
                    self._plan_tx.send_step(seqs, is_prefill)
            with nvtx("step:prefill" if is_prefill else "step:decode"):
                toks = self.runner.run(seqs, is_prefill)
        except BaseException as e:
            # a communication error usually means a peer failed first (its connection closed, or the process-group
            # timeout released this rank): give its abort reason a moment to reach the store before blaming itself
            comm = isinstance(e, torch.distributed.DistError)
            if ps.peer_aborted(wait_s=2.0 if comm else 0.0):
                raise TensorParallelAbort(ps.abort_reason()) from e
            ps.signal_abort(f"{type(e).__name__}: {e}")
            raise
        with nvtx("postprocess"):
            finished = self.scheduler.postprocess(seqs, toks, is_prefill, appended_out)
        for s in finished:
            s.t_finish = time.perf_counter()
        return seqs, is_prefill, finished

    def _fit_sampling(self, prompt_len: int, sp: SamplingParams) -> SamplingParams:
        room = self.cfg.max_model_len - prompt_len
        if room <= 0:
            raise ValueError(f"prompt of {prompt_len} tokens leaves no room in max_model_len={self.cfg.max_model_len}")
        if sp.max_tokens > room:
            sp = sp.with_(max_tokens=room)
        return sp

    # ------------------------------------------------------------------ generate family
    def generate_token_ids(self, prompts: Seq[List[int]], sampling: Optional[Union[SamplingParams, Seq[SamplingParams]]] = None,
                           on_token: Optional[Callable[[int, int, int], None]] = None,
                           timeout_s: Optional[float] = None, stats: Optional[GenerationStats] = None
                           ) -> List[GenerationOutput]:
        """Generate for a batch of token-id prompts; ``on_token(prompt_index, seq_id, token)`` streams."""
        if not self._lock.acquire(blocking=False):
            raise NanoLlvmException("another generate call is already running on this engine")
        self._cancel.clear()
        t0 = time.perf_counter()
        deadline = t0 + timeout_s if timeout_s else None
        seqs: List[Sequence] = []
        try:
            for i, p in enumerate(prompts):
                sp = sampling[i] if isinstance(sampling, (list, tuple)) else (sampling or self.default_sampling)
                seqs.append(self.add_request(list(p), sp, tag=i))
            by_id = {s.seq_id: s for s in seqs}
            st = stats if stats is not None else GenerationStats()
            while self.has_unfinished():
                if self._cancel.is_set():
                    raise GenerationCancelledException("generation cancelled")
                if deadline is not None and time.perf_counter() > deadline:
                    raise GenerationTimeoutException(f"generation exceeded {timeout_s}s")
                appended = [] if on_token is not None else None
                _, is_prefill, _ = self.step(appended)
                if is_prefill:
                    st.prefill_steps += 1
                else:
                    st.decode_steps += 1
                if appended:
                    for sid, tok in appended:
                        s = by_id.get(sid)
                        if s is not None:
                            on_token(s.user_tag, sid, tok)
            st.elapsed_s = time.perf_counter() - t0
            st.preemptions = self.scheduler.num_preemptions
            outs = []
            for s in seqs:
                st.prompt_tokens += s.num_prompt_tokens
                st.completion_tokens += s.num_completion_tokens
                ttft = (s.t_first_token - s.t_arrival) if s.t_first_token else None
                if ttft is not None:
                    st.ttft_s.append(ttft)
                if s.t_first_token and s.t_finish and s.num_completion_tokens > 1:
                    st.tpot_s.append((s.t_finish - s.t_first_token) / (s.num_completion_tokens - 1))
                reason = "length" if s.num_completion_tokens >= s.max_tokens else "stop"
                outs.append(GenerationOutput(s.prompt_token_ids, s.completion_token_ids, None, reason, ttft))
            self.last_stats = st
            return outs
        except BaseException:
            self.scheduler.clear()
            raise
        finally:
            self._lock.release()

    def generate(self, prompts: Union[str, Seq[str]], sampling: Optional[SamplingParams] = None,
                 on_token: Optional[Callable] = None, timeout_s: Optional[float] = None) -> List[GenerationOutput]:
        if self.tokenizer is None:
            raise NanoLlvmException("this engine has no tokenizer; use generate_token_ids")
        single = isinstance(prompts, str)
        texts = [prompts] if single else list(prompts)
        ids = [self.tokenizer.encode(t) for t in texts]
        outs = self.generate_token_ids(ids, sampling, on_token, timeout_s)
        for o in outs:
            o.text = self.tokenizer.decode(o.token_ids, skip_special=True)
        return outs

    def complete(self, prompt: str, sampling: Optional[SamplingParams] = None) -> str:
        return self.generate([prompt], sampling)[0].text

    def chat_once(self, user: str, system: Optional[str] = None, sampling: Optional[SamplingParams] = None) -> str:
        from .chat.messages import ChatMessage
        msgs = ([ChatMessage.system(system)] if system else []) + [ChatMessage.user(user)]
        prompt = self.tokenizer.apply_chat_template(msgs, add_generation_prompt=True)
        ids = self.tokenizer.encode(prompt, allow_special=True)
        out = self.generate_token_ids([ids], sampling)[0]
        return self.tokenizer.decode(out.token_ids, skip_special=True)

    # ------------------------------------------------------------------ sessions (LLM.java:1066-1128, 1332-1362)
    def _assert_open(self) -> None:
        if self._closed:
            raise NanoLlvmException("this engine is closed")

    def chat(self, sampling: Optional[Union[SamplingParams, int]] = None, **session_options):
        """A multi-turn ``ChatSession`` on this engine (history, think-tag parsing, streaming events, advisors).
        ``sampling``: a SamplingParams for every turn, or an int = max new tokens per turn with the engine's
        default temperature / top-k / top-p; extra keyword options go to ``ChatSession``."""
        self._assert_open()
        from .chat.session import ChatSession
        if isinstance(sampling, int):
            if sampling < 1:
                raise ValueError("max_tokens must be >= 1")
            sampling = self.default_sampling.with_(max_tokens=sampling)
        return ChatSession(self, sampling=sampling, **session_options)

    def rag(self, index, max_tokens: Optional[int] = None, **session_options):
        """A retrieval-augmented session over ``index`` (BM25 / dense / hybrid): every turn retrieves passages and
        chat-generates from them; thinking is off and grounded turns cap the temperature."""
        self._assert_open()
        if index is None:
            raise ValueError("index must not be None")
        from .rag.session import RagSession
        sp = None
        if max_tokens is not None:
            if max_tokens < 1:
                raise ValueError("max_tokens must be >= 1")
            sp = self.default_sampling.with_(max_tokens=int(max_tokens))
        return RagSession(self, index, sampling=sp, **session_options)

    def run_advisors(self, model_user_text: str, prior_dialog=(), sampling: Optional[SamplingParams] = None):
        """Run this engine's advisors (``LLM.Builder.advisors``) as ONE batched generate over the user text and
        the prior dialog; returns the ``AdvisorEnrichment`` (mixed prompt, per-advisor notes)."""
        self._assert_open()
        if model_user_text is None:
            raise ValueError("model_user_text must not be None")
        from .chat.markup import ThinkTags
        from .chat.session import AdvisorRunner
        return AdvisorRunner.enrich(self, list(self.advisors or []), model_user_text, list(prior_dialog or []),
                                    sampling or self.default_sampling, mixer=self.advisor_mixer,
                                    tags=self.think_tags or ThinkTags(),
                                    note_filter=getattr(self, "advisor_note_filter", None))

    def new_conversation(self):
        """Fresh dialog history: the engine's system prompt as a system turn when it is not blank."""
        self._assert_open()
        from .chat.messages import ChatMessage
        return [ChatMessage.system(self.system_prompt)] if (self.system_prompt or "").strip() else []
