"""LLM inference engine (the reference's engine/llm_engine.py API on the B200 path).

``LLMEngine.from_pretrained(name)`` / ``add_request`` / ``step`` /
``generate`` / ``is_finished`` / ``get_tokens_per_sec`` keep the reference's
contracts (engine/llm_engine.py:146-438).  ``from_model`` builds an engine
around an in-memory HF model (random-init models in tests and benches).

Two modes:

* ``compat`` (default) reproduces the reference engine exactly: one KV pool
  shared by every layer (engine/llm_engine.py:166-193) and no prefill -- a new
  request reserves its prompt slots and only the last prompt token is fed
  (:323-329), so earlier prompt slots are read as whatever the pool holds.
  Greedy tokens then match the reference's.
* ``physical``: one pool per layer and a real prefill of every prompt (and of
  a resumed sequence whose K/V was not swapped), so attention sees the true
  context.  ``swap=True`` also copies preempted blocks to pinned host memory
  and back (the reference's swap moves metadata only).

Per step the decode batch runs every layer with one fused sm_100a attention
kernel; on CUDA the step is a CUDA graph captured per batch bucket
(``engine/decode_graph.py``, ``cuda_graphs=True``), else an eager HF forward.
Greedy sampling of the whole batch is one device argmax and one host copy.

``pipeline=True`` (CUDA graphs of a Llama-family model) takes the host out of
the GPU's critical path.  A sequence finishes only on ``max_tokens`` (the
reference has no other stop rule, core/sequence.py:103-113), so which
sequences run in step k+1, with which slots, is known before step k's token
values are.  ``step()`` therefore schedules and launches step k+1 -- its
input token for a sequence that ran in step k is read on the device from
the ids step k's sampler left there -- and only then waits for step k's ids
and returns step k's outputs.  While the host waits, reads back and
schedules, the GPU already runs the next step.  Scheduling decisions, slots
and tokens are those of the synchronous loop; each ``step()`` returns the
outputs of the step launched by the call before it.
"""

from __future__ import annotations

import logging
import time
from dataclasses import dataclass, field
from types import SimpleNamespace

import torch

from vllm_mps_b200.config import BLOCK_SIZE, MAX_BATCH_SIZE, MAX_TOKENS_PER_STEP, NUM_CPU_BLOCKS, NUM_GPU_BLOCKS
from vllm_mps_b200.core.kv_cache_manager import KVCacheManager
from vllm_mps_b200.core.model_config import ModelConfig
from vllm_mps_b200.core.sequence import SamplingParams, Sequence, SequenceGroup, SequenceStatus
from vllm_mps_b200.engine.scheduler import Scheduler
from vllm_mps_b200.memory.cuda_memory_pool import CUDAMemoryPool, SwapSpace
from vllm_mps_b200.model.sampler import Sampler

logger = logging.getLogger(__name__)


@dataclass
class RequestOutput:
    """State of one request (engine/llm_engine.py:45-63)."""

    request_id: int
    prompt: str
    generated_text: str = ""
    token_ids: list[int] = field(default_factory=list)
    finished: bool = False
    num_steps: int = 0


class LLMEngine:
    """Scheduler + paged KV cache + HF model with paged attention layers."""

    def __init__(self) -> None:
        raise TypeError("use LLMEngine.from_pretrained(...) or LLMEngine.from_model(...)")

    # ── construction ─────────────────────────────────────────────────────────

    @classmethod
    def from_pretrained(cls, model_name: str, sampling_params: SamplingParams | None = None,
                        **kwargs) -> "LLMEngine":
        """Load a HF model (hub name or local directory) and build the engine (:146-205)."""
        from transformers import AutoModelForCausalLM, AutoTokenizer

        cfg = ModelConfig.from_pretrained(model_name)
        hf = AutoModelForCausalLM.from_pretrained(model_name, torch_dtype=cfg.dtype)
        try:
            tok = AutoTokenizer.from_pretrained(model_name)
        except Exception:  # tokenizer files are optional
            tok = None
        return cls.from_model(hf, model_config=cfg, tokenizer=tok, model_name=model_name, **kwargs)

    @classmethod
    def from_model(cls, hf_model, model_config: ModelConfig | None = None, tokenizer=None,
                   model_name: str = "model", num_gpu_blocks: int = NUM_GPU_BLOCKS,
                   num_cpu_blocks: int = NUM_CPU_BLOCKS, max_batch_size: int = MAX_BATCH_SIZE,
                   max_tokens_per_step: int = MAX_TOKENS_PER_STEP, mode: str = "compat",
                   swap: bool = False, preempt_watermark: float | None = None,
                   dtype: torch.dtype | None = None,
                   device: torch.device | str | None = None,
                   max_prefill_rows: int = 8192, cuda_graphs: bool = True,
                   pipeline: bool = False) -> "LLMEngine":
        from vllm_mps_b200.models.llama_adapter import LlamaAdapter

        if mode not in ("compat", "physical"):
            raise ValueError(f"mode must be 'compat' or 'physical', got {mode!r}")
        cfg = model_config or ModelConfig.from_hf_config(hf_model.config, model_name, dtype, device)
        if dtype is not None:
            cfg.dtype = dtype
        if device is not None:
            cfg.device = torch.device(device)
        pool = CUDAMemoryPool(num_gpu_blocks, BLOCK_SIZE, cfg.n_kv_heads, cfg.d_k, cfg.dtype,
                              cfg.device, num_layers=cfg.n_layers if mode == "physical" else None)
        swap_space = SwapSpace(pool, num_cpu_blocks) if swap else None
        kv = KVCacheManager(num_gpu_blocks, num_cpu_blocks, swap_space=swap_space)

        eng = cls.__new__(cls)
        eng.mode = mode
        eng.model_config = cfg
        eng.memory_pool = pool
        eng.kv_cache_manager = kv
        eng.scheduler = Scheduler(kv, max_batch_size, max_tokens_per_step, preempt_watermark)
        eng.sampler = Sampler()
        eng.adapter = LlamaAdapter(model_name)
        eng.adapter.attach(hf_model, cfg, kv, pool, tokenizer)
        eng.tokenizer = tokenizer
        eng._request_counter = 0
        eng._outputs: dict[int, RequestOutput] = {}
        eng._seq_to_request: dict[int, int] = {}
        eng._seq_to_params: dict[int, SamplingParams] = {}
        eng._seqs: dict[int, Sequence] = {}
        eng._prefilled: set[int] = set()
        if max_prefill_rows < 1:
            raise ValueError("max_prefill_rows must be >= 1")
        eng.max_prefill_rows = int(max_prefill_rows)
        eng._graphs = None
        if cuda_graphs and cfg.device.type == "cuda":
            from vllm_mps_b200.engine.decode_graph import DecodeGraphRunner

            max_blocks = (max(cfg.max_seq_len, 1) + BLOCK_SIZE - 1) // BLOCK_SIZE + 1
            eng._graphs = DecodeGraphRunner(eng.adapter, kv, BLOCK_SIZE, max_blocks)
        eng.pipeline = bool(pipeline)
        eng._inflight = None
        if eng.pipeline:
            if eng._graphs is None or not eng._graphs.fused:
                raise ValueError("pipeline=True needs CUDA graphs of a Llama-family model")
            # Two pinned landing buffers for the sampled ids, used in turn.
            eng._ids_host = [torch.zeros(len(eng._graphs.prev_tokens), dtype=torch.long)
                             .pin_memory() for _ in range(2)]
            eng._ids_ready = [torch.cuda.Event() for _ in range(2)]
            eng._ids_turn = 0
        eng.total_tokens_generated = 0
        eng.start_time = time.time()
        return eng

    def warm_prefill_gemms(self) -> int:
        """Startup work for a serving run: meet every prefill GEMM shape up to
        ``max_prefill_rows`` once (fused Llama path; returns how many row
        counts, 0 when there is nothing to warm)."""
        if self._graphs is None:
            return 0
        return self._graphs.warm_prefill_gemms(self.max_prefill_rows)

    def capture_decode_graphs(self) -> list[int]:
        """Capture the decode step's CUDA graph for every batch bucket up to
        ``max_batch_size`` now instead of on first use; returns the buckets."""
        if self._graphs is None:
            return []
        return self._graphs.capture_all(self.scheduler.max_batch_size)

    # ── requests ─────────────────────────────────────────────────────────────

    def add_request(self, prompt: str | list[int], sampling_params: SamplingParams | None = None) -> int:
        """Queue a request (text, or a list of token ids); returns its id (:247-282)."""
        if sampling_params is None:
            sampling_params = SamplingParams()
        request_id = self._request_counter
        self._request_counter += 1
        if isinstance(prompt, str):
            if self.tokenizer is None:
                raise ValueError("text prompt given but the engine has no tokenizer")
            token_ids, text = self.tokenizer.encode(prompt), prompt
        else:
            token_ids, text = [int(t) for t in prompt], ""
        seq = Sequence(request_id, text, token_ids, sampling_params)
        self.scheduler.add_request(SequenceGroup(request_id, [seq], sampling_params))
        self._outputs[request_id] = RequestOutput(request_id=request_id, prompt=text)
        self._seq_to_request[request_id] = request_id
        self._seq_to_params[request_id] = sampling_params
        self._seqs[request_id] = seq
        return request_id

    # ── stepping ─────────────────────────────────────────────────────────────

    def step(self) -> list[RequestOutput]:
        """One scheduling + decode step over every running sequence (:286-346).

        With ``pipeline=True`` this launches the next step and returns the
        outputs of the one launched before it (module docstring)."""
        if self.pipeline:
            return self._step_pipelined()
        seqs = self._schedule()
        if not seqs:
            return []
        seq_ids = [s.seq_id for s in seqs]
        token_ids = [s.get_last_token_id() for s in seqs]
        positions = [s.get_total_len() - 1 for s in seqs]
        seq_lens = [s.get_total_len() for s in seqs]
        if self._graphs is not None and self._graphs.can_run(seq_ids):
            logits = self._graphs.run(token_ids, seq_ids, positions, seq_lens)
        else:
            logits = self.adapter.forward_batch(token_ids, seq_ids, positions, seq_lens)
        next_tokens = self.sampler.sample_rows(
            logits, [self._seq_to_params.get(sid, SamplingParams()) for sid in seq_ids])
        return self._update_sequences(seq_ids, next_tokens)

    def _step_pipelined(self) -> list[RequestOutput]:
        seqs = self._schedule()
        if not seqs:
            return self._resolve()
        seq_ids = [s.seq_id for s in seqs]
        positions = [s.get_total_len() - 1 for s in seqs]
        seq_lens = [s.get_total_len() for s in seqs]
        params = [self._seq_to_params.get(sid, SamplingParams()) for sid in seq_ids]
        g = self._graphs
        if not g.can_run(seq_ids):
            # The eager forward takes host token ids: settle the step in flight
            # first.  This step's ids are then known at once, but they are
            # still reported by the next call, so that every call returns one
            # step (a RequestOutput is updated in place: two steps of one
            # request in one return would both show the later token).
            done = self._resolve()
            token_ids = [s.get_last_token_id() for s in seqs]
            logits = self.adapter.forward_batch(token_ids, seq_ids, positions, seq_lens)
            ids = self.sampler.sample_rows(logits, params)
            self._inflight = self._book(seqs, ids, rows={}, host=None, ready=None)
            return done
        # A sequence of the step in flight has a placeholder as its last token;
        # its input is that step's sampled id, at the row it had there.
        rows = self._inflight.rows if self._inflight is not None else {}
        src = [rows.get(sid, -1) for sid in seq_ids]
        token_ids = [0 if r >= 0 else s.token_ids[-1] for s, r in zip(seqs, src)]
        logits = g.run(token_ids, seq_ids, positions, seq_lens, src=src)
        B = len(seqs)
        ids = g.prev_tokens[:B]
        self.sampler.sample_rows_device(logits, params, out=ids)
        j = self._ids_turn
        self._ids_turn ^= 1
        self._ids_host[j][:B].copy_(ids, non_blocking=True)
        self._ids_ready[j].record()
        # Book the step now with placeholder ids (lengths and finishes do not
        # depend on the values), so the next schedule sees the same state as
        # after a synchronous step.
        launched = self._book(seqs, [-1] * B, rows={sid: i for i, sid in enumerate(seq_ids)},
                              host=self._ids_host[j], ready=self._ids_ready[j])
        done = self._resolve()
        self._inflight = launched
        return done

    def _book(self, seqs, ids, rows, host, ready) -> SimpleNamespace:
        """Append one id per sequence (placeholders when ``host`` is given) and
        retire the sequences that reach ``max_tokens``; the step's record."""
        booked = []
        for s, t in zip(seqs, ids):
            booked.append((s, len(s.token_ids)))
            s.add_token(t)
            if s.is_finished():
                self._retire(s.seq_id)
        return SimpleNamespace(booked=booked, rows=rows, host=host, ready=ready,
                               ids=None if host is not None else list(ids))

    def _resolve(self) -> list[RequestOutput]:
        """Wait for the step in flight's ids, write them over its placeholders."""
        fl = self._inflight
        if fl is None:
            return []
        self._inflight = None
        if fl.ids is not None:
            ids = fl.ids
        else:
            fl.ready.synchronize()
            ids = fl.host[:len(fl.booked)].numpy().tolist()
        updated = []
        for (seq, at), token_id in zip(fl.booked, ids):
            seq.token_ids[at] = token_id
            self.total_tokens_generated += 1
            request_id = self._seq_to_request.get(seq.seq_id)
            if request_id is None:
                continue
            out = self._outputs[request_id]
            out.token_ids.append(token_id)
            if self.tokenizer is not None:
                out.generated_text = self.tokenizer.decode(seq.token_ids[seq.prompt_len:at + 1],
                                                           skip_special_tokens=True)
            out.finished = at + 1 - seq.prompt_len >= seq.sampling_params.max_tokens
            out.num_steps += 1
            updated.append(out)
        return updated

    def _retire(self, seq_id: int) -> None:
        self.scheduler.mark_finished(seq_id)
        self._prefilled.discard(seq_id)
        for pl in self.adapter.paged_layers:
            pl.evict_sequence(seq_id)

    def _schedule(self) -> list[Sequence]:
        """Schedule a step; give every sequence its slots; prefill what needs it."""
        sched_out = self.scheduler.schedule()
        for group in sched_out.preempted_groups:
            for s in group.sequences:
                if self.kv_cache_manager.swap_space is None:
                    self._prefilled.discard(s.seq_id)  # its K/V is gone
        if not sched_out.scheduled_groups:
            return []
        seqs = [s for g in sched_out.scheduled_groups for s in g.get_seqs(SequenceStatus.RUNNING)]
        if not seqs:
            return []
        # A sequence resumed from preemption gets its old slots back but no
        # slot for the token it processes now: the reference scheduler appends
        # only for groups that were already running (engine/scheduler.py:98-125,
        # 189-196), and its engine then writes that token past the block
        # table's count (an IndexError at a page boundary, mps_memory_pool.py:257-268).
        # Give every scheduled sequence a slot for each of its tokens.
        kv = self.kv_cache_manager
        for s in seqs:
            short = s.get_total_len() - kv.num_tokens(s.seq_id)
            if short > 0:
                kv.append_slots(s.seq_id, short)
        if self.mode == "physical":
            self._prefill([s for s in seqs if s.seq_id not in self._prefilled])
        return seqs

    def _prefill(self, seqs: list[Sequence]) -> None:
        """Write the K/V of every token but the last of each sequence, all layers.

        The prompt rows go through the model in chunks of at most
        ``max_prefill_rows`` rows (a longer sequence is split, later pieces
        attending to the earlier ones through the pool).  Per layer, kernel 1
        writes every row's rotated K and V, then kernel 3 (tcgen05 causal
        prefill) computes each row against its sequence's slots
        ``0..position``.  With the CUDA-graph runner's fused Llama layers the
        chunk runs through ``DecodeGraphRunner.prefill_rows`` (no HF forward),
        else through the HF model with the paged attention layers.
        """
        pieces, rows = [], 0
        for s in seqs:
            self._prefilled.add(s.seq_id)
            n = len(s.token_ids) - 1
            start = 0
            while start < n:
                take = min(n - start, self.max_prefill_rows - rows)
                pieces.append((s, start, take))
                rows += take
                start += take
                if rows == self.max_prefill_rows:
                    self._prefill_chunk(pieces)
                    pieces, rows = [], 0
        if pieces:
            self._prefill_chunk(pieces)

    def _prefill_chunk(self, pieces) -> None:
        from vllm_mps_b200.models import llama_adapter as la

        dev = self.model_config.device
        meta = la.build_prefill_metadata(self.kv_cache_manager,
                                         [(s.seq_id, qs, ql) for s, qs, ql in pieces],
                                         BLOCK_SIZE, dev)
        toks = [t for s, qs, ql in pieces for t in s.token_ids[qs:qs + ql]]
        if self._graphs is not None and self._graphs.fused:
            toks += [0] * (self._graphs.padded_rows(len(toks)) - len(toks))
            tok = torch.tensor(toks, dtype=torch.int32).pin_memory()
            with torch.no_grad():
                self._graphs.prefill_rows(tok.to(dev, non_blocking=True), meta)
            return
        tok = torch.tensor(toks, dtype=torch.long)
        if dev.type == "cuda":
            tok = tok.pin_memory()
        embeds = self.adapter.hf_model.model.embed_tokens(tok.to(dev, non_blocking=True)).unsqueeze(1)
        ctx = la._batch_context
        ctx.is_batch = True
        ctx.prefill = True
        ctx.prefill_meta = meta
        try:
            with torch.no_grad():
                self.adapter.hf_model.model(inputs_embeds=embeds, use_cache=False)
        finally:
            ctx.is_batch = False
            ctx.prefill = False
            ctx.prefill_meta = None

    def _update_sequences(self, seq_ids: list[int], next_tokens: list[int]) -> list[RequestOutput]:
        updated = []
        for seq_id, token_id in zip(seq_ids, next_tokens):
            request_id = self._seq_to_request.get(seq_id)
            seq = self._seqs.get(seq_id)
            if request_id is None or seq is None:
                continue
            seq.add_token(token_id)
            self.total_tokens_generated += 1
            if seq.is_finished():
                self._retire(seq_id)
            out = self._outputs[request_id]
            out.token_ids.append(token_id)  # mirrors seq.output_token_ids
            if self.tokenizer is not None:
                out.generated_text = self.tokenizer.decode(seq.output_token_ids,
                                                           skip_special_tokens=True)
            out.finished = seq.is_finished()
            out.num_steps += 1
            updated.append(out)
        return updated

    def generate(self, prompt: str | list[int], max_tokens: int = 50,
                 temperature: float = 1.0) -> str | list[int]:
        """Run one request to completion; text if a tokenizer is present, else ids (:387-417)."""
        req = self.add_request(prompt, SamplingParams(max_tokens=max_tokens, temperature=temperature))
        while not self._outputs[req].finished:
            self.step()
        out = self._outputs[req]
        return out.generated_text if self.tokenizer is not None else list(out.token_ids)

    def get_output(self, request_id: int) -> RequestOutput:
        return self._outputs[request_id]

    # ── queries ──────────────────────────────────────────────────────────────

    def is_finished(self) -> bool:
        return (self.scheduler.get_num_waiting() == 0 and self.scheduler.get_num_running() == 0
                and self.scheduler.get_num_preempted() == 0 and self._inflight is None)

    def get_elapsed(self) -> float:
        return time.time() - self.start_time

    def get_tokens_per_sec(self) -> float:
        elapsed = self.get_elapsed()
        return 0.0 if elapsed == 0 else self.total_tokens_generated / elapsed
