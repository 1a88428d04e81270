"""Continuous batching: drop-in for the reference's ``GenerationRequest`` / ``ContinuousBatcher``
(engine/scheduler.py:11-281).

Public surface kept: ``ContinuousBatcher(model, kv_cache, eos_token_id=None)`` with
``async generate_stream(prompt_tokens, max_new_tokens, temperature=0.7, p_value=0.9,
top_k=20)`` (yields ints; a request's error is re-raised in its consumer), ``async generate``,
``async run_loop``, the ``requests_queue`` / ``active_slots`` / ``cos_cache`` / ``sin_cache``
attributes and the tick: fill free slots lowest-first from the queue (:159-167); prefill every
new request (:190-196), then one batched decode step over all prefilled slots, in slot order
(:199-206); a request finishes on EOS or ``max_new_tokens`` (:240-245, :276-281) and its slot's
blocks go back to the pool (:208-217); errors finish the affected requests (:193-206).

What changes is underneath, in the backend (:class:`EngineBackend`): the tick's prefills run
as one packed ragged forward (blocks still allocated request by request, in the reference's
order, so a failing request fails alone); decode is one CUDA-graph replay of
``engine.DecodeEngine`` (argmax in the lm_head epilogue when every row is greedy, else logits
plus the device sampler); sampling uses each request's own Philox stream
(``sampler.sample_next_token``).  A backend only has to provide ``prefill(slots, requests)`` and
``decode(slots, requests)``; tests drive the scheduler with a host-only stand-in.

Observability (no counterpart in the reference, which only prints): ``stats()`` returns host-side
counters of the serving loop -- ticks, prompt tokens prefilled, tokens emitted, finished and
failed requests, the last and mean tick time and the KV pool's occupancy -- kept with a clock
read per tick and no device synchronisation; with ``TI_NVTX=1`` each tick's prefill and decode
phases are NVTX ranges (``tick.prefill`` / ``tick.decode``) for Nsight timelines.
"""
from __future__ import annotations

import asyncio
import contextlib
import logging
import os
import time
from dataclasses import dataclass
from typing import AsyncGenerator, List, Optional

import numpy as np
import torch

log = logging.getLogger(__name__)

_END_OF_STREAM = object()   # sentinel closing a request's token stream


@dataclass
class SchedulerStats:
    """Host-side counters of a ContinuousBatcher (see ``ContinuousBatcher.stats``)."""
    ticks: int = 0
    prefill_tokens: int = 0        # prompt tokens prefilled (chunks included)
    emitted_tokens: int = 0        # tokens handed to consumers (prefill's first + decode)
    decode_steps: int = 0
    requests_finished: int = 0
    requests_failed: int = 0
    last_tick_s: float = 0.0
    total_tick_s: float = 0.0


def _nvtx_range(name: str):
    """An NVTX range when TI_NVTX=1 (read per call: cheap, and settable at run time)."""
    if os.environ.get("TI_NVTX") == "1":
        return torch.cuda.nvtx.range(name)
    return contextlib.nullcontext()


class GenerationRequest:
    """One generation request (engine/scheduler.py:11-22), plus the request's random stream."""

    _next_id = 0

    def __init__(self, prompt_tokens: List[int], max_new_tokens: int, temperature: float = 0.7,
                 p_value: float = 0.9, top_k: int = 20, seed: Optional[int] = None):
        self.prompt_tokens = prompt_tokens
        self.max_new_tokens = max_new_tokens
        self.temperature = temperature
        self.p_value = p_value
        self.top_k = top_k
        self.generated_tokens: List[int] = []
        self.token_queue: asyncio.Queue = asyncio.Queue()
        self.completion_event = asyncio.Event()
        self.error: Optional[BaseException] = None
        self.is_prefilled = False
        self.prefill_pos = 0      # prompt tokens already in the KV cache (chunked prefill)
        self.request_id = GenerationRequest._next_id
        GenerationRequest._next_id += 1
        s = self.request_id if seed is None else seed
        self.rng = np.random.Generator(np.random.Philox(key=int(s)))


class ContinuousBatcher:
    def __init__(self, model, kv_cache, eos_token_id: Optional[int] = None, *, backend=None,
                 prefill_chunk_tokens: Optional[int] = None):
        """``prefill_chunk_tokens``: at most this many prompt tokens are prefilled per tick
        (chunked prefill interleaved with decode; a request's first token is emitted after its
        last chunk).  None: whole prompts every tick, as the reference (block tables then match
        the reference's bit for bit; with chunking the allocation order interleaves with decode).
        """
        self.model = model
        self.prefill_chunk_tokens = prefill_chunk_tokens
        self.kv_cache = kv_cache
        self.requests_queue: asyncio.Queue = asyncio.Queue()
        self.max_batch_size = kv_cache.max_batch_size
        self.active_slots: List[Optional[GenerationRequest]] = [None] * self.max_batch_size
        self.device = kv_cache.device
        self.cos_cache, self.sin_cache = self._init_rope_cache()
        self.eos_token_id = eos_token_id
        self.backend = backend if backend is not None else EngineBackend(
            model, kv_cache, self.cos_cache, self.sin_cache)
        self._stats = SchedulerStats()

    def stats(self) -> dict:
        """Counters of the serving loop so far, plus the KV pool's occupancy (blocks held by
        sequences / all blocks) and the number of occupied slots."""
        st = self._stats
        d = dict(st.__dict__)
        d["mean_tick_s"] = st.total_tick_s / st.ticks if st.ticks else 0.0
        alloc = getattr(self.kv_cache, "alloc", None)
        if alloc is not None:
            total = int(alloc.total_physical_blocks)
            d["pool_blocks"] = total
            d["pool_occupancy"] = (total - len(alloc.free_blocks)) / total if total else 0.0
        d["active_slots"] = sum(r is not None for r in self.active_slots)
        return d

    def _init_rope_cache(self):
        """cos/sin [max_seq_len, head_dim/2] float32 with base 1e6 (engine/scheduler.py:36-48)."""
        max_seq_len = self.kv_cache.max_seq_len
        head_dim = self.kv_cache.head_dim
        inv_freq = 1.0 / (1000000.0 ** (torch.arange(0, head_dim, 2, device=self.device).float()
                                        / head_dim))
        t = torch.arange(max_seq_len, device=self.device, dtype=torch.float32)
        freqs = torch.einsum("i,j->ij", t, inv_freq)
        return freqs.cos().to(torch.float32), freqs.sin().to(torch.float32)

    # ---- request side ---------------------------------------------------------------------
    async def generate_stream(self, prompt_tokens: List[int], max_new_tokens: int,
                              temperature: float = 0.7, p_value: float = 0.9,
                              top_k: int = 20) -> AsyncGenerator[int, None]:
        if len(prompt_tokens) >= self.kv_cache.max_seq_len:                    # :59-64
            raise ValueError(
                f"Prompt length ({len(prompt_tokens)}) exceeds or matches maximum "
                f"allowed sequence length ({self.kv_cache.max_seq_len}).")
        request = GenerationRequest(prompt_tokens, max_new_tokens, temperature, p_value, top_k)
        await self.requests_queue.put(request)
        while True:
            next_token = await request.token_queue.get()
            if next_token is _END_OF_STREAM:
                if request.error is not None:
                    raise request.error
                break
            yield next_token

    async def generate(self, prompt_tokens: List[int], max_new_tokens: int,
                       temperature: float = 0.7, p_value: float = 0.9,
                       top_k: int = 20) -> List[int]:
        tokens = []
        async for token in self.generate_stream(prompt_tokens, max_new_tokens, temperature,
                                                p_value, top_k):
            tokens.append(token)
        return tokens

    async def run_loop(self):
        """The scheduler loop (engine/scheduler.py:89-103)."""
        log.info("continuous batcher started")
        while True:
            self._fill_active_slots()
            if self._has_active_requests():
                self._step_generation()
            else:
                await asyncio.sleep(0.01)
            await asyncio.sleep(0)

    # ---- tick -------------------------------------------------------------------------------
    def _sample_next_token(self, logits: torch.Tensor, requests: List[GenerationRequest]) -> List[int]:
        """engine/scheduler.py:104-156 (device sampler; ``requests`` form one batch)."""
        from . import sampler
        return sampler.sample_next_token(logits, requests)

    def _fill_active_slots(self):
        for i in range(self.max_batch_size):
            if self.active_slots[i] is None and not self.requests_queue.empty():
                self.active_slots[i] = self.requests_queue.get_nowait()
                log.debug("assigned request to cache slot %d", i)

    def _has_active_requests(self) -> bool:
        return any(req is not None for req in self.active_slots)

    def _step_generation(self):
        t0 = time.perf_counter()
        prefill_indices, decode_indices = [], []
        for slot_idx, req in enumerate(self.active_slots):
            if req is not None:
                (decode_indices if req.is_prefilled else prefill_indices).append(slot_idx)
        if prefill_indices:
            with _nvtx_range("tick.prefill"):
                self._execute_prefill_batch(prefill_indices)
        if decode_indices:
            try:
                with _nvtx_range("tick.decode"):
                    self._execute_decode(decode_indices)
            except Exception as e:   # noqa: BLE001 - the reference fails the whole decode batch
                for slot_idx in decode_indices:
                    self._finish_request(slot_idx, reason="Error during decode", error=e)
        st = self._stats
        st.ticks += 1
        st.last_tick_s = time.perf_counter() - t0
        st.total_tick_s += st.last_tick_s

    def _finish_request(self, slot_idx: int, reason: str, error: Optional[BaseException] = None):
        req = self.active_slots[slot_idx]
        if req is None:
            return
        req.error = error
        req.completion_event.set()
        req.token_queue.put_nowait(_END_OF_STREAM)
        self.kv_cache.free_batch_slot(slot_idx)
        self.active_slots[slot_idx] = None
        if error:
            self._stats.requests_failed += 1
            log.warning("slot %d request terminated due to error: %s", slot_idx, error)
        else:
            self._stats.requests_finished += 1
            log.debug("slot %d request completed: %s", slot_idx, reason)

    def _emit(self, slot_idx: int, token: int, phase: str) -> None:
        req = self.active_slots[slot_idx]
        req.generated_tokens.append(token)
        req.token_queue.put_nowait(token)
        self._stats.emitted_tokens += 1
        hit_eos = self.eos_token_id is not None and token == self.eos_token_id
        hit_max = len(req.generated_tokens) >= req.max_new_tokens
        if hit_eos or hit_max:
            why = "EOS Token" if hit_eos else "Max Tokens"
            self._finish_request(slot_idx, reason=f"{phase} ({why})" if phase else why)
        elif phase:
            req.is_prefilled = True

    def _execute_prefill_batch(self, slots: List[int]):
        """Prefill each new request (engine/scheduler.py:224-248); a request whose prefill fails
        finishes with its error, the others go on.  With ``prefill_chunk_tokens`` the tick's
        prompt tokens are capped and a request may take several ticks."""
        budget = self.prefill_chunk_tokens
        run, counts = [], []
        for s in slots:
            req = self.active_slots[s]
            left = len(req.prompt_tokens) - req.prefill_pos
            n = left if budget is None else min(left, budget)
            if n <= 0:
                break
            run.append(s)
            counts.append(n)
            if budget is not None:
                budget -= n
                if budget == 0:
                    break
        if not run:
            return
        reqs = [self.active_slots[s] for s in run]
        results = self.backend.prefill(run, reqs, counts)
        for slot_idx, req, n, res in zip(run, reqs, counts, results):
            if isinstance(res, BaseException):
                self._finish_request(slot_idx, reason="Error during prefill", error=res)
                continue
            req.prefill_pos += n
            self._stats.prefill_tokens += n
            if req.prefill_pos >= len(req.prompt_tokens):
                self._emit(slot_idx, int(res), "prefill")

    def _execute_decode(self, decode_indices: List[int]):
        """One batched decode step (engine/scheduler.py:250-281)."""
        reqs = [self.active_slots[s] for s in decode_indices]
        tokens = self.backend.decode(decode_indices, reqs)
        self._stats.decode_steps += 1
        for slot_idx, tok in zip(decode_indices, tokens):
            self._emit(slot_idx, int(tok), "")


class EngineBackend:
    """GPU backend of the scheduler: packed prefill through ``Qwen2ForCausalLM.forward_packed``,
    graph-captured decode through ``engine.DecodeEngine``, device sampling."""

    def __init__(self, model, kv_cache, cos, sin):
        from .engine import DecodeEngine
        self.model, self.kv = model, kv_cache
        self.cos = cos.to(model.device, torch.float32).contiguous()
        self.sin = sin.to(model.device, torch.float32).contiguous()
        self.engine = DecodeEngine(model, kv_cache)

    @staticmethod
    def _params(reqs, vocab):
        from .sampler import SamplingParams, request_uniforms
        return SamplingParams([r.temperature for r in reqs], [r.top_k for r in reqs],
                              [r.p_value for r in reqs], request_uniforms(reqs), vocab)

    def prefill(self, slots, reqs, counts=None):
        """Prefill ``counts[i]`` more prompt tokens of each request (default: the whole rest).
        Plans each request's blocks (reference order; failures stay per request), runs the
        successful ones as one packed forward, advances their lengths and samples each request
        whose prompt is complete as its own batch (the reference samples a prefill alone)."""
        from . import sampler
        from .sampler import SamplingParams
        if counts is None:
            counts = [len(r.prompt_tokens) - r.prefill_pos for r in reqs]
        out: list = [None] * len(slots)
        ok, maps = [], []
        kv, m = self.kv, self.model
        for i, (slot, n) in enumerate(zip(slots, counts)):
            try:
                mapping, _ = kv.plan_tokens([slot], [n])
                ok.append(i)
                maps.append(mapping)
            except (ValueError, RuntimeError) as e:
                out[i] = e
        if not ok:
            return out
        try:
            chunk = [np.asarray(reqs[i].prompt_tokens[reqs[i].prefill_pos:reqs[i].prefill_pos +
                                                      counts[i]], np.int32) for i in ok]
            pb = m.packed_batch(kv, [slots[i] for i in ok], [counts[i] for i in ok],
                                np.concatenate(chunk), np.concatenate(maps))
            logits = m.forward_packed(pb, kv, self.cos, self.sin, rows="last")
            kv.advance_device([slots[i] for i in ok], [counts[i] for i in ok])
            done = [j for j, i in enumerate(ok)
                    if reqs[i].prefill_pos + counts[i] >= len(reqs[i].prompt_tokens)]
            if not done:
                return out
            logits = logits[done] if len(done) < len(ok) else logits
            ok = [ok[j] for j in done]
            V = logits.shape[-1]
            sp = SamplingParams.concat([self._params([reqs[i]], V) for i in ok])
            pd = torch.from_numpy(sp.packed()).to(logits.device)
            toks = torch.empty(len(ok), dtype=torch.int32, device=logits.device)
            sampler.launch_sample(logits, pd, toks)
            for j, t in zip(ok, toks.cpu().tolist()):
                out[j] = int(t)
        except Exception as e:   # noqa: BLE001 - every request of the failed pack gets the error
            for j in ok:
                out[j] = e
        return out

    def decode(self, slots, reqs):
        vocab = self.model.config.vocab_size
        params = self._params(reqs, vocab)
        tokens = [r.generated_tokens[-1] for r in reqs]
        return [int(t) for t in self.engine.step(slots, tokens, None if params.all_greedy
                                                 else params)]
