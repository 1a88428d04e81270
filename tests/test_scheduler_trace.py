"""The continuous-batching scheduler against the reference's own trace (CPU).

tests/golden/scheduler_trace.json was recorded by driving the reference's ContinuousBatcher
(engine/scheduler.py:159-281) with staggered arrivals, greedy requests, an EOS id and a
deterministic stand-in model (next token = (7 * last + 3 * position + 1) % vocab) over the
reference KVCacheManager.  Here the same arrivals drive tiny_infra_b200.scheduler with a
host-only backend that computes the same stand-in tokens on top of the library's
BlockAllocator; every tick must match: slot assignment, emitted tokens (and stream ends),
block tables, sequence lengths and the free list.
"""
import asyncio
import json
import os

import numpy as np
import torch

from tiny_infra_b200.cache_manager import BlockAllocator
from tiny_infra_b200.scheduler import _END_OF_STREAM, ContinuousBatcher, GenerationRequest

HERE = os.path.dirname(os.path.abspath(__file__))


class _HostKV:
    """The attributes the scheduler reads from a KV cache, over a BlockAllocator."""

    def __init__(self, c):
        self.alloc = BlockAllocator(c["max_batch_size"], c["max_seq_len"], c["block_size"])
        self.max_batch_size = c["max_batch_size"]
        self.max_seq_len = c["max_seq_len"]
        self.head_dim = c["head_dim"]
        self.device = torch.device("cpu")

    def free_batch_slot(self, slot):
        self.alloc.free_slot(slot)


class _StandInBackend:
    """The trace's stand-in model: allocation exactly as a forward over the KV manager, then
    the deterministic next token of the last input token and its position."""

    def __init__(self, kv, vocab):
        self.kv, self.vocab = kv, vocab

    def _next(self, last, pos):
        return (last * 7 + pos * 3 + 1) % self.vocab

    def prefill(self, slots, reqs, counts):
        out = []
        for slot, req, S in zip(slots, reqs, counts):
            start = int(self.kv.alloc.seq_len[slot])
            try:
                self.kv.alloc.plan_tokens([slot], [S])
            except (ValueError, RuntimeError) as e:
                out.append(e)
                continue
            self.kv.alloc.advance([slot], S)
            last = req.prompt_tokens[req.prefill_pos + S - 1]
            out.append(self._next(last, start + S - 1))
        return out

    def decode(self, slots, reqs):
        pos = [int(self.kv.alloc.seq_len[s]) for s in slots]
        self.kv.alloc.plan_decode(slots)          # raises for the whole batch, as the reference
        self.kv.alloc.advance(slots, 1)
        return [self._next(r.generated_tokens[-1], p) for r, p in zip(reqs, pos)]


def test_scheduler_matches_reference_trace():
    g = json.load(open(os.path.join(HERE, "golden", "scheduler_trace.json")))
    kv = _HostKV(g["cache"])
    sched = ContinuousBatcher(None, kv, eos_token_id=g["eos"],
                              backend=_StandInBackend(kv, g["vocab"]))
    arrivals = {int(k): v for k, v in g["arrivals"].items()}
    specs = iter(g["requests"])
    requests = []

    async def drive():
        for rec in g["steps"]:
            step = rec["step"]
            for _ in range(arrivals.get(step, 0)):
                spec = next(specs)
                req = GenerationRequest(spec["prompt"], spec["max_new_tokens"], temperature=0.0,
                                        p_value=0.9, top_k=20)
                requests.append(req)
                await sched.requests_queue.put(req)
            sched._fill_active_slots()
            slots = [requests.index(r) if r is not None else None for r in sched.active_slots]
            assert slots == rec["slots"], step
            if sched._has_active_requests():
                sched._step_generation()
            emitted = {}
            for ri, r in enumerate(requests):
                toks = []
                while not r.token_queue.empty():
                    t = r.token_queue.get_nowait()
                    toks.append("END" if t is _END_OF_STREAM else int(t))
                if toks:
                    emitted[str(ri)] = toks
            assert emitted == rec["emitted"], step
            assert kv.alloc.block_tables.tolist() == rec["block_tables"], step
            assert kv.alloc.seq_len.tolist() == rec["seq_len"], step
            assert list(kv.alloc.free_blocks) == rec["free_blocks"], step

    asyncio.run(drive())
    assert [r.generated_tokens for r in requests] == g["final"]
    # the serving counters agree with the trace
    st = sched.stats()
    assert st["emitted_tokens"] == sum(len(t) for t in g["final"])
    assert st["requests_finished"] + st["requests_failed"] == len(requests)
    assert st["prefill_tokens"] == sum(len(r.prompt_tokens) for r in requests
                                       if r.generated_tokens or r.error is None)
    assert st["ticks"] >= st["decode_steps"] > 0 and st["mean_tick_s"] > 0.0
    used = sum(1 for row in kv.alloc.block_tables.tolist() for b in row if b != -1)
    assert abs(st["pool_occupancy"] - used / st["pool_blocks"]) < 1e-12
    assert st["active_slots"] == sum(r is not None for r in sched.active_slots)


def test_generate_stream_end_to_end():
    """generate / generate_stream / run_loop as a user drives them: two concurrent requests,
    one stopped by EOS, one by max_new_tokens; a prompt at max_seq_len is refused."""
    cfg = {"max_batch_size": 2, "max_seq_len": 64, "block_size": 16, "head_dim": 8}
    kv = _HostKV(cfg)
    vocab = 97
    sched = ContinuousBatcher(None, kv, eos_token_id=13, backend=_StandInBackend(kv, vocab))

    def expect(prompt, n):
        out, last, pos = [], prompt[-1], len(prompt) - 1
        while len(out) < n:
            last = (last * 7 + pos * 3 + 1) % vocab
            out.append(last)
            pos += 1
            if last == 13:
                break
        return out

    async def main():
        loop = asyncio.create_task(sched.run_loop())
        a = [5, 9, 2, 11]
        b = list(range(30))
        ra, rb = await asyncio.gather(sched.generate(a, 6, temperature=0.0),
                                      sched.generate(b, 9, temperature=0.0))
        try:
            await sched.generate(list(range(64)), 3)
            refused = False
        except ValueError:
            refused = True
        loop.cancel()
        return ra, rb, refused

    ra, rb, refused = asyncio.run(main())
    assert ra == expect([5, 9, 2, 11], 6)
    assert rb == expect(list(range(30)), 9)
    assert refused
    assert all(s is None for s in sched.active_slots)
    assert len(kv.alloc.free_blocks) == kv.alloc.total_physical_blocks


def test_chunked_prefill_same_tokens():
    """With prefill_chunk_tokens the prompts are prefilled over several ticks interleaved with
    decode; every request's tokens are the same as with whole-prompt prefill."""
    cfg = {"max_batch_size": 3, "max_seq_len": 96, "block_size": 16, "head_dim": 8}
    job = [([(7 * i + 3 * j) % 97 for j in range(5 + 13 * i)], 4 + i) for i in range(5)]

    def run(chunk):
        kv = _HostKV(cfg)
        sched = ContinuousBatcher(None, kv, eos_token_id=None, backend=_StandInBackend(kv, 97),
                                  prefill_chunk_tokens=chunk)

        async def main():
            loop = asyncio.create_task(sched.run_loop())
            outs = await asyncio.gather(*[sched.generate(p, n, temperature=0.0) for p, n in job])
            loop.cancel()
            return outs

        outs = asyncio.run(main())
        assert len(kv.alloc.free_blocks) == kv.alloc.total_physical_blocks
        return outs

    whole = run(None)
    assert run(16) == whole
    assert run(7) == whole
