"""Batched decode step with device-side packing, captured as one CUDA graph per batch bucket.

This is the B200 form of the reference's decode phase (engine/scheduler.py:250-281 +
Qwen2ForCausalLM.forward for S == 1 + _sample_next_token for greedy rows): per step the host
only plans which slots need a new KV block (FIFO, bit-exact with the reference allocator) and
copies three small int32 vectors; everything else -- slot compaction, positions, pool slots,
context lengths, the 24 layers, lm_head with an in-epilogue argmax and the seq_len advance --
runs as one graph replay.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _native as N
from .qwen2 import LM_TILE, PackedBatch, Qwen2ForCausalLM

BUCKETS = (1, 2, 4, 8, 16, 32, 64, 128, 256, 512)


class DecodeEngine:
    def __init__(self, model: Qwen2ForCausalLM, kv_cache, max_rows: int | None = None,
                 use_graphs: bool = True) -> None:
        self.model, self.kv = model, kv_cache
        c = model.config
        dev = model.device
        self.max_rows = int(max_rows or kv_cache.max_batch_size)
        R = self.max_rows
        self.use_graphs = use_graphs
        self.cos, self.sin = model.rope_tables(kv_cache.max_seq_len)
        # inputs of a step: tokens, slots (-1 = padding row), new block per row (-1 = none)
        self.d_in = torch.zeros(3, R, dtype=torch.int32, device=dev)
        self.h_in = torch.zeros(3, R, dtype=torch.int32).pin_memory()
        self.positions = torch.zeros(R, dtype=torch.int32, device=dev)
        self.slot_mapping = torch.zeros(R, dtype=torch.int64, device=dev)
        self.ctx_lens = torch.zeros(R, dtype=torch.int32, device=dev)
        self.hidden = torch.zeros(R, c.hidden_size, dtype=torch.float32, device=dev)
        self.xf = torch.zeros(R, c.hidden_size, dtype=model.dtype, device=dev)
        self.ntiles = c.vocab_size // LM_TILE
        self.part_val = torch.zeros(R, self.ntiles, dtype=torch.float32, device=dev)
        self.part_idx = torch.zeros(R, self.ntiles, dtype=torch.int32, device=dev)
        self.next_tok = torch.zeros(R, dtype=torch.int32, device=dev)
        self.h_out = torch.zeros(R, dtype=torch.int32).pin_memory()
        self.bufs: dict = {}
        model.scratch(R, self.bufs)
        need = N.lib().ti_paged_attention_workspace_bytes(
            R, c.num_attention_heads, c.num_key_value_heads, c.head_dim,
            kv_cache.max_blocks_per_seq, 0)
        self.ws = torch.zeros(need, dtype=torch.uint8, device=dev)
        self.plan = torch.zeros(N.lib().ti_paged_attention_plan_bytes(R), dtype=torch.uint8,
                                device=dev)
        self.graphs: dict[tuple, torch.cuda.CUDAGraph] = {}
        self.launches_per_step: dict[tuple, int] = {}
        # sampled steps (allocated on first use): logits [R, V] and the per-row sampling
        # parameters (temperature, cut rank, top-p, uniform) copied in with the step's inputs
        self.logits = None
        self.d_params = torch.zeros(4, R, dtype=torch.float32, device=dev)
        self.h_params = torch.zeros(4, R, dtype=torch.float32).pin_memory()

    @staticmethod
    def bucket(n: int) -> int:
        for b in BUCKETS:
            if n <= b:
                return b
        return n

    def _batch(self, rows: int) -> PackedBatch:
        return PackedBatch(
            input_ids=self.d_in[0, :rows], positions=self.positions[:rows],
            slot_mapping=self.slot_mapping[:rows], seq_slots=self.d_in[1, :rows],
            start_pos=self.positions[:rows], cu_seqlens=None, ctx_lens=self.ctx_lens[:rows],
            tile_seq=None, tile_q0=None, num_tokens=rows, num_seqs=rows, decode=True,
            last_rows=None)

    def _launch(self, rows: int, sampled: bool = False) -> None:
        """All launches of one decode step for ``rows`` (bucket-padded) rows: greedy (lm_head
        with the argmax epilogue) or sampled (logits, then the device sampler)."""
        m, c, lib = self.model, self.model.config, N.lib()
        s = torch.cuda.current_stream(m.device).cuda_stream
        dt = N.dtype_code(m.dtype)
        kv = self.kv
        N.check(lib.ti_decode_prepare(
            self.d_in[0].data_ptr(), self.d_in[1].data_ptr(), self.d_in[2].data_ptr(),
            kv.seq_len.data_ptr(), kv.block_tables.data_ptr(), kv.block_tables.stride(0),
            kv.block_tables.shape[0], kv.block_tables.shape[1], kv.total_physical_blocks,
            kv.block_size, self.positions.data_ptr(), self.slot_mapping.data_ptr(),
            self.ctx_lens.data_ptr(), self.hidden.data_ptr(), m.weights["embed"].data_ptr(),
            c.hidden_size, c.vocab_size, rows, dt, s))
        m._layers(self._batch(rows), kv, self.cos, self.sin, self.hidden[:rows], s,
                  bufs=self.bufs, ws=self.ws, plan=self.plan, final_norm_out=self.xf[:rows])
        if sampled:
            N.check(lib.ti_gemm(N.TI_EPI_STORE, self.xf.data_ptr(), c.hidden_size,
                                m.weights["lm_head"].data_ptr(), c.hidden_size, rows,
                                c.vocab_size, c.hidden_size, self.logits.data_ptr(),
                                c.vocab_size, None, None, None, dt, LM_TILE, 1, s))
            dp = self.d_params
            N.check(lib.ti_sample(self.logits.data_ptr(), c.vocab_size, dt, rows, c.vocab_size,
                                  dp[0].data_ptr(), dp[1].data_ptr(), dp[2].data_ptr(),
                                  dp[3].data_ptr(), self.next_tok.data_ptr(),
                                  self.d_in[1].data_ptr(), kv.seq_len.data_ptr(), 1, s))
            return
        if "lm_head_q" in m.weights:        # weight-only int8 lm_head, 256 rows per launch
            q, sc = m.weights["lm_head_q"], m.weights["lm_head_scale"]
            for r0 in range(0, rows, 256):
                n = min(256, rows - r0)
                N.check(lib.ti_lm_head_argmax_int8(
                    self.xf[r0].data_ptr(), c.hidden_size, q.data_ptr(), q.stride(0),
                    sc.data_ptr(), n, c.vocab_size, c.hidden_size, self.part_val[r0].data_ptr(),
                    self.part_idx[r0].data_ptr(), dt, s))
        else:
            N.check(lib.ti_gemm(N.TI_EPI_ARGMAX, self.xf.data_ptr(), c.hidden_size,
                                m.weights["lm_head"].data_ptr(), c.hidden_size, rows,
                                c.vocab_size, c.hidden_size, None, 0, None,
                                self.part_val.data_ptr(), self.part_idx.data_ptr(), dt, LM_TILE,
                                1, s))
        N.check(lib.ti_argmax_finish(self.part_val.data_ptr(), self.part_idx.data_ptr(),
                                     self.ntiles, rows, self.next_tok.data_ptr(),
                                     self.d_in[1].data_ptr(), kv.seq_len.data_ptr(), 1, s))

    def _copy_in(self, rows: int, sampled: bool) -> None:
        # row by row: each [i, :rows] slice of the pinned staging buffers is contiguous (a
        # [:, :rows] slice is not, and would be copied through an unpinned temporary)
        for i in range(self.d_in.shape[0]):
            self.d_in[i, :rows].copy_(self.h_in[i, :rows], non_blocking=True)
        if sampled:
            for i in range(self.d_params.shape[0]):
                self.d_params[i, :rows].copy_(self.h_params[i, :rows], non_blocking=True)

    def _replay(self, rows: int, sampled: bool = False, io: bool = False) -> None:
        """Run one decode step: the kernels alone, or with ``io`` the host->device copy of the
        staged inputs before them and the device->host copy of the tokens after them, all in one
        graph replay (pinned host buffers), so a host-driven step costs one launch."""
        if sampled and self.logits is None:
            c = self.model.config
            self.logits = torch.empty(self.max_rows, c.vocab_size, dtype=self.model.dtype,
                                      device=self.model.device)
        if not self.use_graphs:
            if io:
                self._copy_in(rows, sampled)
            self._launch(rows, sampled)
            if io:
                self.h_out[:rows].copy_(self.next_tok[:rows], non_blocking=True)
            return
        key = (rows, sampled, io)
        g = self.graphs.get(key)
        if g is None:
            # one eager run sets kernel attributes / tensor-map caches outside the capture; it
            # must not change state, so it runs on a padding-only input
            saved = self.d_in.clone()
            seq_saved = self.kv.seq_len.clone()
            self.d_in[1].fill_(-1)
            self.d_in[2].fill_(-1)
            before = N.launch_count()
            self._launch(rows, sampled)
            self.launches_per_step[key] = N.launch_count() - before
            torch.cuda.current_stream().synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                if io:
                    self._copy_in(rows, sampled)
                self._launch(rows, sampled)
                if io:
                    self.h_out[:rows].copy_(self.next_tok[:rows], non_blocking=True)
            self.d_in.copy_(saved)
            self.kv.seq_len.copy_(seq_saved)
            self.graphs[key] = g
        g.replay()

    def stage(self, slots, tokens, copy: bool = True) -> int:
        """Plan block allocation for one new token per slot and stage the step's inputs in
        pinned host memory (and, with ``copy``, copy them to the device asynchronously); returns
        the padded row count."""
        n = len(slots)
        if n > self.max_rows:
            raise ValueError(f"decode batch {n} exceeds the engine's {self.max_rows} rows")
        rows = self.bucket(n) if self.use_graphs else n
        rows = min(rows, self.max_rows)
        slots = np.asarray(slots, np.int32)        # one conversion of a host list per step
        new_block = self.kv.plan_decode(slots)
        h = self.h_in.numpy()
        h[0, :n] = tokens
        h[1, :n] = slots
        h[2, :n] = new_block
        h[0, n:rows] = 0
        h[1, n:rows] = -1
        h[2, n:rows] = -1
        if copy:
            for i in range(self.d_in.shape[0]):
                self.d_in[i, :rows].copy_(self.h_in[i, :rows], non_blocking=True)
        return rows

    def step(self, slots, tokens, params=None) -> np.ndarray:
        """One decode step for the given slots (public API: host ints in, host ints out).

        ``tokens[i]`` is the last token of the sequence in ``slots[i]``; returns the next token
        of each: greedy, or drawn with ``params`` (a ``sampler.SamplingParams`` of the batch;
        rows with temperature 0 stay greedy).  Blocks are allocated as the reference would;
        ``seq_len`` advances by one.
        """
        n = len(slots)
        if n == 0:
            return np.zeros(0, np.int32)
        slots = np.asarray(slots, np.int32)
        rows = self.stage(slots, tokens, copy=False)
        sampled = params is not None and not params.all_greedy
        if sampled:
            h = self.h_params.numpy()
            h[:, :n] = params.packed()
            h[0, n:rows] = 0.0                    # padding rows: greedy, no cut
            h[1, n:rows] = 0.0
            h[2, n:rows] = 1.0
            h[3, n:rows] = 0.0
        self._replay(rows, sampled, io=True)   # inputs in, the step, tokens out: one replay
        self.kv.advance(slots, 1)      # host mirror, while the step runs (the device advances
        torch.cuda.current_stream().synchronize()   # its own copy in the step's last kernel)
        return self.h_out[:n].numpy().copy()

    # ---- device-resident decoding (no host round trip between steps) -----------------------
    def plan_steps(self, slots, steps: int) -> torch.Tensor:
        """Pre-plan ``steps`` decode steps' block allocations (host mirrors advance as the
        steps will); returns int32 [steps, rows] new-block ids on the device."""
        n = len(slots)
        rows = min(self.bucket(n), self.max_rows)
        plan = np.full((steps, rows), -1, np.int32)
        for k in range(steps):
            plan[k, :n] = self.kv.plan_decode(slots)
            self.kv.advance(slots, 1)
        return torch.from_numpy(plan).to(self.model.device)

    def run_resident(self, slots, first_tokens: torch.Tensor, plan: torch.Tensor,
                     out_tokens: torch.Tensor | None = None) -> None:
        """Run ``plan.shape[0]`` greedy steps back to back: each step's input tokens are the
        previous step's outputs, copied on the device.  The host mirrors must already have been
        advanced by :meth:`plan_steps`.  ``out_tokens`` [steps, n] receives every step's tokens."""
        n = len(slots)
        rows = plan.shape[1]
        self.d_in[1, :n].copy_(torch.as_tensor(np.asarray(slots, np.int32)), non_blocking=False)
        self.d_in[1, n:rows] = -1
        self.d_in[0, :n].copy_(first_tokens[:n])
        self.d_in[0, n:rows] = 0
        for k in range(plan.shape[0]):
            self.d_in[2, :rows].copy_(plan[k])
            self._replay(rows)
            self.d_in[0, :n].copy_(self.next_tok[:n])
            if out_tokens is not None:
                out_tokens[k, :n].copy_(self.next_tok[:n])
