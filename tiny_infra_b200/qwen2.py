"""Qwen2 (Qwen2.5-0.5B architecture) forward on the sm_100a kernels of this package.

Drop-in for the reference's ``Qwen2ForCausalLM`` (models/qwen_25.py:232-251): same call
``model(input_ids [B, S] int32, batch_indices [B], kv_cache, cos, sin) -> logits [B, S, V]``,
same semantics (positions start at ``kv_cache.seq_len[batch_indices]``, the cache is written
for every layer, ``seq_len`` is NOT advanced -- the caller does that, engine/scheduler.py:234,266;
decode attends over seq_len + 1 tokens, models/qwen_25.py:115), and weights load from the
reference's state-dict names (``load_reference_state_dict``).

Per layer the decode forward is 8 kernel launches:
  rmsnorm -> QKV GEMM (+bias, RoPE, KV append) -> paged attention -> its split-K merge
  -> O GEMM (+residual, split-K) -> rmsnorm -> gate/up GEMM (+SwiGLU) -> down GEMM (+residual)
(no merge when every sequence fits 32 blocks: the attention then finishes each sequence in one
CTA; prefill: one ragged prefill-attention launch instead of the attention and its merge)
with the residual stream kept in float32 (the reference keeps it in the model dtype; float32
is closer to the float32 oracle).  The lm_head runs only on the rows whose logits are needed
and, for greedy decoding, reduces to one token per row inside the GEMM epilogue.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _native as N
from .config import QwenConfig

GATE_UP_GROUP = 8           # gate/up weight rows interleaved 8 gate, 8 up (TI_EPI_SWIGLU16)
LM_TILE = 128               # block_n of the lm_head GEMM (argmax partials per 128 columns)
O_TILE = 64                 # block_n of the o_proj GEMM (+residual, split-K)
DOWN_TILE = 128             # block_n of the down_proj GEMM (+residual, split-K)


def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


@dataclass
class PackedBatch:
    """One forward call over packed tokens.  ``decode``: every sequence has exactly one new
    token; otherwise prefill chunks (query tiles of 16 tokens)."""
    input_ids: torch.Tensor        # int32 [T]
    positions: torch.Tensor        # int32 [T]
    slot_mapping: torch.Tensor     # int64 [T]
    seq_slots: torch.Tensor        # int32 [nseq] block-table row of each sequence
    start_pos: torch.Tensor        # int32 [nseq]
    cu_seqlens: torch.Tensor       # int32 [nseq + 1]
    ctx_lens: torch.Tensor         # int32 [nseq] (decode: start + 1)
    tile_seq: torch.Tensor | None  # int32 [tiles] (prefill)
    tile_q0: torch.Tensor | None
    num_tokens: int
    num_seqs: int
    decode: bool
    last_rows: torch.Tensor        # int64 [nseq] row of each sequence's last token


class Qwen2ForCausalLM:
    def __init__(self, config: QwenConfig | None = None, device="cuda",
                 dtype: torch.dtype = torch.bfloat16) -> None:
        self.config = config or QwenConfig()
        self.device = torch.device(device)
        self.dtype = dtype
        if self.device.type != "cuda":
            raise RuntimeError("tiny_infra_b200 runs on a CUDA device only")
        c = self.config
        if c.hidden_size % c.num_attention_heads or c.intermediate_size % GATE_UP_GROUP:
            raise RuntimeError("unsupported model dimensions")
        self.weights: dict[str, torch.Tensor] = {}
        self._ws = N.Workspace()
        self._plan_ws = N.Workspace()
        self._bufs: dict[str, torch.Tensor] = {}
        self.tied = False
        # True: the residual projections sum their K slices in a fixed order (bit-reproducible
        # hidden states and greedy streams, ~13 % slower decode steps); False: every K slice
        # adds into the residual stream on its own (fastest; the last bits vary between runs).
        self.deterministic = False
        # True: decode attention starts streaming the KV blocks that no kernel of the step writes
        # while the QKV GEMM still runs (TI_ATTN_EARLY_KV; same output)
        self.early_attention = True
        # True: the per-step attention plan gives the attention CTAs that start behind the QKV
        # GEMM's SMs fewer KV blocks (TI_ATTN_PLAN_AFTER_QKV; float32 summation order only)
        self.skewed_plan = True

    # ---- weights -------------------------------------------------------------------------
    def load_reference_state_dict(self, sd: dict) -> "Qwen2ForCausalLM":
        """Load weights named as the reference module's state dict (models/qwen_25.py), fusing
        q/k/v (+biases) into one [(NH+2KVH)*D, H] matrix and interleaving gate/up rows in
        groups of 8 for the SwiGLU epilogue (any GEMM tile width that is a multiple of 16
        then holds matching gate / up rows).  A missing ``lm_head.weight`` or one identical to the
        embedding means tied embeddings."""
        c, dev, dt = self.config, self.device, self.dtype

        def get(name):
            t = sd[name]
            if isinstance(t, np.ndarray):
                t = torch.from_numpy(np.ascontiguousarray(t))
            return t.to(device=dev, dtype=dt).contiguous()

        W = {}
        W["embed"] = get("model.embed_tokens.weight")
        lm = sd.get("lm_head.weight")
        self.tied = lm is None or lm is sd["model.embed_tokens.weight"]
        W["lm_head"] = W["embed"] if self.tied else get("lm_head.weight")
        W["norm"] = get("model.norm.weight")
        h = GATE_UP_GROUP
        for i in range(c.num_layers):
            p = f"model.layers.{i}"
            W[f"{i}.qkv"] = torch.cat([get(f"{p}.self_attn.q_proj.weight"),
                                       get(f"{p}.self_attn.k_proj.weight"),
                                       get(f"{p}.self_attn.v_proj.weight")]).contiguous()
            W[f"{i}.qkv_bias"] = torch.cat([get(f"{p}.self_attn.q_proj.bias"),
                                            get(f"{p}.self_attn.k_proj.bias"),
                                            get(f"{p}.self_attn.v_proj.bias")]).contiguous()
            W[f"{i}.o"] = get(f"{p}.self_attn.o_proj.weight")
            g, u = get(f"{p}.mlp.gate_proj.weight"), get(f"{p}.mlp.up_proj.weight")
            I, H = g.shape
            W[f"{i}.gate_up"] = torch.stack([g.view(I // h, h, H), u.view(I // h, h, H)],
                                            dim=1).reshape(2 * I, H).contiguous()
            W[f"{i}.down"] = get(f"{p}.mlp.down_proj.weight")
            W[f"{i}.ln1"] = get(f"{p}.input_layernorm.weight")
            W[f"{i}.ln2"] = get(f"{p}.post_attention_layernorm.weight")
        self.weights = W
        return self

    @staticmethod
    def random_state_dict(config: QwenConfig, seed: int = 0, std: float = 0.02,
                          tied: bool = True, device="cuda",
                          dtype: torch.dtype = torch.bfloat16) -> dict:
        """Seeded random-init weights N(0, std) in the reference's state-dict naming, generated
        on ``device`` (RMSNorm weights are ones, as the reference initialises them)."""
        c = config
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        H, D, NH, KVH, I, V = (c.hidden_size, c.head_dim, c.num_attention_heads,
                               c.num_key_value_heads, c.intermediate_size, c.vocab_size)

        def rnd(*shape):
            return (torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * std).to(dtype)

        sd = {"model.embed_tokens.weight": rnd(V, H)}
        for i in range(c.num_layers):
            p = f"model.layers.{i}"
            sd[f"{p}.self_attn.q_proj.weight"] = rnd(NH * D, H)
            sd[f"{p}.self_attn.q_proj.bias"] = rnd(NH * D)
            sd[f"{p}.self_attn.k_proj.weight"] = rnd(KVH * D, H)
            sd[f"{p}.self_attn.k_proj.bias"] = rnd(KVH * D)
            sd[f"{p}.self_attn.v_proj.weight"] = rnd(KVH * D, H)
            sd[f"{p}.self_attn.v_proj.bias"] = rnd(KVH * D)
            sd[f"{p}.self_attn.o_proj.weight"] = rnd(H, NH * D)
            sd[f"{p}.mlp.gate_proj.weight"] = rnd(I, H)
            sd[f"{p}.mlp.up_proj.weight"] = rnd(I, H)
            sd[f"{p}.mlp.down_proj.weight"] = rnd(H, I)
            sd[f"{p}.input_layernorm.weight"] = torch.ones(H, device=device, dtype=dtype)
            sd[f"{p}.post_attention_layernorm.weight"] = torch.ones(H, device=device, dtype=dtype)
        sd["model.norm.weight"] = torch.ones(H, device=device, dtype=dtype)
        sd["lm_head.weight"] = sd["model.embed_tokens.weight"] if tied else rnd(V, H)
        return sd

    def quantize_lm_head_int8(self) -> "Qwen2ForCausalLM":
        """Add a weight-only int8 copy of the lm_head (one float32 scale per vocab row,
        ``ti_quantize_rows_int8``) that greedy decode steps of ``DecodeEngine`` then read instead
        of the bf16 matrix: 136 MB instead of 272 MB per step.  This changes the model's logits
        by the int8 rounding of the weights (the reference lists weight-only INT8 as its next
        step, README.md:156-157); sampled steps and ``forward`` keep the bf16 lm_head."""
        W = self.weights["lm_head"]
        V, H = W.shape
        q = torch.empty(V, H, dtype=torch.int8, device=self.device)
        scale = torch.empty(V, dtype=torch.float32, device=self.device)
        N.check(N.lib().ti_quantize_rows_int8(
            W.data_ptr(), W.stride(0), V, H, q.data_ptr(), q.stride(0), scale.data_ptr(),
            N.dtype_code(self.dtype), torch.cuda.current_stream(self.device).cuda_stream))
        self.weights["lm_head_q"] = q
        self.weights["lm_head_scale"] = scale
        return self

    def weight_bytes(self) -> int:
        """Bytes of weights one greedy decode step streams: every layer's weights and the
        lm_head once (the tied embedding is the same matrix; with the int8 lm_head its int8
        copy and scales instead of the bf16 matrix, of which the step reads only its tokens'
        embedding rows)."""
        skip = {"lm_head", "embed"} if "lm_head_q" in self.weights else set()
        seen, total = set(), 0
        for k, t in self.weights.items():
            if k in skip or t.data_ptr() in seen:
                continue
            seen.add(t.data_ptr())
            total += t.numel() * t.element_size()
        return total

    # ---- scratch buffers ---------------------------------------------------------------------
    def _buf(self, name: str, shape, dtype) -> torch.Tensor:
        n = int(np.prod(shape))
        b = self._bufs.get(name)
        if b is None or b.numel() < n or b.dtype != dtype:
            b = torch.empty(max(n, 1), dtype=dtype, device=self.device)
            self._bufs[name] = b
        return b[:n].view(*shape)

    # ---- packed-batch planning (host) -----------------------------------------------------------
    def plan(self, kv_cache, slots, counts, token_ids) -> PackedBatch:
        """Allocate the new tokens' blocks (reference order) and build the batch metadata."""
        mapping, _ = kv_cache.plan_tokens(slots, counts)
        return self.packed_batch(kv_cache, slots, counts, token_ids, mapping)

    def packed_batch(self, kv_cache, slots, counts, token_ids, mapping) -> PackedBatch:
        """Batch metadata for new tokens whose blocks are allocated (``mapping``: pool slot of
        every new token, in order); the slots' lengths have not been advanced yet."""
        dev = self.device
        nseq = len(slots)
        start = np.array([kv_cache.seq_len_host(s) for s in slots], np.int32)
        counts = np.asarray(counts, np.int32)
        cu = np.zeros(nseq + 1, np.int32)
        cu[1:] = np.cumsum(counts)
        T = int(cu[-1])
        pos = np.concatenate([start[i] + np.arange(counts[i], dtype=np.int32)
                              for i in range(nseq)]) if T else np.zeros(0, np.int32)
        decode = bool((counts == 1).all())
        tseq, tq0 = None, None
        if not decode:
            # query tiles of 16 tokens, longest causal prefix first: a tile's work grows with
            # its last position, and the GPU starts CTAs in grid order, so the long ones should
            # not be left for the tail of the launch
            ts, tq, work = [], [], []
            for i in range(nseq):
                for q0 in range(0, int(counts[i]), 16):
                    ts.append(i)
                    tq.append(q0)
                    work.append(int(start[i]) + min(q0 + 16, int(counts[i])))
            order = np.argsort(-np.asarray(work, np.int64), kind="stable")
            tseq = torch.tensor(np.asarray(ts, np.int32)[order], dtype=torch.int32, device=dev)
            tq0 = torch.tensor(np.asarray(tq, np.int32)[order], dtype=torch.int32, device=dev)
        as_dev = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a)).to(dev, dt)  # noqa: E731
        return PackedBatch(
            input_ids=as_dev(np.asarray(token_ids, np.int32), torch.int32),
            positions=as_dev(pos, torch.int32), slot_mapping=as_dev(mapping, torch.int64),
            seq_slots=as_dev(np.asarray(slots, np.int32), torch.int32),
            start_pos=as_dev(start, torch.int32), cu_seqlens=as_dev(cu, torch.int32),
            ctx_lens=as_dev(start + counts, torch.int32), tile_seq=tseq, tile_q0=tq0,
            num_tokens=T, num_seqs=nseq, decode=decode,
            last_rows=as_dev(cu[1:] - 1, torch.int64))

    # ---- forward -----------------------------------------------------------------------------
    def scratch(self, rows: int, owner: dict | None = None) -> dict:
        """Per-call activation buffers for ``rows`` tokens.  With ``owner`` (a dict kept by the
        caller, e.g. a graph-captured engine) the buffers are allocated once there and never
        move; otherwise the model's own growable buffers are used."""
        c = self.config
        D, NH, KVH = c.head_dim, c.num_attention_heads, c.num_key_value_heads
        shapes = {"xn": (rows, c.hidden_size), "qkv": (rows, (NH + 2 * KVH) * D),
                  "attn": (rows, NH * D), "act": (rows, c.intermediate_size)}
        if owner is None:
            return {k: self._buf(k, v, self.dtype) for k, v in shapes.items()}
        for k, v in shapes.items():
            if k not in owner:
                owner[k] = torch.empty(*v, dtype=self.dtype, device=self.device)
        return owner

    @staticmethod
    def _splits(k: int) -> int:
        """Requested split-K factor of a residual projection with reduction length k: up to 16
        slices of at least two 64-wide K blocks (the library lowers it to fit one wave)."""
        return int(max(1, min(16, k // 128)))

    def _layers(self, pb: PackedBatch, kv_cache, cos: torch.Tensor, sin: torch.Tensor,
                hidden: torch.Tensor, stream: int, num_layers: int | None = None,
                bufs: dict | None = None, ws: torch.Tensor | None = None,
                plan: torch.Tensor | None = None, first_layer: int = 0,
                trace=None, final_norm_out: torch.Tensor | None = None) -> None:
        """Layers first_layer .. num_layers-1 over the packed batch, in place on ``hidden``.

        With ``final_norm_out`` (and the last layer run) the model's final RMSNorm of every row
        is written there.
        ``trace(layer, stage, bufs)`` (optional) is called after each stage's kernel is issued
        (stages xn1, qkv, attn, h_mid, xn2, act, h_out; ``bufs`` holds xn / qkv / attn / act
        and the stream ``hidden``), e.g. to copy intermediate tensors for a parity check."""
        c, W, lib = self.config, self.weights, N.lib()
        dt = N.dtype_code(self.dtype)
        T, H, D = pb.num_tokens, c.hidden_size, c.head_dim
        NH, KVH, I = c.num_attention_heads, c.num_key_value_heads, c.intermediate_size
        QKV = (NH + 2 * KVH) * D
        bufs = bufs or self.scratch(T)
        xn, qkv, attn, act = bufs["xn"], bufs["qkv"], bufs["attn"], bufs["act"]
        nb = kv_cache.total_physical_blocks
        bt = kv_cache.block_tables
        maxb = kv_cache.max_blocks_per_seq
        if pb.decode and ws is None:
            need = lib.ti_paged_attention_workspace_bytes(pb.num_seqs, NH, KVH, D, maxb, 0)
            ws = self._ws.get(self.device, need)
        if pb.decode:
            # the batch's attention work split, resolved once for all layers
            if plan is None:
                plan = self._plan_ws.get(self.device,
                                         lib.ti_paged_attention_plan_bytes(pb.num_seqs))
            # each layer's attention follows its QKV GEMM: the CTAs behind that GEMM's SMs start
            # late, so they get fewer KV blocks (TI_ATTN_PLAN_AFTER_QKV)
            N.check(lib.ti_paged_attention_plan_ex(
                bt.data_ptr(), bt.stride(0), pb.seq_slots.data_ptr(), pb.ctx_lens.data_ptr(),
                pb.num_seqs, NH, KVH, D, maxb, nb, plan.data_ptr(), plan.numel(),
                N.TI_ATTN_PLAN_AFTER_QKV if self.skewed_plan else 0, H, dt, stream))
        split_o = self._splits(NH * D)
        split_d = self._splits(I)
        residual = N.TI_EPI_RESIDUAL_DET if self.deterministic else N.TI_EPI_RESIDUAL
        tb = dict(bufs, hidden=hidden)
        end = c.num_layers if num_layers is None else num_layers

        def mark(li, stage):
            if trace is not None:
                trace(li, stage, tb)

        def rmsnorm(out, weight, rows):
            N.check(lib.ti_rmsnorm(out.data_ptr(), hidden.data_ptr(), N.TI_DTYPE_FP32,
                                   weight.data_ptr(), c.rms_norm_eps, rows, H, dt, stream))

        for li in range(first_layer, end):
            kc, vc = kv_cache.key_cache[li], kv_cache.value_cache[li]
            rmsnorm(xn, W[f"{li}.ln1"], T)
            mark(li, "xn1")
            N.check(lib.ti_gemm_qkv_rope(
                xn.data_ptr(), H, W[f"{li}.qkv"].data_ptr(), H, W[f"{li}.qkv_bias"].data_ptr(),
                T, H, NH, KVH, D, qkv.data_ptr(), QKV, kc.data_ptr(), vc.data_ptr(),
                pb.slot_mapping.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                pb.positions.data_ptr(), kv_cache.block_size, dt, stream))
            mark(li, "qkv")
            if pb.decode:
                # the plan and every KV block but each sequence's last (the one the QKV epilogue
                # appends to) are final before the QKV GEMM starts (the RMSNorm before it lets it
                # launch only once the plan kernel has completed): the attention streams them
                # while that GEMM still runs
                early = self.early_attention
                N.check(lib.ti_paged_attention_decode_planned_ex(
                    attn.data_ptr(), NH * D, qkv.data_ptr(), QKV, kc.data_ptr(), vc.data_ptr(), nb,
                    bt.data_ptr(), bt.stride(0), pb.seq_slots.data_ptr(), pb.ctx_lens.data_ptr(),
                    pb.num_seqs, NH, KVH, D, kv_cache.block_size, maxb, dt, ws.data_ptr(),
                    ws.numel(), plan.data_ptr(), N.TI_ATTN_EARLY_KV if early else 0, stream))
            else:
                N.check(lib.ti_paged_prefill_attention(
                    attn.data_ptr(), NH * D, qkv.data_ptr(), QKV, kc.data_ptr(), vc.data_ptr(), nb,
                    bt.data_ptr(), bt.stride(0), pb.seq_slots.data_ptr(), pb.start_pos.data_ptr(),
                    pb.cu_seqlens.data_ptr(), pb.tile_seq.data_ptr(), pb.tile_q0.data_ptr(),
                    pb.tile_seq.numel(), NH, KVH, D, kv_cache.block_size, dt, stream))
            mark(li, "attn")
            N.check(lib.ti_gemm(residual, attn.data_ptr(), NH * D, W[f"{li}.o"].data_ptr(),
                                NH * D, T, H, NH * D, hidden.data_ptr(), H, None, None, None, dt,
                                O_TILE, split_o, stream))
            mark(li, "h_mid")
            rmsnorm(xn, W[f"{li}.ln2"], T)
            mark(li, "xn2")
            N.check(lib.ti_gemm(N.TI_EPI_SWIGLU16, xn.data_ptr(), H,
                                W[f"{li}.gate_up"].data_ptr(), H, T, 2 * I, H, act.data_ptr(), I,
                                None, None, None, dt, 0, 1, stream))
            mark(li, "act")
            N.check(lib.ti_gemm(residual, act.data_ptr(), I, W[f"{li}.down"].data_ptr(),
                                I, T, H, I, hidden.data_ptr(), H, None, None, None, dt,
                                DOWN_TILE, split_d, stream))
            mark(li, "h_out")
        if final_norm_out is not None and end == c.num_layers:
            rmsnorm(final_norm_out, W["norm"], final_norm_out.shape[0])

    def _final_norm(self, hidden_rows: torch.Tensor, stream: int) -> torch.Tensor:
        c = self.config
        R = hidden_rows.shape[0]
        xf = self._buf("xf", (R, c.hidden_size), self.dtype)
        N.check(N.lib().ti_rmsnorm(xf.data_ptr(), hidden_rows.data_ptr(), N.TI_DTYPE_FP32,
                                   self.weights["norm"].data_ptr(), c.rms_norm_eps, R,
                                   c.hidden_size, N.dtype_code(self.dtype), stream))
        return xf

    def lm_head_logits(self, xf: torch.Tensor, stream: int) -> torch.Tensor:
        c = self.config
        R = xf.shape[0]
        logits = torch.empty(R, c.vocab_size, dtype=self.dtype, device=self.device)
        N.check(N.lib().ti_gemm(N.TI_EPI_STORE, xf.data_ptr(), c.hidden_size,
                                self.weights["lm_head"].data_ptr(), c.hidden_size, R,
                                c.vocab_size, c.hidden_size, logits.data_ptr(), c.vocab_size,
                                None, None, None, N.dtype_code(self.dtype), LM_TILE, 1, stream))
        return logits

    def forward_packed(self, pb: PackedBatch, kv_cache, cos, sin, *, rows: str = "all",
                       num_layers: int | None = None, return_hidden: bool = False,
                       first_layer: int = 0, hidden_in: torch.Tensor | None = None, trace=None):
        """Run the layers over a packed batch; returns logits of every token (rows='all') or of
        each sequence's last token (rows='last').  ``hidden_in`` (float32 [T, H]) starts the
        residual stream at layer ``first_layer`` instead of the embedding at layer 0; ``trace``
        is passed to every layer (see ``_layers``)."""
        c = self.config
        stream = torch.cuda.current_stream(self.device).cuda_stream
        if hidden_in is not None:
            hidden = hidden_in.to(self.device, torch.float32).contiguous().clone()
        else:
            hidden = torch.empty(pb.num_tokens, c.hidden_size, dtype=torch.float32,
                                 device=self.device)
            N.check(N.lib().ti_embedding(hidden.data_ptr(), self.weights["embed"].data_ptr(),
                                         pb.input_ids.data_ptr(), pb.num_tokens, c.hidden_size,
                                         c.vocab_size, N.dtype_code(self.dtype), stream))
        self._layers(pb, kv_cache, cos, sin, hidden, stream, num_layers, first_layer=first_layer,
                     trace=trace)
        if return_hidden:
            return hidden
        h = hidden if rows == "all" else hidden.index_select(0, pb.last_rows).contiguous()
        return self.lm_head_logits(self._final_norm(h, stream), stream)

    def __call__(self, input_ids, batch_indices, kv_cache, cos_cache, sin_cache):
        return self.forward(input_ids, batch_indices, kv_cache, cos_cache, sin_cache)

    def forward(self, input_ids: torch.Tensor, batch_indices: torch.Tensor, kv_cache,
                cos_cache: torch.Tensor, sin_cache: torch.Tensor) -> torch.Tensor:
        """Reference-compatible forward (models/qwen_25.py:239-251): logits [B, S, V] for every
        position; KV written for every layer; ``kv_cache.seq_len`` left unchanged."""
        kv_cache.sync_from_device()   # callers may have advanced seq_len on the device
        B, S = input_ids.shape
        slots = [int(x) for x in batch_indices.reshape(-1).tolist()]
        ids = input_ids.reshape(-1).to(torch.int32).cpu().numpy()
        pb = self.plan(kv_cache, slots, [S] * B, ids)
        cos = cos_cache.to(self.device, torch.float32).contiguous()
        sin = sin_cache.to(self.device, torch.float32).contiguous()
        logits = self.forward_packed(pb, kv_cache, cos, sin, rows="all")
        return logits.view(B, S, -1)

    # ---- RoPE tables -------------------------------------------------------------------------
    def rope_tables(self, max_positions: int):
        """cos/sin [max_positions, D/2] float32, built like engine/scheduler.py:36-48."""
        D = self.config.head_dim
        inv_freq = 1.0 / (self.config.rope_theta ** (
            torch.arange(0, D, 2, device=self.device).float() / D))
        t = torch.arange(max_positions, device=self.device, dtype=torch.float32)
        freqs = torch.einsum("i,j->ij", t, inv_freq)
        return freqs.cos().contiguous(), freqs.sin().contiguous()
