"""Restatement of the reference's Qwen2 forward (models/qwen_25.py) in numpy float32.

Weights are a dict keyed by the reference module's ``state_dict`` names
(``model.layers.{i}.self_attn.q_proj.weight`` ...), so the same arrays can be loaded into the
reference ``Qwen2ForCausalLM`` by ``load_state_dict`` when generating golden vectors.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import kernels
from .cache import OracleKVCache
from .numerics import bf16_round, round_to


@dataclass
class OracleConfig:
    """models/config.py:4-11 (head_dim = hidden/heads, models/qwen_25.py:44)."""
    vocab_size: int = 151936
    hidden_size: int = 896
    num_layers: int = 24
    num_attention_heads: int = 14
    num_key_value_heads: int = 2
    intermediate_size: int = 4864
    rope_theta: float = 1000000.0
    rms_norm_eps: float = 1e-6

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads


def init_weights(cfg: OracleConfig, seed: int = 0, std: float = 0.02, tied: bool = True,
                 bf16: bool = True) -> dict:
    """Seeded random-init weights N(0, std) (numpy PCG64), rounded to bf16 values when ``bf16``.

    RMSNorm weights are ones, as the reference module initialises them (models/qwen_25.py:20).
    With ``tied`` the lm_head is the embedding matrix (same array object).
    """
    rng = np.random.default_rng(seed)
    H, D = cfg.hidden_size, cfg.head_dim
    NH, KVH, I, V = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size, cfg.vocab_size

    def rnd(*shape):
        w = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)
        return bf16_round(w) if bf16 else w

    W = {"model.embed_tokens.weight": rnd(V, H)}
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}"
        W[f"{p}.self_attn.q_proj.weight"] = rnd(NH * D, H)
        W[f"{p}.self_attn.q_proj.bias"] = rnd(NH * D)
        W[f"{p}.self_attn.k_proj.weight"] = rnd(KVH * D, H)
        W[f"{p}.self_attn.k_proj.bias"] = rnd(KVH * D)
        W[f"{p}.self_attn.v_proj.weight"] = rnd(KVH * D, H)
        W[f"{p}.self_attn.v_proj.bias"] = rnd(KVH * D)
        W[f"{p}.self_attn.o_proj.weight"] = rnd(H, NH * D)
        W[f"{p}.mlp.gate_proj.weight"] = rnd(I, H)
        W[f"{p}.mlp.up_proj.weight"] = rnd(I, H)
        W[f"{p}.mlp.down_proj.weight"] = rnd(H, I)
        W[f"{p}.input_layernorm.weight"] = np.ones(H, np.float32)
        W[f"{p}.post_attention_layernorm.weight"] = np.ones(H, np.float32)
    W["model.norm.weight"] = np.ones(H, np.float32)
    W["lm_head.weight"] = W["model.embed_tokens.weight"] if tied else rnd(V, H)
    return W


STAGES = ("xn1", "q", "k", "v", "attn", "h_mid", "xn2", "act", "h_out")


def decoder_layer(W: dict, cfg: OracleConfig, li: int, h: np.ndarray, pos: np.ndarray,
                  batch_indices: np.ndarray, cache: OracleKVCache, cos: np.ndarray,
                  sin: np.ndarray, *, device_rounding: str | None = None,
                  chunked_prefill: bool = False, record: dict | None = None,
                  given: dict | None = None) -> np.ndarray:
    """One ``Qwen2DecoderLayer`` (models/qwen_25.py:161-192 with Qwen2Attention :51-131 and
    Qwen2MLP :140-151) on the float32 residual stream h [B, S, H]; returns the new stream.

    The stages, named as in :data:`STAGES`: ``xn1`` (input RMSNorm), ``q`` / ``k`` / ``v``
    (projections + bias, RoPE on q and k, [B, S, heads, D]), ``attn`` ([B, S, H]), ``h_mid``
    (stream after the attention residual), ``xn2`` (post-attention RMSNorm), ``act`` (SwiGLU
    output [B, S, I]) and ``h_out``.  ``record`` (a dict) receives every stage's value as
    computed here; ``given`` (a dict) then replaces the named stages by the caller's values, so
    that each later stage is computed from them -- with another implementation's stored tensors,
    ``record`` holds what each of its stages should have produced from its own inputs.
    """
    rd = (lambda x: round_to(x, device_rounding))
    given = given or {}
    B, S = h.shape[:2]
    D = cfg.head_dim
    NH, KVH = cfg.num_attention_heads, cfg.num_key_value_heads
    eps = cfg.rms_norm_eps
    p = f"model.layers.{li}"

    def stage(name, value):
        if record is not None:
            record[name] = np.array(value, np.float32, copy=True)
        if name in given:
            value = np.asarray(given[name], np.float32).reshape(np.shape(value))
        return value

    res = h
    x = stage("xn1", rd(kernels.rmsnorm(h, W[f"{p}.input_layernorm.weight"], eps,
                                        round_fn=rd if device_rounding else None)))
    q = x @ W[f"{p}.self_attn.q_proj.weight"].T + W[f"{p}.self_attn.q_proj.bias"]
    k = x @ W[f"{p}.self_attn.k_proj.weight"].T + W[f"{p}.self_attn.k_proj.bias"]
    v = x @ W[f"{p}.self_attn.v_proj.weight"].T + W[f"{p}.self_attn.v_proj.bias"]
    q = q.reshape(B, S, NH, D).astype(np.float32)
    k = k.reshape(B, S, KVH, D).astype(np.float32)
    v = v.reshape(B, S, KVH, D).astype(np.float32)
    q3 = q.reshape(B * S, NH, D)
    k3 = k.reshape(B * S, KVH, D)
    kernels.rope_inplace(q3, k3, cos, sin, pos.reshape(-1))              # :79
    q = stage("q", rd(q3.reshape(B, S, NH, D)))
    k = stage("k", rd(k3.reshape(B, S, KVH, D)))
    v = stage("v", rd(v))
    cache.allocate_and_insert(li, batch_indices, k.transpose(0, 2, 1, 3),   # :82-87
                              v.transpose(0, 2, 1, 3))
    if S > 1 and not chunked_prefill:
        attn = kernels.causal_self_attention(q, k, v)                       # :89-104
    elif S > 1:
        attn = np.stack([kernels.paged_prefill_attention(
            q[i], cache.key_cache[li], cache.value_cache[li],
            cache.block_tables[b], int(cache.seq_len[b]), cache.block_size)
            for i, b in enumerate(batch_indices.tolist())])
    else:
        bt = cache.block_tables[batch_indices]                              # :114
        ctx = cache.seq_len[batch_indices] + S                              # :115
        out = np.zeros((B, NH, D), np.float32)
        kernels.paged_attention(out, q[:, 0], cache.key_cache[li], cache.value_cache[li],
                                bt, ctx, cache.block_size)                  # :117-125
        attn = out[:, None]
    attn = stage("attn", rd(attn.reshape(B, S, NH * D)))
    h = stage("h_mid", attn @ W[f"{p}.self_attn.o_proj.weight"].T + res)  # :130, :182
    res = h
    x = stage("xn2", rd(kernels.rmsnorm(h, W[f"{p}.post_attention_layernorm.weight"], eps,
                                        round_fn=rd if device_rounding else None)))
    g = x @ W[f"{p}.mlp.gate_proj.weight"].T
    u = x @ W[f"{p}.mlp.up_proj.weight"].T
    a = stage("act", rd(kernels.swiglu(np.concatenate([g, u], axis=-1))))  # :146-148
    return stage("h_out", a @ W[f"{p}.mlp.down_proj.weight"].T + res)     # :151, :191


def embed(W: dict, input_ids: np.ndarray) -> np.ndarray:
    """models/qwen_25.py:224: the float32 residual stream's starting value."""
    return W["model.embed_tokens.weight"][input_ids].astype(np.float32)


def positions(cache: OracleKVCache, batch_indices: np.ndarray, S: int) -> np.ndarray:
    """models/qwen_25.py:218-222: positions of the call's tokens, from seq_len."""
    start = cache.seq_len[np.asarray(batch_indices).reshape(-1)].astype(np.int64)
    return np.arange(S)[None, :] + start[:, None]


def forward(W: dict, cfg: OracleConfig, input_ids: np.ndarray, batch_indices: np.ndarray,
            cache: OracleKVCache, cos: np.ndarray, sin: np.ndarray, *,
            device_rounding: str | None = None, last_only: bool = False,
            chunked_prefill: bool = False, layer_hook=None) -> np.ndarray:
    """``Qwen2ForCausalLM.forward`` (models/qwen_25.py:239-251, :205-230, :161-192, :51-151).

    input_ids [B, S] -> logits [B, S, V] (or [B, 1, V] with ``last_only``).  The cache is
    written through :meth:`OracleKVCache.allocate_and_insert` exactly as the reference does; like
    the reference, ``cache.seq_len`` is NOT advanced here (the scheduler does it after the
    forward, engine/scheduler.py:234,266).

    ``device_rounding='bf16'`` rounds to bf16 at the points where the CUDA path stores bf16
    (normed activations -- also before the RMSNorm weight multiply, as the reference rounds
    them -- q/k/v after RoPE and the KV pool, attention output, SwiGLU output); the residual
    stream and the logits stay float32 as on the device.  ``None`` is pure fp32.

    ``chunked_prefill`` makes S>1 calls attend over the paged pool (earlier tokens of the
    sequence included) instead of the reference's self-only SDPA; both agree when the call
    starts at seq_len 0.

    ``layer_hook(layer_index, h)`` (optional) sees the float32 residual stream ``h`` [B, S, H]
    after every decoder layer (models/qwen_25.py:226-228).
    """
    rd = (lambda x: round_to(x, device_rounding))
    B, S = input_ids.shape
    eps = cfg.rms_norm_eps
    batch_indices = np.asarray(batch_indices).reshape(-1)
    pos = positions(cache, batch_indices, S)
    h = embed(W, input_ids)
    for li in range(cfg.num_layers):
        h = decoder_layer(W, cfg, li, h, pos, batch_indices, cache, cos, sin,
                          device_rounding=device_rounding, chunked_prefill=chunked_prefill)
        if layer_hook is not None:
            layer_hook(li, h)
    if last_only:
        h = h[:, -1:]
    h = kernels.rmsnorm(h, W["model.norm.weight"], eps,                       # :230
                        round_fn=rd if device_rounding else None)
    h = rd(h)
    return (h @ W["lm_head.weight"].T).astype(np.float32)                     # :250
