"""numpy float32 restatements of the reference's device kernels and per-layer math.

Every function cites the reference file:line it follows.  All arithmetic is float32; the
caller decides whether inputs carry bf16/fp16-representable values.
"""
from __future__ import annotations

import math

import numpy as np


# ---------------------------------------------------------------------------------------------
# Paged decode attention -- src/attention.cu:54-154 (kernel) and :156-197 (launcher)
# ---------------------------------------------------------------------------------------------
def paged_attention(out: np.ndarray, q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray,
                    block_tables: np.ndarray, context_lens: np.ndarray, block_size: int) -> None:
    """Single-query GQA attention over a paged KV pool, written into ``out`` in place.

    Shapes follow the reference launcher (src/attention.cu:165-169):
      q, out        [B, NH, D]
      k/v_cache     [NB, KVH, block_size, D]
      block_tables  [B, max_blocks]  int32, -1 = unassigned
      context_lens  [B]              int32

    Semantics kept from the kernel:
      * scale 1/sqrt(D) applied to q (attention.cu:70,184);
      * kv head = h // (NH // KVH) (attention.cu:92);
      * ctx == 0 returns early and leaves ``out`` untouched (attention.cu:62);
      * reading stops at the first negative block-table entry (attention.cu:90); if that leaves
        no token at all, the kernel's final ``o / d`` is 0/0, i.e. NaN (attention.cu:150);
      * block-table columns beyond ``max_blocks`` and block ids outside the pool are treated as
        absent (the reference kernel would read outside the table / pool there, which is
        undefined for a caller).
    """
    B, NH, D = q.shape
    KVH = k_cache.shape[1]
    max_blocks = block_tables.shape[1]
    group = NH // KVH
    scale = np.float32(1.0) / np.float32(math.sqrt(D))
    head_to_kv = np.arange(NH) // group
    for b in range(B):
        ctx = int(context_lens[b])
        if ctx <= 0:
            continue
        nblk = (ctx + block_size - 1) // block_size
        ks, vs = [], []
        for bi in range(min(nblk, max_blocks)):
            phys = int(block_tables[b, bi])
            if phys < 0 or phys >= k_cache.shape[0]:
                break
            ntok = min(block_size, ctx - bi * block_size)
            ks.append(k_cache[phys, :, :ntok, :])
            vs.append(v_cache[phys, :, :ntok, :])
        if not ks:
            out[b] = np.nan
            continue
        K = np.concatenate(ks, axis=1).astype(np.float32)   # [KVH, T, D]
        V = np.concatenate(vs, axis=1).astype(np.float32)
        qs = q[b].astype(np.float32) * scale                  # [NH, D]
        s = np.einsum("hd,htd->ht", qs, K[head_to_kv])        # [NH, T]
        m = s.max(axis=-1, keepdims=True)
        p = np.exp(s - m)
        l = p.sum(axis=-1, keepdims=True)
        out[b] = np.einsum("ht,htd->hd", p, V[head_to_kv]) / l


# ---------------------------------------------------------------------------------------------
# Prefill attention
# ---------------------------------------------------------------------------------------------
def causal_self_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """Prefill attention of models/qwen_25.py:89-104.

    q [B, S, NH, D], k/v [B, S, KVH, D] -> [B, S, NH, D].  K/V are repeated per GQA group
    (``repeat_interleave``, :91-93) and ``F.scaled_dot_product_attention(is_causal=True)`` runs
    over this call's own tokens only, with its default scale 1/sqrt(D) (:101-103).
    """
    B, S, NH, D = q.shape
    KVH = k.shape[2]
    rep = NH // KVH
    kk = np.repeat(k, rep, axis=2).astype(np.float32)
    vv = np.repeat(v, rep, axis=2).astype(np.float32)
    scale = np.float32(1.0 / math.sqrt(D))
    s = np.einsum("bihd,bjhd->bhij", q.astype(np.float32), kk) * scale
    mask = np.triu(np.ones((S, S), dtype=bool), k=1)
    s = np.where(mask[None, None], -np.inf, s)
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("bhij,bjhd->bihd", p, vv)


def paged_prefill_attention(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray,
                            block_table: np.ndarray, start_pos: int, block_size: int) -> np.ndarray:
    """Causal attention for a chunk of ``S`` new tokens at positions ``start_pos..start_pos+S-1``
    of one sequence, reading every key/value (earlier chunks and this chunk) from the paged pool.

    q [S, NH, D] -> [S, NH, D].  For ``start_pos == 0`` this equals
    :func:`causal_self_attention` on the same tokens, which is the reference's prefill
    (models/qwen_25.py:89-104); for ``start_pos > 0`` it is the chunked-prefill generalisation.
    """
    S, NH, D = q.shape
    KVH = k_cache.shape[1]
    total = start_pos + S
    pos = np.arange(total)
    phys = block_table[pos // block_size]
    if (phys < 0).any():
        raise ValueError("block table does not cover the chunk")
    K = k_cache[phys, :, pos % block_size, :].astype(np.float32)   # [total, KVH, D]
    V = v_cache[phys, :, pos % block_size, :].astype(np.float32)
    rep = NH // KVH
    K = np.repeat(K, rep, axis=1)
    V = np.repeat(V, rep, axis=1)
    scale = np.float32(1.0 / math.sqrt(D))
    s = np.einsum("ihd,jhd->hij", q.astype(np.float32), K) * scale    # [NH, S, total]
    qpos = start_pos + np.arange(S)
    mask = pos[None, :] > qpos[:, None]
    s = np.where(mask[None], -np.inf, s)
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("hij,jhd->ihd", p, V)


# ---------------------------------------------------------------------------------------------
# RoPE -- table of engine/scheduler.py:36-48, kernel of src/fused_rope.cu:6-81
# ---------------------------------------------------------------------------------------------
def rope_table(max_seq_len: int, head_dim: int, theta: float = 1000000.0):
    """cos/sin tables [max_seq_len, head_dim/2] float32 (engine/scheduler.py:36-48).

    inv_freq = 1 / theta^(arange(0, D, 2)/D); freqs = outer(t, inv_freq); cos/sin of freqs.
    """
    exponent = np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)
    inv_freq = (np.float32(1.0) / np.power(np.float32(theta), exponent, dtype=np.float32)).astype(np.float32)
    t = np.arange(max_seq_len, dtype=np.float32)
    freqs = (t[:, None] * inv_freq[None, :]).astype(np.float32)
    return np.cos(freqs).astype(np.float32), np.sin(freqs).astype(np.float32)


def rope_inplace(q: np.ndarray, k: np.ndarray, cos: np.ndarray, sin: np.ndarray,
                 pos: np.ndarray) -> None:
    """Rotate-half RoPE on q [T, NH, D] and k [T, KVH, D] in place (src/fused_rope.cu:24-79).

    Pairs are (d, d + D/2); out1 = x1*c - x2*s, out2 = x1*s + x2*c with c = cos[pos, d].
    """
    half = q.shape[-1] // 2
    c = cos[pos][:, None, :]
    s = sin[pos][:, None, :]
    for x in (q, k):
        x1 = x[..., :half].astype(np.float32).copy()
        x2 = x[..., half:].astype(np.float32).copy()
        x[..., :half] = x1 * c - x2 * s
        x[..., half:] = x1 * s + x2 * c


# ---------------------------------------------------------------------------------------------
# SwiGLU -- src/fused_swiglu.cu:10-54 and :56-93
# ---------------------------------------------------------------------------------------------
def swiglu(x: np.ndarray) -> np.ndarray:
    """[..., 2I] (gate half first) -> [..., I]: silu(gate) * up (fused_swiglu.cu:39-50)."""
    inter = x.shape[-1] // 2
    g = x[..., :inter].astype(np.float32)
    u = x[..., inter:].astype(np.float32)
    return (g / (np.float32(1.0) + np.exp(-g))) * u


# ---------------------------------------------------------------------------------------------
# RMSNorm -- models/qwen_25.py:24-36
# ---------------------------------------------------------------------------------------------
def rmsnorm(x: np.ndarray, weight: np.ndarray, eps: float = 1e-6, round_fn=None) -> np.ndarray:
    """w * (x * rsqrt(mean(x^2) + eps)) computed in float32 (models/qwen_25.py:30-36).

    ``round_fn`` (optional) rounds the normalised row to the model dtype before the weight
    multiply, as the reference's ``weight * hidden_states.to(input_dtype)`` does (:36)."""
    xf = x.astype(np.float32)
    var = np.mean(xf * xf, axis=-1, keepdims=True)
    rstd = (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    xhat = xf * rstd
    if round_fn is not None:
        xhat = round_fn(xhat)
    return weight.astype(np.float32) * xhat
