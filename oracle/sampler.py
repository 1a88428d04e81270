"""Restatement of the reference sampler ``ContinuousBatcher._sample_next_token``
(engine/scheduler.py:104-156) in numpy float32.

``torch.multinomial``'s random stream cannot be reproduced, so the restatement returns the
filtered distribution it samples from, plus an explicit inverse-CDF draw for a given uniform
``u`` (the draw the device sampler makes, candidates in descending-logit order).
"""
from __future__ import annotations

import numpy as np


def _softmax(x: np.ndarray) -> np.ndarray:
    m = np.max(x, axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    e = np.exp(x - m)
    return e / e.sum(axis=-1, keepdims=True)


def filter_logits(logits: np.ndarray, temps, top_ks, top_ps) -> np.ndarray:
    """Temperature, top-k and top-p filtering of scheduler.py:111-146; returns the filtered
    float32 logits [B, V] with removed entries at -inf.

    Kept reference behaviour:
      * temperature 0 divides by 1 (:114-115);
      * top_k <= 0 means the whole vocabulary (:117);
      * the per-row cutoff is ``where(k_mask, topk_values, -inf).min()`` (:126-127), so a row
        whose top_k is smaller than the batch's largest top_k gets cutoff -inf, i.e. no top-k
        filtering at all; values equal to the cutoff are kept (:128);
      * top-p runs over the descending sort of every row whenever any row has p < 1 (:131-146):
        remove where cumsum(softmax) > p, shifted right by one, first entry always kept.
    """
    x = np.array(logits, dtype=np.float32, copy=True)
    B, V = x.shape
    t = np.asarray(temps, dtype=np.float32).reshape(B, 1)
    x = x / np.where(t == 0.0, np.float32(1.0), t)
    kv = [min(int(k), V) if int(k) > 0 else V for k in top_ks]
    max_k = max(kv)
    if max_k < V:
        topv = -np.sort(-x, axis=-1)[:, :max_k]
        kmask = np.arange(max_k)[None, :] < np.asarray(kv)[:, None]
        cutoff = np.where(kmask, topv, -np.inf).min(axis=-1, keepdims=True)
        x[x < cutoff] = -np.inf
    p = np.asarray(top_ps, dtype=np.float32).reshape(B)
    if (p < 1.0).any():
        order = np.argsort(-x, axis=-1, kind="stable")
        sl = np.take_along_axis(x, order, axis=-1)
        cp = np.cumsum(_softmax(sl), axis=-1)
        remove = cp > p[:, None]
        remove[:, 1:] = remove[:, :-1].copy()
        remove[:, 0] = False
        rm = np.zeros_like(remove)
        np.put_along_axis(rm, order, remove, axis=-1)
        x[rm] = -np.inf
    return x


def sample_probs(logits, temps, top_ks, top_ps) -> np.ndarray:
    """The distribution ``torch.multinomial`` draws from (scheduler.py:149-152)."""
    return _softmax(filter_logits(logits, temps, top_ks, top_ps))


def greedy(logits, temps=None, top_ks=None, top_ps=None) -> np.ndarray:
    """``argmax`` of the filtered logits (scheduler.py:153), first index on ties."""
    x = np.asarray(logits, np.float32)
    if temps is not None:
        x = filter_logits(x, temps, top_ks, top_ps)
    return np.argmax(x, axis=-1).astype(np.int64)


def draw(probs_row: np.ndarray, logits_row: np.ndarray, u: float) -> int:
    """Inverse-CDF draw over the kept tokens in descending-logit order (ties: lower index
    first): the first token whose cumulative probability exceeds ``u``.  This is the draw
    the device sampler makes for a uniform ``u`` in [0, 1)."""
    keep = np.nonzero(probs_row > 0)[0]
    order = keep[np.lexsort((keep, -logits_row[keep]))]
    c = np.cumsum(probs_row[order].astype(np.float64))
    idx = int(np.searchsorted(c, u * c[-1], side="right"))
    return int(order[min(idx, len(order) - 1)])


def sample_next_token(logits, temps, top_ks, top_ps, uniforms) -> list[int]:
    """Full sampler: greedy where temperature == 0 (scheduler.py:153-156), else the draw."""
    x = filter_logits(logits, temps, top_ks, top_ps)
    probs = _softmax(x)
    out = []
    for b in range(x.shape[0]):
        if float(temps[b]) == 0.0:
            out.append(int(np.argmax(x[b])))
        else:
            out.append(draw(probs[b], x[b], float(uniforms[b])))
    return out
