"""Weight-only INT8 for the lm_head, restated in numpy (test infrastructure, never the product).

The reference names weight-only INT8/INT4 quantised projections as its next step
(README.md:156-157) but ships no code for it, so there is no reference behaviour to follow: this
module is the definition the CUDA path (``ti_quantize_rows_int8``, ``ti_lm_head_argmax_int8``)
is checked against -- symmetric per-row scales, round to nearest even, the logits of the
dequantised weights computed in float32 (models/qwen_25.py:250 with W = scale * q).
"""
from __future__ import annotations

import numpy as np


def quantize_rows_int8(w: np.ndarray):
    """Per row r: scale = max|w[r]| / 127 (1 for an all-zero row), q = rint(w / scale) clamped to
    [-127, 127].  float32 arithmetic (IEEE division, ties to even), so the result is bit-exact
    with the device kernel.  Returns (q int8 [rows, cols], scale float32 [rows])."""
    w = np.asarray(w, np.float32)
    amax = np.abs(w).max(axis=1)
    scale = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint(w / scale[:, None]), -127, 127).astype(np.int8)
    return q, scale


def int8_logits(x: np.ndarray, q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """logits[m, n] = scale[n] * sum_k x[m, k] q[n, k] in float32 (x: the final normed hidden
    rows, bf16 values as float32)."""
    acc = np.asarray(x, np.float32) @ q.astype(np.float32).T
    return (acc * scale[None, :]).astype(np.float32)
