"""Device sampling for the scheduler: drop-in for ``ContinuousBatcher._sample_next_token``
(engine/scheduler.py:104-156) on logits that stay on the GPU.

``sample_next_token(logits, requests)`` takes the [B, V] (or [B, S, V], last position used)
logits of a batch and the batch's requests (``temperature``, ``top_k``, ``p_value``) and
returns their next tokens, computed by ``ti_sample`` (one CTA per row: radix selects for the
top-k cutoff, the top-p boundary and the inverse-CDF draw; no vocabulary sort).  Temperature 0
rows take the argmax.  The reference's batch-level rules are applied here when the per-row
parameters are built (:class:`SamplingParams`): top-k cuts only the rows whose top_k equals the
batch's largest top_k (and only if that is below the vocabulary size), top-p runs in every row
once any row of the batch has p < 1.

Randomness: the reference calls ``torch.multinomial`` on the global generator.  Here each
request owns a counter-based ``numpy.random.Philox`` stream, from which one uniform per sampled
token is drawn on the host and passed to the kernel with the step's inputs -- a request's tokens
do not depend on which other requests share its batches.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _native as N


def effective_top_k(top_k: int, vocab: int) -> int:
    """engine/scheduler.py:119: top_k <= 0 means the whole vocabulary."""
    return min(int(top_k), vocab) if int(top_k) > 0 else vocab


class SamplingParams:
    """Per-row kernel parameters of one batch (the batch as the reference samples it)."""

    def __init__(self, temps, top_ks, top_ps, uniforms, vocab: int):
        self.temps = np.asarray(temps, np.float32)
        ks = np.asarray([effective_top_k(k, vocab) for k in top_ks], np.int32)
        max_k = int(ks.max()) if len(ks) else vocab
        # top-k cuts the rows whose top_k is the batch's largest (scheduler.py:123-130)
        self.cut_ks = np.where((ks == max_k) & (max_k < vocab), ks, 0).astype(np.int32)
        ps = np.asarray(top_ps, np.float32)
        # top-p runs in every row once any row has p < 1 (scheduler.py:133-146)
        self.top_ps = ps if bool((ps < 1.0).any()) else np.ones_like(ps)
        self.uniforms = np.asarray(uniforms, np.float32)
        self.all_greedy = bool((self.temps == 0.0).all())

    @staticmethod
    def concat(parts: list["SamplingParams"]) -> "SamplingParams":
        """Rows of several batches (each keeping its own batch rules) in one launch."""
        out = SamplingParams.__new__(SamplingParams)
        out.temps = np.concatenate([p.temps for p in parts])
        out.cut_ks = np.concatenate([p.cut_ks for p in parts])
        out.top_ps = np.concatenate([p.top_ps for p in parts])
        out.uniforms = np.concatenate([p.uniforms for p in parts])
        out.all_greedy = bool((out.temps == 0.0).all())
        return out

    def packed(self) -> np.ndarray:
        """[4, B] float32 block (temps, cut_ks as int32 bits, top_ps, uniforms): one copy."""
        B = len(self.temps)
        out = np.empty((4, B), np.float32)
        out[0] = self.temps
        out[1] = self.cut_ks.view(np.float32)
        out[2] = self.top_ps
        out[3] = self.uniforms
        return out


def launch_sample(logits: torch.Tensor, params_dev: torch.Tensor, out_tokens: torch.Tensor,
                  slots: torch.Tensor | None = None, seq_len: torch.Tensor | None = None,
                  seq_inc: int = 0, rows: int | None = None, stream: int | None = None) -> None:
    """Run ``ti_sample`` on device tensors: ``logits`` [B, V] (row stride logits.stride(0)),
    ``params_dev`` the [4, >=B] float32 block of :meth:`SamplingParams.packed` on the device."""
    B = logits.shape[0] if rows is None else rows
    V = logits.shape[-1]
    if stream is None:
        stream = torch.cuda.current_stream(logits.device).cuda_stream
    pd = params_dev
    N.check(N.lib().ti_sample(
        logits.data_ptr(), logits.stride(0), N.dtype_code(logits.dtype), B, V,
        pd[0].data_ptr(), pd[1].data_ptr(), pd[2].data_ptr(), pd[3].data_ptr(),
        out_tokens.data_ptr(), slots.data_ptr() if slots is not None else None,
        seq_len.data_ptr() if seq_len is not None else None, seq_inc, stream))


def request_uniforms(requests) -> list[float]:
    """One uniform per request from its own stream (``rng``), else from numpy's default."""
    return [float(r.rng.random()) if getattr(r, "rng", None) is not None
            else float(np.random.random()) for r in requests]


def sample_next_token(logits: torch.Tensor, requests, uniforms=None) -> list[int]:
    """engine/scheduler.py:104-156 on the device, the requests forming one batch."""
    if logits.dim() == 3:
        logits = logits[:, -1, :]
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    B, V = logits.shape
    if uniforms is None:
        uniforms = request_uniforms(requests)
    sp = SamplingParams([r.temperature for r in requests], [r.top_k for r in requests],
                        [r.p_value for r in requests], uniforms, V)
    pd = torch.from_numpy(sp.packed()).to(logits.device)
    out = torch.empty(B, dtype=torch.int32, device=logits.device)
    launch_sample(logits, pd, out)
    return [int(x) for x in out.cpu().tolist()]
