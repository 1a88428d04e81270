"""Drop-in for the reference's ``custom_swiglu`` extension module (src/swiglu_binding.cpp:3-6,
src/fused_swiglu.cu:56-93): ``forward(input[..., 2I]) -> Tensor[..., I]`` = silu(gate) * up,
gate half first.  fp16 (the reference's dtype) and bf16 are accepted; the reference's checks
and messages are kept (fused_swiglu.cu:57-68).
"""
from __future__ import annotations

import torch

from . import _native as N


def forward(input: torch.Tensor) -> torch.Tensor:  # noqa: A002 - reference argument name
    if not input.is_cuda:
        raise RuntimeError("Input tensor must be on CUDA.")
    if input.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("Input tensor must be FP16 (or BF16).")
    if not input.is_contiguous():
        raise RuntimeError("Input tensor must be contiguous in memory.")
    total = input.shape[-1]
    if total % 2 != 0:
        raise RuntimeError("Input hidden dimension must be even.")
    inter = total // 2
    if inter % 8 != 0:
        raise RuntimeError("Hidden size must be a multiple of 8 for vectorized access.")
    out = torch.empty(*input.shape[:-1], inter, dtype=input.dtype, device=input.device)
    tokens = input.numel() // total if total else 0
    N.check(N.lib().ti_swiglu(out.data_ptr(), input.data_ptr(), tokens, inter,
                              N.dtype_code(input.dtype), N.stream_of(input)))
    return out
