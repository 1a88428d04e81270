"""Drop-in for the reference's ``custom_rope`` extension module (src/rope_binding.cpp:3-11,
src/fused_rope.cu:84-128): ``apply_inplace(q, k, cos, sin, pos_ids)``.

Rotate-half RoPE in place on q [T, NH, D] and k [T, KVH, D] with float32 cos/sin tables
[max_pos, D/2] and int32 positions.  fp16 (the reference's dtype) and bf16 are accepted; the
error messages of the reference's checks (fused_rope.cu:92-95) are kept.
"""
from __future__ import annotations

import torch

from . import _native as N


def apply_inplace(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                  pos_ids: torch.Tensor) -> None:
    if not (q.is_cuda and k.is_cuda and cos.is_cuda and sin.is_cuda and pos_ids.is_cuda):
        raise RuntimeError("All tensors must be CUDA tensors.")
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype:
        raise RuntimeError("Query and Key tensors must be of type half (or bfloat16).")
    if cos.dtype != torch.float32 or sin.dtype != torch.float32:
        raise RuntimeError("Cosine and Sine tensors must be of type float.")
    if pos_ids.dtype != torch.int32:
        raise RuntimeError("Position IDs tensor must be of type int.")
    if q.dim() != 3 or k.dim() != 3 or q.shape[0] != k.shape[0] or q.shape[2] != k.shape[2]:
        raise RuntimeError("q must be [T, NH, D] and k [T, KVH, D]")
    T, NH, D = q.shape
    KVH = k.shape[1]
    if pos_ids.numel() != T:
        raise RuntimeError("pos_ids must hold one position per token")
    if not (q.stride(2) == 1 and q.stride(1) == D and k.stride(2) == 1 and k.stride(1) == D):
        raise RuntimeError("q and k must have contiguous [heads, D] rows")
    if not (cos.is_contiguous() and sin.is_contiguous() and cos.shape[-1] == D // 2):
        raise RuntimeError("cos/sin must be contiguous [max_pos, D/2]")
    pos = pos_ids.contiguous()
    N.check(N.lib().ti_rope_inplace(q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0),
                                    cos.data_ptr(), sin.data_ptr(), pos.data_ptr(), T, NH, KVH,
                                    D, N.dtype_code(q.dtype), N.stream_of(q)))
