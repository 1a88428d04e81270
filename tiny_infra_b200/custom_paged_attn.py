"""Drop-in for the reference's ``custom_paged_attn`` extension module
(src/attention_binding.cpp:3-13, src/attention.cu:156-197).

``launch_paged_attention(out, q, k_cache, v_cache, block_tables, context_lens, block_size)``
writes ``out`` in place, like the reference; it runs the sm_100a split-K kernel of
``csrc/paged_attention.cu`` on the current CUDA stream and accepts fp16 (the reference's
dtype) and bf16.  Argument errors raise ``RuntimeError`` as the reference's TORCH_CHECKs do.

Its split-K scratch is kept per (device, stream): calls on different streams may run at the
same time, as calls of the reference op (which keeps no state) may.
"""
from __future__ import annotations

import torch

from . import _native as N

_ws = N.Workspace()


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def launch_paged_attention(out: torch.Tensor, q: torch.Tensor, k_cache: torch.Tensor,
                           v_cache: torch.Tensor, block_tables: torch.Tensor,
                           context_lens: torch.Tensor, block_size: int, *,
                           row_index: torch.Tensor | None = None,
                           partition_blocks: int = 0) -> None:
    """Single-query GQA attention over the paged pool (reference src/attention.cu:54-154).

    q, out: [B, NH, D]; k_cache/v_cache: [num_blocks, KVH, block_size, D]; block_tables
    [B, max_blocks] int32 (or any rows, selected by ``row_index``); context_lens [B] int32.
    """
    for name, t in (("out", out), ("q", q), ("k_cache", k_cache), ("v_cache", v_cache),
                    ("block_tables", block_tables), ("context_lens", context_lens)):
        _check(t.is_cuda, f"{name} must be a CUDA tensor")
    _check(q.dim() == 3 and out.dim() == 3 and out.shape == q.shape, "q and out must be [B, NH, D]")
    _check(k_cache.dim() == 4 and v_cache.shape == k_cache.shape,
           "k_cache/v_cache must be [num_blocks, num_kv_heads, block_size, head_dim]")
    _check(q.dtype == out.dtype == k_cache.dtype == v_cache.dtype and q.dtype in
           (torch.float16, torch.bfloat16), "q, out and the caches must share dtype fp16 or bf16")
    _check(block_tables.dtype == torch.int32 and context_lens.dtype == torch.int32,
           "block_tables and context_lens must be int32")
    B, NH, D = q.shape
    NB, KVH, bs, Dk = k_cache.shape
    _check(Dk == D and bs == block_size, "cache shape does not match q / block_size")
    _check(q.stride(2) == 1 and q.stride(1) == D and out.stride(2) == 1 and out.stride(1) == D,
           "q and out must have contiguous [NH, D] rows")
    _check(k_cache.is_contiguous() and v_cache.is_contiguous(), "caches must be contiguous")
    _check(block_tables.dim() == 2 and block_tables.stride(1) == 1, "block_tables must be 2-D")
    _check(context_lens.is_contiguous() and context_lens.numel() == B, "context_lens must be [B]")
    if row_index is None:
        _check(block_tables.shape[0] >= B, "block_tables has fewer rows than the batch")
    if B == 0:
        return
    max_blocks = block_tables.shape[1]
    lib = N.lib()
    need = lib.ti_paged_attention_workspace_bytes(B, NH, KVH, D, max_blocks, partition_blocks)
    stream = N.stream_of(q)
    ws = _ws.get(q.device, need, stream)       # one split-K scratch per (device, stream)
    N.check(lib.ti_paged_attention_decode(
        out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0), k_cache.data_ptr(),
        v_cache.data_ptr(), NB, block_tables.data_ptr(), block_tables.stride(0),
        row_index.data_ptr() if row_index is not None else None, context_lens.data_ptr(), B, NH,
        KVH, D, block_size, max_blocks, N.dtype_code(q.dtype), partition_blocks, ws.data_ptr(),
        ws.numel(), stream))
