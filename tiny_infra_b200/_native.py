"""ctypes binding of ``libtiny_infra_b200.so`` (the C ABI declared in include/tiny_infra_b200.h).

The library is built in-tree by ``python -m tiny_infra_b200.build``.  There is no fallback: if
the library is missing, every op raises ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib",
                        "libtiny_infra_b200.so")

TI_DTYPE_BF16, TI_DTYPE_FP16, TI_DTYPE_FP32 = 0, 1, 2
_DT = {torch.bfloat16: TI_DTYPE_BF16, torch.float16: TI_DTYPE_FP16, torch.float32: TI_DTYPE_FP32}

P, I64, I32, SZ, F32, U64 = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t,
                             ctypes.c_float, ctypes.c_uint64)

# name -> (restype, argtypes); every symbol include/tiny_infra_b200.h declares is listed here.
SIGNATURES: dict[str, tuple] = {
    "ti_last_error": (ctypes.c_char_p, []),
    "ti_version": (I32, []),
    "ti_launch_count": (U64, []),
    "ti_device_status": (I32, [ctypes.POINTER(ctypes.c_uint), I32, P]),
    "ti_paged_attention_workspace_bytes": (SZ, [I32, I32, I32, I32, I32, I32]),
    "ti_paged_attention_decode": (I32, [P, I64, P, I64, P, P, I64, P, I64, P, P, I32, I32, I32,
                                        I32, I32, I32, I32, I32, P, SZ, P]),
    "ti_paged_attention_decode_noalloc": (I32, [P, I64, P, I64, P, P, I64, P, I64, P, P, I32, I32,
                                                I32, I32, I32, I32, I32, P]),
    "ti_rope_inplace": (I32, [P, I64, P, I64, P, P, P, I32, I32, I32, I32, I32, P]),
    "ti_rope_kv_append": (I32, [P, I64, P, P, P, P, P, P, I32, I32, I32, I32, I32, I32, P]),
    "ti_swiglu": (I32, [P, P, I64, I32, I32, P]),
    "ti_rmsnorm": (I32, [P, P, I32, P, F32, I32, I32, I32, P]),
    "ti_embedding": (I32, [P, P, P, I32, I32, I64, I32, P]),
    "ti_gemm": (I32, [I32, P, I64, P, I64, I32, I32, I32, P, I64, P, P, P, I32, I32, I32, P]),
    "ti_paged_prefill_attention": (I32, [P, I64, P, I64, P, P, I64, P, I64, P, P, P, P, P, I32,
                                         I32, I32, I32, I32, I32, P]),
    "ti_decode_prepare": (I32, [P, P, P, P, P, I64, I32, I32, I64, I32, P, P, P, P, P, I32, I64,
                                I32, I32, P]),
    "ti_argmax_finish": (I32, [P, P, I32, I32, P, P, P, I32, P]),
    "ti_kv_scatter": (I32, [P, P, P, I64, I64, P, I64, I64, P, I32, I64, I32, I32, I32, I32, P]),
    "ti_quantize_rows_int8": (I32, [P, I64, I32, I32, P, I64, P, I32, P]),
    "ti_lm_head_argmax_int8": (I32, [P, I64, P, I64, P, I32, I32, I32, P, P, I32, P]),
    "ti_gemm_qkv_rope": (I32, [P, I64, P, I64, P, I32, I32, I32, I32, I32, P, I64, P, P, P, P, P,
                               P, I32, I32, P]),
    "ti_sample": (I32, [P, I64, I32, I32, I32, P, P, P, P, P, P, P, I32, P]),
    "ti_paged_attention_plan_bytes": (SZ, [I32]),
    "ti_paged_attention_plan": (I32, [P, I64, P, P, I32, I32, I32, I32, I32, I64, P, SZ, P]),
    "ti_paged_attention_plan_ex": (I32, [P, I64, P, P, I32, I32, I32, I32, I32, I64, P, SZ, I32,
                                         I32, I32, P]),
    "ti_paged_attention_decode_planned": (I32, [P, I64, P, I64, P, P, I64, P, I64, P, P, I32, I32,
                                                I32, I32, I32, I32, I32, P, SZ, P, P]),
    "ti_paged_attention_decode_planned_ex": (I32, [P, I64, P, I64, P, P, I64, P, I64, P, P, I32,
                                                   I32, I32, I32, I32, I32, I32, P, SZ, P, I32,
                                                   P]),
}

TI_EPI_STORE, TI_EPI_SWIGLU, TI_EPI_RESIDUAL, TI_EPI_ARGMAX = 0, 1, 2, 3
TI_EPI_SWIGLU16 = 5
TI_EPI_RESIDUAL_DET = 6
# device status bits (ti_device_status)
TI_DEVERR_ATTN_WAIT, TI_DEVERR_GEMM_WAIT, TI_DEVERR_PREFILL_WAIT, TI_DEVERR_ATTN_PLAN = 1, 2, 4, 8
TI_DEVERR_BAD_INPUT = 16
# ti_paged_attention_decode_planned_ex / ti_paged_attention_plan_ex flags
TI_ATTN_EARLY_KV = 1
TI_ATTN_PLAN_AFTER_QKV = 1

_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load the native library once (raises RuntimeError if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"tiny_infra_b200 native library not found at {LIB_PATH}; "
                    "build it with `python -m tiny_infra_b200.build`")
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(rc: int) -> None:
    if rc != 0:
        msg = lib().ti_last_error().decode(errors="replace")
        raise RuntimeError(msg or f"tiny_infra_b200 call failed with code {rc}")


def dtype_code(t: torch.dtype) -> int:
    try:
        return _DT[t]
    except KeyError:
        raise RuntimeError(f"unsupported dtype {t}") from None


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def launch_count() -> int:
    return int(lib().ti_launch_count())


def device_status(clear: bool = True, device: torch.device | None = None) -> int:
    """TI_DEVERR_* bits raised by kernels (bounded waits that gave up, rejected plans) since
    the last clear."""
    bits = ctypes.c_uint(0)
    s = torch.cuda.current_stream(device).cuda_stream
    check(lib().ti_device_status(ctypes.byref(bits), int(clear), s))
    return int(bits.value)


class Workspace:
    """Zero-initialised scratch buffer per device -- and per stream when ``get`` is given one --
    that grows on demand (kernels that use arrival counters leave them at zero, so a buffer is
    reusable by every later launch on its stream).  Launches on different streams get different
    buffers, so they may overlap on the GPU; a buffer is created on its own stream, so its
    zero fill is ordered before that stream's first launch."""

    def __init__(self) -> None:
        self._buf: dict[tuple, torch.Tensor] = {}
        self._lock = threading.Lock()

    def get(self, device: torch.device, nbytes: int, stream: int | None = None) -> torch.Tensor:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        key = (idx, stream)
        with self._lock:
            buf = self._buf.get(key)
            if buf is None or buf.numel() < nbytes:
                buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
                self._buf[key] = buf
        return buf
