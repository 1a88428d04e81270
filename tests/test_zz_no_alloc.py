"""The paged-attention entry point that allocates nothing (ti_paged_attention_decode_noalloc).

It exists for callers that cannot call cudaMalloc -- for example a serving process that has
already given all of its device memory to the KV pool and to an allocator it does not control,
or code on a path where a device allocation would stall the GPU.  Instead of a caller-provided
workspace it uses a fixed 16 MiB scratch array inside the library.  These checks call it
through the C ABI and compare it with the regular entry point (caller-provided workspace) on
the same inputs, for several calls in a row of different shapes and dtypes (bf16 and fp16,
head_dim 64 and 128, with and without split-K), with the attention tolerance used by the other
GPU tests; they also check that an over-size batch is refused with a clear message.  Kept in the
last-collected test file so that a run stopping at the first failure has run everything else.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(seed, B, NB, ctx_hi, NH=14, KVH=2, D=64, dtype=torch.bfloat16):
    rng = np.random.default_rng(seed)
    bs = 16
    ctx = rng.integers(1, ctx_hi + 1, B).astype(np.int32)
    mb = (ctx_hi + bs - 1) // bs
    perm = rng.permutation(NB)
    bt = np.full((B, mb), -1, np.int32)
    off = 0
    for b in range(B):
        n = (int(ctx[b]) + bs - 1) // bs
        bt[b, :n] = perm[off:off + n]
        off += n
    dev = torch.device("cuda:0")
    q = torch.randn(B, NH, D, device=dev, dtype=dtype, generator=None)
    k = torch.randn(NB, KVH, bs, D, device=dev, dtype=dtype)
    v = torch.randn(NB, KVH, bs, D, device=dev, dtype=dtype)
    return q, k, v, torch.from_numpy(bt).to(dev), torch.from_numpy(ctx).to(dev), mb


def _call(lib, fn, out, q, k, v, bt, ctx, mb, *extra):
    B, NH, D = q.shape
    NB, KVH = k.shape[0], k.shape[1]
    dt = 1 if q.dtype == torch.float16 else 0
    args = [out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(),
            NB, bt.data_ptr(), bt.stride(0), None, ctx.data_ptr(), B, NH, KVH, D, 16, mb, dt]
    return getattr(lib, fn)(*args, *extra, torch.cuda.current_stream().cuda_stream)


CASES = [  # (seed, batch, pool blocks, max ctx, query heads, kv heads, head_dim, dtype)
    (1, 96, 9000, 2048, 14, 2, 64, torch.bfloat16),    # the decode step's kernel (v5)
    (2, 40, 3000, 1200, 14, 2, 64, torch.bfloat16),    # a second shape on the same array
    (3, 40, 3000, 1200, 14, 2, 64, torch.float16),     # fp16, the reference's dtype
    (4, 40, 3000, 1200, 16, 2, 128, torch.bfloat16),   # head_dim 128: split-K partitions (v1)
    (5, 3000, 48100, 256, 16, 2, 128, torch.bfloat16), # head_dim 128, <= 16 blocks: no split
]


def test_noalloc_matches_workspace_entry_point(cuda_device):
    """Each case on the no-alloc entry point and on the workspace one, in this order, so every
    call after the first finds the array as another shape left it."""
    from tiny_infra_b200 import _native as N
    lib = N.lib()
    torch.manual_seed(0)
    for call, (seed, B, NB, ctx_hi, NH, KVH, D, dt) in enumerate(CASES):
        q, k, v, bt, ctx, mb = _case(seed, B, NB, ctx_hi, NH, KVH, D, dt)
        need = lib.ti_paged_attention_workspace_bytes(B, NH, KVH, D, mb, 0)
        ws = torch.zeros(need, dtype=torch.uint8, device=cuda_device)
        ref = torch.full_like(q, 5.0)
        assert _call(lib, "ti_paged_attention_decode", ref, q, k, v, bt, ctx, mb, 0,
                     ws.data_ptr(), need) == 0, lib.ti_last_error()
        got = torch.full_like(q, 5.0)
        assert _call(lib, "ti_paged_attention_decode_noalloc", got, q, k, v, bt, ctx, mb) == 0, \
            lib.ti_last_error()
        torch.cuda.synchronize()
        r, g = ref.float().cpu().numpy(), got.float().cpu().numpy()
        err = np.abs(g - r)
        half_ulp = 2.0 ** -9 if dt == torch.bfloat16 else 2.0 ** -12
        assert (err <= 2e-3 + half_ulp * np.abs(r)).all(), (call, float(err.max()))
        assert N.device_status() == 0


def test_noalloc_rejects_oversize_batch(cuda_device):
    from tiny_infra_b200 import _native as N
    lib = N.lib()
    B, mb = 4096, 2048                       # needs far more than the 16 MiB scratch
    dummy = torch.zeros(16, dtype=torch.bfloat16, device=cuda_device)
    rc = lib.ti_paged_attention_decode_noalloc(
        dummy.data_ptr(), 896, dummy.data_ptr(), 896, dummy.data_ptr(), dummy.data_ptr(), 1,
        dummy.data_ptr(), mb, None, dummy.data_ptr(), B, 14, 2, 64, 16, mb, 0,
        torch.cuda.current_stream().cuda_stream)
    assert rc == 4 and b"static scratch holds" in lib.ti_last_error()
