"""The paged-attention entry point that allocates nothing (ti_paged_attention_decode_noalloc).

It exists for callers that cannot call cudaMalloc -- for example a serving process that has
already given all of its device memory to the KV pool and to an allocator it does not control,
or code on a path where a device allocation would stall the GPU.  Instead of a caller-provided
workspace it uses a fixed 16 MiB scratch array inside the library.  These checks call it
through the C ABI and compare it with the regular entry point (caller-provided workspace) on
the same inputs, for two calls in a row, with the attention tolerance used by the other GPU
tests; they also check that an over-size batch is refused with a clear message.  Kept in the
last-collected test file so that a run stopping at the first failure has run everything else.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(seed, B, NB, ctx_hi):
    rng = np.random.default_rng(seed)
    bs, NH, KVH, D = 16, 14, 2, 64
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
    q = torch.randn(B, NH, D, device=dev, dtype=torch.bfloat16, generator=None)
    k = torch.randn(NB, KVH, bs, D, device=dev, dtype=torch.bfloat16)
    v = torch.randn(NB, KVH, bs, D, device=dev, dtype=torch.bfloat16)
    return q, k, v, torch.from_numpy(bt).to(dev), torch.from_numpy(ctx).to(dev), mb


def _call(lib, fn, out, q, k, v, bt, ctx, mb, *extra):
    B, NH, D = q.shape
    NB, KVH = k.shape[0], k.shape[1]
    args = [out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(),
            NB, bt.data_ptr(), bt.stride(0), None, ctx.data_ptr(), B, NH, KVH, D, 16, mb, 0]
    return getattr(lib, fn)(*args, *extra, torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_workspace_entry_point(cuda_device):
    from tiny_infra_b200 import _native as N
    lib = N.lib()
    torch.manual_seed(0)
    for call, (seed, B, NB, ctx_hi) in enumerate([(1, 96, 9000, 2048), (2, 40, 3000, 1200)]):
        q, k, v, bt, ctx, mb = _case(seed, B, NB, ctx_hi)
        need = lib.ti_paged_attention_workspace_bytes(B, 14, 2, 64, mb, 0)
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
        assert (err <= 2e-3 + 2.0 ** -9 * np.abs(r)).all(), (call, float(err.max()))
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
