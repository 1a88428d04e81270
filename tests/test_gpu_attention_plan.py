"""The per-step attention plan (ti_paged_attention_plan) and the attention call that reads it
(ti_paged_attention_decode_planned), through the C ABI.

* the planned call runs the same kernel with the same split of the batch as the plain call, so
  its output must equal the plain call's bit for bit (ragged batches, long contexts cut into
  many pieces, four kv heads, negative and out-of-pool block-table entries, empty rows);
* a plan of another batch is rejected on the device (TI_DEVERR_ATTN_PLAN), the context stays
  usable; the plan buffer is sized for the larger batch so every read stays inside it;
* a shape the planned kernel does not serve (head_dim 128) gets a zero header and the planned
  call equals the plain one.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(seed, B, NH, KVH, D, NB, lo, hi, dev):
    rng = np.random.default_rng(seed)
    bs = 16
    ctx = rng.integers(lo, hi + 1, B).astype(np.int32)
    mb = (hi + bs - 1) // bs
    perm = rng.permutation(NB)
    bt = np.full((B, mb), -1, np.int32)
    off = 0
    for b in range(B):
        n = (int(ctx[b]) + bs - 1) // bs
        bt[b, :n] = perm[off:off + n]
        off += n
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(B, NH, D, device=dev, generator=g).bfloat16()
    k = torch.randn(NB, KVH, bs, D, device=dev, generator=g).bfloat16()
    v = torch.randn(NB, KVH, bs, D, device=dev, generator=g).bfloat16()
    return q, k, v, bt, ctx, mb


def _args(q, k, v, bt, ctx, mb, out):
    B, NH, D = q.shape
    NB, KVH = k.shape[0], k.shape[1]
    return [out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(),
            NB, bt.data_ptr(), bt.stride(0), None, ctx.data_ptr(), B, NH, KVH, D, 16, mb]


def _plain_and_planned(lib, N, q, k, v, bt_np, ctx_np, mb, plan_batch=None):
    dev = q.device
    B, NH, D = q.shape
    NB, KVH = k.shape[0], k.shape[1]
    bt, ctx = torch.from_numpy(bt_np).to(dev), torch.from_numpy(ctx_np).to(dev)
    s = torch.cuda.current_stream().cuda_stream
    need = lib.ti_paged_attention_workspace_bytes(B, NH, KVH, D, mb, 0)
    ws = torch.zeros(need, dtype=torch.uint8, device=dev)
    ref = torch.full_like(q, 3.0)
    N.check(lib.ti_paged_attention_decode(*_args(q, k, v, bt, ctx, mb, ref), N.dtype_code(q.dtype),
                                          0, ws.data_ptr(), need, s))
    plan = torch.zeros(lib.ti_paged_attention_plan_bytes(max(B, plan_batch or B)),
                       dtype=torch.uint8, device=dev)
    pb = plan_batch or B
    N.check(lib.ti_paged_attention_plan(bt.data_ptr(), bt.stride(0), None, ctx.data_ptr(), pb, NH,
                                        KVH, D, mb, NB, plan.data_ptr(), plan.numel(), s))
    got = torch.full_like(q, 3.0)
    N.check(lib.ti_paged_attention_decode_planned(*_args(q, k, v, bt, ctx, mb, got),
                                                  N.dtype_code(q.dtype), ws.data_ptr(), need,
                                                  plan.data_ptr(), s))
    torch.cuda.synchronize()
    return ref, got, plan


CASES = [(4, 256, 14, 2, 64, 256 * 128, 128, 2048), (1, 12, 14, 2, 64, 3200, 1, 4096),
         (5, 40, 16, 4, 64, 2000, 1, 700), (6, 3, 14, 2, 64, 64, 1, 300)]


@pytest.mark.parametrize("case", CASES)
def test_planned_equals_plain(cuda_device, case):
    from tiny_infra_b200 import _native as N
    lib = N.lib()
    q, k, v, bt, ctx, mb = _case(*case, dev=cuda_device)
    ref, got, _ = _plain_and_planned(lib, N, q, k, v, bt, ctx, mb)
    assert torch.equal(ref.view(torch.int16), got.view(torch.int16))


def test_planned_edge_cases(cuda_device):
    from tiny_infra_b200 import _native as N
    lib = N.lib()
    q, k, v, bt, ctx, mb = _case(2, 6, 14, 2, 64, 600, 200, 1500, dev=cuda_device)
    ctx[0] = 0
    bt[1, 3] = -1
    bt[2, 20] = -1
    bt[3, 0] = -1
    bt[4, 5] = 600 + 7
    ref, got, _ = _plain_and_planned(lib, N, q, k, v, bt, ctx, mb)
    assert torch.equal(ref.view(torch.int16), got.view(torch.int16))
    assert (got[0].float() == 3.0).all() and torch.isnan(got[3].float()).all()


def test_plan_of_another_batch_is_rejected(cuda_device):
    import ctypes
    from tiny_infra_b200 import _native as N
    lib = N.lib()
    s = torch.cuda.current_stream().cuda_stream
    bits = ctypes.c_uint(0)
    N.check(lib.ti_device_status(ctypes.byref(bits), 1, s))
    q, k, v, bt, ctx, mb = _case(7, 64, 14, 2, 64, 6000, 1, 1500, dev=cuda_device)
    _plain_and_planned(lib, N, q, k, v, bt, ctx, mb, plan_batch=50)
    N.check(lib.ti_device_status(ctypes.byref(bits), 1, s))
    assert bits.value & N.TI_DEVERR_ATTN_PLAN
    # the context is still usable: a matching plan works afterwards
    ref, got, _ = _plain_and_planned(lib, N, q, k, v, bt, ctx, mb)
    assert torch.equal(ref.view(torch.int16), got.view(torch.int16))
    N.check(lib.ti_device_status(ctypes.byref(bits), 1, s))
    assert bits.value == 0


def test_unplanned_shape_gets_zero_header(cuda_device):
    from tiny_infra_b200 import _native as N
    lib = N.lib()
    q, k, v, bt, ctx, mb = _case(3, 5, 8, 2, 128, 300, 1, 900, dev=cuda_device)
    ref, got, plan = _plain_and_planned(lib, N, q, k, v, bt, ctx, mb)
    assert torch.equal(ref.view(torch.int16), got.view(torch.int16))
    assert (plan[:32] == 0).all()


def test_v5_long_ranges(cuda_device, monkeypatch):
    """64 sequences of 76k-90k tokens: more than 2048 stream positions per v5 CTA (the kernel
    holds up to 4096; the planned call loads its slot in two rounds).  Planned equals plain bit
    for bit, both agree with the v2 kernel, and three sequences agree with an fp32 torch
    reference (tolerance: 2e-3 + half a bf16 ulp of the reference)."""
    from tiny_infra_b200 import _native as N
    lib = N.lib()
    B, NH, KVH, D = 64, 14, 2, 64
    rng = np.random.default_rng(8)
    ctx_np = rng.integers(76000, 90001, B).astype(np.int32)
    nblk = (ctx_np + 15) // 16
    assert int(nblk.sum()) > 148 * 2048          # more than 2048 positions per CTA
    NB = int(nblk.sum()) + 16
    mb = int((90000 + 15) // 16)
    perm = rng.permutation(NB).astype(np.int32)
    bt_np = np.full((B, mb), -1, np.int32)
    off = 0
    for b in range(B):
        bt_np[b, :nblk[b]] = perm[off:off + nblk[b]]
        off += int(nblk[b])
    g = torch.Generator(device=cuda_device).manual_seed(8)
    q = torch.randn(B, NH, D, device=cuda_device, generator=g).bfloat16()
    k = torch.randn(NB, KVH, 16, D, device=cuda_device, generator=g).bfloat16()
    v = torch.randn(NB, KVH, 16, D, device=cuda_device, generator=g).bfloat16()
    ref5, got5, _ = _plain_and_planned(lib, N, q, k, v, bt_np, ctx_np, mb)
    assert N.device_status() == 0
    assert torch.equal(ref5.view(torch.int16), got5.view(torch.int16))
    monkeypatch.setenv("TI_PAGED_ATTN_KERNEL", "v2")
    ref2, _, _ = _plain_and_planned(lib, N, q, k, v, bt_np, ctx_np, mb)
    monkeypatch.delenv("TI_PAGED_ATTN_KERNEL")
    a, b2 = got5.float(), ref2.float()
    assert ((a - b2).abs() <= 2e-3 + 2.0 ** -8 * b2.abs()).all(), float((a - b2).abs().max())
    for b in (0, 31, 63):
        n = int(ctx_np[b])
        ids = torch.from_numpy(bt_np[b, :nblk[b]].astype(np.int64)).to(cuda_device)
        kk = k[ids].float().permute(1, 0, 2, 3).reshape(KVH, -1, D)[:, :n]
        vv = v[ids].float().permute(1, 0, 2, 3).reshape(KVH, -1, D)[:, :n]
        qq = q[b].float().view(KVH, NH // KVH, D)
        p = torch.softmax(qq @ kk.transpose(1, 2) / 8.0, dim=-1)
        want = (p @ vv).reshape(NH, D)
        err = (got5[b].float() - want).abs()
        assert (err <= 2e-3 + 2.0 ** -9 * want.abs()).all(), float(err.max())


@pytest.mark.parametrize("case", [(11, 256, 128, 2048), (12, 32, 128, 2048), (13, 7, 1, 300)])
def test_early_kv_after_qkv_append(cuda_device, case):
    """TI_ATTN_EARLY_KV right behind the QKV GEMM that writes q and appends each sequence's new
    token to its last block (the decode step's order): the attention streams the other blocks
    while the GEMM runs and must still see the new q and the appended token.  Its output equals
    the plain call's, run after a full synchronisation on the same q and pool, bit for bit."""
    from tiny_infra_b200 import _native as N
    lib = N.lib()
    seed, B, lo, hi = case
    NH, KVH, D, H = 14, 2, 64, 896
    QKV = (NH + 2 * KVH) * D
    rng = np.random.default_rng(seed)
    ctx_np = rng.integers(lo, hi + 1, B).astype(np.int32)
    nblk = (ctx_np + 15) // 16
    NB = int(nblk.sum()) + 64
    mb = (hi + 15) // 16
    perm = rng.permutation(NB).astype(np.int32)
    bt_np = np.full((B, mb), -1, np.int32)
    off = 0
    for b in range(B):
        bt_np[b, :nblk[b]] = perm[off:off + nblk[b]]
        off += int(nblk[b])
    last = ctx_np - 1
    slots_np = bt_np[np.arange(B), last // 16].astype(np.int64) * 16 + last % 16
    dev = cuda_device
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(B, H, device=dev, generator=g).bfloat16()
    w = (torch.randn(QKV, H, device=dev, generator=g) * 0.05).bfloat16()
    bias = (torch.randn(QKV, device=dev, generator=g) * 0.1).bfloat16()
    k = torch.randn(NB, KVH, 16, D, device=dev, generator=g).bfloat16()
    v = torch.randn(NB, KVH, 16, D, device=dev, generator=g).bfloat16()
    pos = torch.from_numpy(last).to(dev)
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, dtype=torch.float64) / D))
    ang = torch.arange(hi + 1, dtype=torch.float64)[:, None] * inv[None]
    cos = ang.cos().float().to(dev).contiguous()
    sin = ang.sin().float().to(dev).contiguous()
    bt, ctx = torch.from_numpy(bt_np).to(dev), torch.from_numpy(ctx_np).to(dev)
    slots = torch.from_numpy(slots_np).to(dev)
    qkv = torch.zeros(B, QKV, dtype=torch.bfloat16, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    need = lib.ti_paged_attention_workspace_bytes(B, NH, KVH, D, mb, 0)
    ws = torch.zeros(need, dtype=torch.uint8, device=dev)
    plan = torch.zeros(lib.ti_paged_attention_plan_bytes(B), dtype=torch.uint8, device=dev)
    N.check(lib.ti_paged_attention_plan(bt.data_ptr(), bt.stride(0), None, ctx.data_ptr(), B, NH,
                                        KVH, D, mb, NB, plan.data_ptr(), plan.numel(), s))
    torch.cuda.synchronize()                 # the plan is final before the QKV GEMM starts

    def args(out):
        return [out.data_ptr(), NH * D, qkv.data_ptr(), QKV, k.data_ptr(), v.data_ptr(), NB,
                bt.data_ptr(), bt.stride(0), None, ctx.data_ptr(), B, NH, KVH, D, 16, mb,
                N.dtype_code(torch.bfloat16), ws.data_ptr(), need, plan.data_ptr()]

    got = torch.full((B, NH * D), 3.0, dtype=torch.bfloat16, device=dev)
    N.check(lib.ti_gemm_qkv_rope(x.data_ptr(), H, w.data_ptr(), H, bias.data_ptr(), B, H, NH, KVH,
                                 D, qkv.data_ptr(), QKV, k.data_ptr(), v.data_ptr(),
                                 slots.data_ptr(), cos.data_ptr(), sin.data_ptr(), pos.data_ptr(),
                                 16, N.dtype_code(torch.bfloat16), s))
    N.check(lib.ti_paged_attention_decode_planned_ex(*args(got), N.TI_ATTN_EARLY_KV, s))
    torch.cuda.synchronize()
    assert N.device_status() == 0
    ref = torch.full_like(got, 3.0)
    N.check(lib.ti_paged_attention_decode(*args(ref)[:-3], 0, ws.data_ptr(), need, s))
    torch.cuda.synchronize()
    assert torch.equal(ref.view(torch.int16), got.view(torch.int16))
    # a second, unsynchronised round (q and the appended token rewritten by a new GEMM input)
    x2 = torch.randn(B, H, device=dev, generator=g).bfloat16()
    got2 = torch.full_like(got, 3.0)
    N.check(lib.ti_gemm_qkv_rope(x2.data_ptr(), H, w.data_ptr(), H, bias.data_ptr(), B, H, NH,
                                 KVH, D, qkv.data_ptr(), QKV, k.data_ptr(), v.data_ptr(),
                                 slots.data_ptr(), cos.data_ptr(), sin.data_ptr(), pos.data_ptr(),
                                 16, N.dtype_code(torch.bfloat16), s))
    N.check(lib.ti_paged_attention_decode_planned_ex(*args(got2), N.TI_ATTN_EARLY_KV, s))
    ref2 = torch.full_like(got, 3.0)
    torch.cuda.synchronize()
    N.check(lib.ti_paged_attention_decode(*args(ref2)[:-3], 0, ws.data_ptr(), need, s))
    torch.cuda.synchronize()
    assert N.device_status() == 0
    assert not torch.equal(got2.view(torch.int16), got.view(torch.int16))
    assert torch.equal(ref2.view(torch.int16), got2.view(torch.int16))


def test_small_batch_many_pieces(cuda_device):
    """Four sequences of 20k-30k tokens: at small batches v5 cuts each (sequence, kv-head pair)
    into up to 65 pieces so that the blocks spread over every SM, and the merge combines them in
    rounds of 16.  Planned equals plain bit for bit, and every row agrees with an fp32 torch
    reference (tolerance: 2e-3 + half a bf16 ulp of the reference); one row stops at a negative
    block-table entry in its last round of pieces."""
    from tiny_infra_b200 import _native as N
    lib = N.lib()
    B, NH, KVH, D = 4, 14, 2, 64
    rng = np.random.default_rng(21)
    ctx_np = rng.integers(20000, 30001, B).astype(np.int32)
    nblk = (ctx_np + 15) // 16
    NB = int(nblk.sum()) + 16
    mb = int((30000 + 15) // 16)
    perm = rng.permutation(NB).astype(np.int32)
    bt_np = np.full((B, mb), -1, np.int32)
    off = 0
    for b in range(B):
        bt_np[b, :nblk[b]] = perm[off:off + nblk[b]]
        off += int(nblk[b])
    stop_at = int(nblk[2]) - 40                   # row 2 reads up to here (attention.cu:99)
    bt_np[2, stop_at] = -1
    g = torch.Generator(device=cuda_device).manual_seed(21)
    q = torch.randn(B, NH, D, device=cuda_device, generator=g).bfloat16()
    k = torch.randn(NB, KVH, 16, D, device=cuda_device, generator=g).bfloat16()
    v = torch.randn(NB, KVH, 16, D, device=cuda_device, generator=g).bfloat16()
    ref, got, _ = _plain_and_planned(lib, N, q, k, v, bt_np, ctx_np, mb)
    assert N.device_status() == 0
    assert torch.equal(ref.view(torch.int16), got.view(torch.int16))
    for b in range(B):
        n = int(ctx_np[b]) if b != 2 else stop_at * 16
        nb = (n + 15) // 16
        ids = torch.from_numpy(bt_np[b, :nb].astype(np.int64)).to(cuda_device)
        kk = k[ids].float().permute(1, 0, 2, 3).reshape(KVH, -1, D)[:, :n]
        vv = v[ids].float().permute(1, 0, 2, 3).reshape(KVH, -1, D)[:, :n]
        qq = q[b].float().view(KVH, NH // KVH, D)
        p = torch.softmax(qq @ kk.transpose(1, 2) / 8.0, dim=-1)
        want = (p @ vv).reshape(NH, D)
        err = (got[b].float() - want).abs()
        assert (err <= 2e-3 + 2.0 ** -9 * want.abs()).all(), (b, float(err.max()))


def _planned_ex(lib, N, q, k, v, bt_np, ctx_np, mb, flags):
    dev = q.device
    B, NH, D = q.shape
    NB, KVH = k.shape[0], k.shape[1]
    bt, ctx = torch.from_numpy(bt_np).to(dev), torch.from_numpy(ctx_np).to(dev)
    s = torch.cuda.current_stream().cuda_stream
    need = lib.ti_paged_attention_workspace_bytes(B, NH, KVH, D, mb, 0)
    ws = torch.zeros(need, dtype=torch.uint8, device=dev)
    plan = torch.zeros(lib.ti_paged_attention_plan_bytes(B), dtype=torch.uint8, device=dev)
    N.check(lib.ti_paged_attention_plan_ex(bt.data_ptr(), bt.stride(0), None, ctx.data_ptr(), B,
                                           NH, KVH, D, mb, NB, plan.data_ptr(), plan.numel(),
                                           flags, 896, N.dtype_code(q.dtype), s))
    got = torch.full_like(q, 3.0)
    N.check(lib.ti_paged_attention_decode_planned(*_args(q, k, v, bt, ctx, mb, got),
                                                  N.dtype_code(q.dtype), ws.data_ptr(), need,
                                                  plan.data_ptr(), s))
    torch.cuda.synchronize()
    return got, plan[:32].view(torch.int32).cpu().numpy()


@pytest.mark.parametrize("case", [(31, 256, 128, 2048, True), (32, 200, 64, 1024, True),
                                  (33, 256, 8192, 32768, False)])
def test_plan_after_qkv_skews_late_ctas(cuda_device, case):
    """TI_ATTN_PLAN_AFTER_QKV: the CTAs that start behind the QKV GEMM's SMs take fewer KV blocks
    (header word 7 < 8 streams, word 6 = CTAs with all 8) when the batch's loop is short enough
    for the few microseconds they start late to matter, and none otherwise (long contexts: the
    unskewed plan, bit for bit).  Skewed output: the plain call's up to the float32 summation
    order (2e-3 + half a bf16 ulp), and an fp32 torch reference on three rows."""
    from tiny_infra_b200 import _native as N
    lib = N.lib()
    seed, B, lo, hi, skewed = case
    NH, KVH, D = 14, 2, 64
    rng = np.random.default_rng(seed)
    ctx_np = rng.integers(lo, hi + 1, B).astype(np.int32)
    nblk = (ctx_np + 15) // 16
    NB = int(nblk.sum()) + 16
    mb = (hi + 15) // 16
    perm = rng.permutation(NB).astype(np.int32)
    bt_np = np.full((B, mb), -1, np.int32)
    off = 0
    for b in range(B):
        bt_np[b, :nblk[b]] = perm[off:off + nblk[b]]
        off += int(nblk[b])
    g = torch.Generator(device=cuda_device).manual_seed(seed)
    q = torch.randn(B, NH, D, device=cuda_device, generator=g).bfloat16()
    k = torch.randn(NB, KVH, 16, D, device=cuda_device, generator=g).bfloat16()
    v = torch.randn(NB, KVH, 16, D, device=cuda_device, generator=g).bfloat16()
    ref, _, _ = _plain_and_planned(lib, N, q, k, v, bt_np, ctx_np, mb)
    got, hdr = _planned_ex(lib, N, q, k, v, bt_np, ctx_np, mb, N.TI_ATTN_PLAN_AFTER_QKV)
    assert N.device_status() == 0
    if skewed:
        assert hdr[7] < 8 and 0 < hdr[6] < hdr[2] // 8, hdr
        a, b2 = got.float(), ref.float()
        assert ((a - b2).abs() <= 2e-3 + 2.0 ** -9 * b2.abs()).all(), float((a - b2).abs().max())
    else:
        assert hdr[7] == 8 and hdr[6] == hdr[2] // 8, hdr
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
    for b in (0, B // 2, B - 1):
        n = int(ctx_np[b])
        ids = torch.from_numpy(bt_np[b, :nblk[b]].astype(np.int64)).to(cuda_device)
        kk = k[ids].float().permute(1, 0, 2, 3).reshape(KVH, -1, D)[:, :n]
        vv = v[ids].float().permute(1, 0, 2, 3).reshape(KVH, -1, D)[:, :n]
        qq = q[b].float().view(KVH, NH // KVH, D)
        p = torch.softmax(qq @ kk.transpose(1, 2) / 8.0, dim=-1)
        want = (p @ vv).reshape(NH, D)
        err = (got[b].float() - want).abs()
        assert (err <= 2e-3 + 2.0 ** -9 * want.abs()).all(), (b, float(err.max()))
