"""GPU parity of the per-op kernels against the CPU oracle (float32 restatements of the
reference kernels), on the same bf16/fp16-representable inputs.

Tolerances (written per test):
  * attention: |gpu - oracle| <= 2e-3 + half an ulp of the stored output dtype at |oracle|
    (2^-9 |ref| for bf16, 2^-11 |ref| for fp16): the kernel accumulates in fp32 (P split into
    bf16 hi + lo for P.V), and storing a value of magnitude >= 1 in bf16 alone can move it by
    up to 0.0039;
  * elementwise ops: one rounding of the output dtype, |err| <= 2^-8 |ref| + 1e-6 (bf16) or
    2^-11 |ref| + 1e-6 (fp16), plus the same for each rounded intermediate the op stores.
  * integer work (slot mapping, KV positions) is compared bit-exactly.
"""
import numpy as np
import pytest
import torch

from oracle import kernels as OK
from oracle.numerics import bf16_round

pytestmark = pytest.mark.gpu

DT = {"bf16": torch.bfloat16, "fp16": torch.float16}


def _to_dev(x, dtype, dev):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(dev).to(dtype)


def _f32(t):
    return t.float().cpu().numpy()


def _attn_case(seed, B, NH, KVH, D, NB, ctx_lo, ctx_hi, max_blocks=None):
    rng = np.random.default_rng(seed)
    bs = 16
    ctx = rng.integers(ctx_lo, ctx_hi + 1, B).astype(np.int32)
    mb = max_blocks or (ctx_hi + bs - 1) // bs
    need = sum((int(c) + bs - 1) // bs for c in ctx)
    assert need <= NB
    perm = rng.permutation(NB)
    bt = np.full((B, mb), -1, np.int32)
    off = 0
    for b in range(B):
        n = (int(ctx[b]) + bs - 1) // bs
        bt[b, :n] = perm[off:off + n]
        off += n
    q = rng.standard_normal((B, NH, D)).astype(np.float32)
    k = rng.standard_normal((NB, KVH, bs, D)).astype(np.float32)
    v = rng.standard_normal((NB, KVH, bs, D)).astype(np.float32)
    return q, k, v, bt, ctx


def _attn_ok(out, ref, dtype=torch.bfloat16):
    # 2e-3 plus one rounding of the output dtype: half an ulp is at most 2^-8 |x| in bf16 (8
    # significant bits; 2^-8 |x| for x just above a power of two) and 2^-11 |x| in fp16
    half_ulp = 2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11
    err = np.abs(out - ref)
    return bool((err <= 2e-3 + half_ulp * np.abs(ref)).all()), float(err.max())


def _run_attn(dev, dtype, q, k, v, bt, ctx, partition_blocks=0, init=0.0):
    from tiny_infra_b200 import custom_paged_attn
    qt, kt, vt = (_to_dev(x, dtype, dev) for x in (q, k, v))
    out = torch.full_like(qt, init)
    custom_paged_attn.launch_paged_attention(out, qt, kt, vt, torch.from_numpy(bt).to(dev),
                                             torch.from_numpy(ctx).to(dev), 16,
                                             partition_blocks=partition_blocks)
    torch.cuda.synchronize()
    # the oracle runs on the same rounded inputs
    rq, rk, rv = (_f32(x) for x in (qt, kt, vt))
    ref = np.full(q.shape, init, np.float32)
    OK.paged_attention(ref, rq, rk, rv, bt, ctx, 16)
    return _f32(out), ref


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_attention_config1(cuda_device, dtype):
    """Paged decode op at its benchmark configuration: B=8, ctx ~ U[1,512], 14/2 heads, D=64,
    512-block pool, each table a slice of a random permutation."""
    q, k, v, bt, ctx = _attn_case(0, 8, 14, 2, 64, 512, 1, 512)
    out, ref = _run_attn(cuda_device, DT[dtype], q, k, v, bt, ctx)
    ok, err = _attn_ok(out, ref, DT[dtype])
    assert ok, err


@pytest.mark.parametrize("pb", [1, 4, 16])
def test_attention_split_k_long(cuda_device, pb):
    """Split-K partitions merged by the last-arriving CTA: contexts up to 4096 tokens."""
    q, k, v, bt, ctx = _attn_case(1, 12, 14, 2, 64, 3200, 1, 4096)
    out, ref = _run_attn(cuda_device, torch.bfloat16, q, k, v, bt, ctx, partition_blocks=pb)
    ok, err = _attn_ok(out, ref)
    assert ok, err


def test_attention_small_batch_many_pieces(cuda_device):
    """Small decode batches cut each sequence into up to 65 pieces so that a few sequences still
    spread over every SM; the merge reads them in rounds of 16: 3 sequences of 8192 tokens (64
    pieces each), one with a -1 entry inside its third round of pieces."""
    q, k, v, bt, ctx = _attn_case(7, 3, 14, 2, 64, 1600, 8000, 8192)
    bt[1, 300] = -1
    out, ref = _run_attn(cuda_device, torch.bfloat16, q, k, v, bt, ctx)
    ok, err = _attn_ok(out, ref)
    assert ok, err


def test_attention_edge_cases(cuda_device):
    """ctx 0 leaves the row untouched; a -1 entry truncates the context (in the first and in a
    later partition); a leading -1 gives NaN; block ids past the pool are treated as -1."""
    q, k, v, bt, ctx = _attn_case(2, 6, 14, 2, 64, 600, 200, 1500)
    ctx[0] = 0
    bt[1, 3] = -1          # inside the first partition
    bt[2, 20] = -1         # inside the second partition
    bt[3, 0] = -1          # nothing readable -> NaN
    bt[4, 5] = 600 + 7     # past the pool -> treated as -1
    for pb in (4, 16):
        out, ref = _run_attn(cuda_device, torch.bfloat16, q, k, v, bt, ctx, pb, init=7.0)
        assert (out[0] == 7.0).all()
        assert np.isnan(out[3]).all() and np.isnan(ref[3]).all()
        rows = [0, 1, 2, 4, 5]
        ok, err = _attn_ok(out[rows], ref[rows])
        assert ok, err


def test_attention_head_dim_128(cuda_device):
    """The reference's own test shape (test/attention_test.py:26-31): 8 q heads, 2 kv heads,
    head_dim 128."""
    q, k, v, bt, ctx = _attn_case(3, 5, 8, 2, 128, 300, 1, 900)
    out, ref = _run_attn(cuda_device, torch.float16, q, k, v, bt, ctx)
    ok, err = _attn_ok(out, ref, torch.float16)
    assert ok, err


def test_attention_256_ragged(cuda_device):
    """North-star shape: 256 ragged sequences, ctx ~ U[128, 2048]."""
    q, k, v, bt, ctx = _attn_case(4, 256, 14, 2, 64, 256 * 128, 128, 2048)
    out, ref = _run_attn(cuda_device, torch.bfloat16, q, k, v, bt, ctx)
    ok, err = _attn_ok(out, ref)
    assert ok, err


@pytest.mark.parametrize("kernel", ["v5", "v4", "v2"])
def test_attention_each_kernel(cuda_device, monkeypatch, kernel):
    """The equivalent head_dim-64 decode kernels selected in turn (TI_PAGED_ATTN_KERNEL): v5
    (producer warp + warp pairs), v4 (a TMA ring per warp), v2 (persistent ring): a ragged
    batch, long split-K contexts (units cut into up to 16 pieces), four kv heads (two units per
    sequence) and the edge cases of test_attention_edge_cases."""
    monkeypatch.setenv("TI_PAGED_ATTN_KERNEL", kernel)
    cases = [(4, 256, 14, 2, 64, 256 * 128, 128, 2048), (1, 12, 14, 2, 64, 3200, 1, 4096),
             (5, 40, 16, 4, 64, 2000, 1, 700)]
    for c in cases:
        q, k, v, bt, ctx = _attn_case(*c)
        out, ref = _run_attn(cuda_device, torch.bfloat16, q, k, v, bt, ctx)
        ok, err = _attn_ok(out, ref)
        assert ok, (c, err)
    q, k, v, bt, ctx = _attn_case(2, 6, 14, 2, 64, 600, 200, 1500)
    ctx[0] = 0
    bt[1, 3] = -1
    bt[2, 20] = -1
    bt[3, 0] = -1
    bt[4, 5] = 600 + 7
    out, ref = _run_attn(cuda_device, torch.bfloat16, q, k, v, bt, ctx, init=7.0)
    assert (out[0] == 7.0).all()
    assert np.isnan(out[3]).all() and np.isnan(ref[3]).all()
    ok, err = _attn_ok(out[[0, 1, 2, 4, 5]], ref[[0, 1, 2, 4, 5]])
    assert ok, err


def _decode_direct(lib, out, q, k, v, bt, ctx, ws=None, ws_bytes=0):
    """ti_paged_attention_decode through the C ABI (partition 0: the library's choice)."""
    B, NH, D = q.shape
    NB, KVH = k.shape[0], k.shape[1]
    dt = 1 if q.dtype == torch.float16 else 0
    return lib.ti_paged_attention_decode(
        out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), NB,
        bt.data_ptr(), bt.stride(0), None, ctx.data_ptr(), B, NH, KVH, D, 16, bt.shape[1], dt, 0,
        ws, ws_bytes, torch.cuda.current_stream().cuda_stream)


def test_attention_unit_kernel(cuda_device, monkeypatch):
    """Calls whose sequences all fit 32 blocks (ctx <= 512) and whose units (a sequence's pair
    of kv heads) fit one wave of CTAs run one CTA per unit: a single launch, no workspace, no
    plan.  Against the oracle: 148 units of ctx U[1, 512] (the wave limit); four kv heads in
    groups of 4 (two units per sequence); a GQA group of 8; fp16; contexts longer than the
    table (clamped to its 512 tokens, as the other kernels); the edge cases (ctx 0 untouched,
    -1 entries truncate, a leading -1 gives NaN, ids past the pool count as -1).  The same
    batch forced through v5 (split-K pieces and the merge kernel) agrees within the tolerance."""
    from tiny_infra_b200 import _native as N
    lib = N.lib()
    cases = [((10, 148, 14, 2, 64, 148 * 32, 1, 512), torch.bfloat16),
             ((11, 20, 16, 4, 64, 800, 1, 512), torch.bfloat16),
             ((12, 16, 16, 2, 64, 600, 1, 500), torch.bfloat16),
             ((13, 8, 14, 2, 64, 512, 1, 512), torch.float16),
             ((14, 6, 14, 2, 64, 600, 520, 700), torch.bfloat16)]
    for c, dt in cases:
        q, k, v, bt, ctx = _attn_case(*c)
        bt = np.ascontiguousarray(bt[:, :32])     # the last case: contexts past the table
        qt, kt, vt = (_to_dev(x, dt, cuda_device) for x in (q, k, v))
        btd, ctxd = torch.from_numpy(bt).to(cuda_device), torch.from_numpy(ctx).to(cuda_device)
        out = torch.zeros_like(qt)
        n0 = lib.ti_launch_count()
        assert _decode_direct(lib, out, qt, kt, vt, btd, ctxd) == 0, lib.ti_last_error()
        assert lib.ti_launch_count() - n0 == 1          # one launch, no workspace given
        torch.cuda.synchronize()
        ref = np.zeros(q.shape, np.float32)
        OK.paged_attention(ref, *(_f32(x) for x in (qt, kt, vt)), bt, ctx, 16)
        got = _f32(out)
        ok, err = _attn_ok(got, ref, dt)
        i = np.unravel_index(np.nanargmax(np.abs(got - ref)), ref.shape)
        assert ok, (c, err, float(ref[i]), float(got[i]), int(ctx[i[0]]))
    # edge cases
    q, k, v, bt, ctx = _attn_case(15, 6, 14, 2, 64, 300, 100, 512)
    ctx[0] = 0
    bt[1, 3] = -1
    bt[2, 20] = -1
    bt[3, 0] = -1
    bt[4, 5] = 300 + 7
    out, ref = _run_attn(cuda_device, torch.bfloat16, q, k, v, bt, ctx, init=7.0)
    assert (out[0] == 7.0).all()
    assert np.isnan(out[3]).all() and np.isnan(ref[3]).all()
    ok, err = _attn_ok(out[[0, 1, 2, 4, 5]], ref[[0, 1, 2, 4, 5]])
    assert ok, err
    # the same batch through v5 (which splits the sequences and merges) agrees
    q, k, v, bt, ctx = _attn_case(16, 40, 14, 2, 64, 40 * 32, 1, 512)
    unit, _ = _run_attn(cuda_device, torch.bfloat16, q, k, v, bt, ctx)
    monkeypatch.setenv("TI_PAGED_ATTN_KERNEL", "v5")
    v5, ref = _run_attn(cuda_device, torch.bfloat16, q, k, v, bt, ctx)
    ok, err = _attn_ok(unit, v5)
    assert ok, err
    assert N.device_status() == 0


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_rope_inplace(cuda_device, dtype):
    """custom_rope.apply_inplace on a packed ragged batch: T=4096, positions in [0, 32768)."""
    from tiny_infra_b200 import custom_rope
    rng = np.random.default_rng(5)
    T = 4096
    q = rng.standard_normal((T, 14, 64)).astype(np.float32)
    k = rng.standard_normal((T, 2, 64)).astype(np.float32)
    pos = rng.integers(0, 32768, T).astype(np.int32)
    cos, sin = OK.rope_table(32768, 64, 1e6)
    qt, kt = _to_dev(q, DT[dtype], cuda_device), _to_dev(k, DT[dtype], cuda_device)
    rq, rk = _f32(qt), _f32(kt)
    custom_rope.apply_inplace(qt, kt, torch.from_numpy(cos).to(cuda_device),
                              torch.from_numpy(sin).to(cuda_device),
                              torch.from_numpy(pos).to(cuda_device))
    OK.rope_inplace(rq, rk, cos, sin, pos)
    tol = 2.0 ** -8 if dtype == "bf16" else 2.0 ** -11
    for got, ref in ((qt, rq), (kt, rk)):
        err = np.abs(_f32(got) - ref)
        assert (err <= tol * np.abs(ref) + 1e-6).all()


def test_rope_kv_append(cuda_device):
    """RoPE fused with the KV-append write through slot_mapping: q/k rotated, k/v written to
    exactly the pool slots the mapping names (bit-exact positions), padded tokens skipped."""
    from tiny_infra_b200 import _native as N
    rng = np.random.default_rng(6)
    T, NH, KVH, D, bs, NB = 4096, 14, 2, 64, 16, 4096
    qkv = rng.standard_normal((T, (NH + 2 * KVH) * D)).astype(np.float32)
    pos = rng.integers(0, 32768, T).astype(np.int32)
    slots = rng.permutation(NB * bs)[:T].astype(np.int64)
    slots[7] = -1                                       # a padded token: no KV write
    cos, sin = OK.rope_table(32768, D, 1e6)
    dev = cuda_device
    t_qkv = _to_dev(qkv, torch.bfloat16, dev)
    kc = torch.zeros(NB, KVH, bs, D, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    ref_qkv = _f32(t_qkv)
    # keep every device tensor referenced until the kernel has run
    d_slots, d_cos = torch.from_numpy(slots).to(dev), torch.from_numpy(cos).to(dev)
    d_sin, d_pos = torch.from_numpy(sin).to(dev), torch.from_numpy(pos).to(dev)
    N.check(N.lib().ti_rope_kv_append(
        t_qkv.data_ptr(), t_qkv.stride(0), kc.data_ptr(), vc.data_ptr(), d_slots.data_ptr(),
        d_cos.data_ptr(), d_sin.data_ptr(), d_pos.data_ptr(), T, NH, KVH, D, bs,
        N.TI_DTYPE_BF16, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    rq = ref_qkv[:, :NH * D].reshape(T, NH, D).copy()
    rk = ref_qkv[:, NH * D:(NH + KVH) * D].reshape(T, KVH, D).copy()
    rv = ref_qkv[:, (NH + KVH) * D:].reshape(T, KVH, D)
    OK.rope_inplace(rq, rk, cos, sin, pos)
    got = _f32(t_qkv)
    tol = 2.0 ** -8
    for a, b in ((got[:, :NH * D], rq.reshape(T, -1)), (got[:, NH * D:(NH + KVH) * D], rk.reshape(T, -1))):
        assert (np.abs(a - b) <= tol * np.abs(b) + 1e-6).all()
    kcf, vcf = _f32(kc), _f32(vc)
    live = slots >= 0
    blk, off = slots[live] // bs, slots[live] % bs
    np.testing.assert_array_equal(kcf[blk, :, off, :], bf16_round(got[live, NH * D:(NH + KVH) * D].reshape(-1, KVH, D)))
    np.testing.assert_array_equal(vcf[blk, :, off, :], rv[live])
    written = np.zeros((NB, bs), bool)
    written[blk, off] = True
    kt, vt = kcf.transpose(0, 2, 1, 3), vcf.transpose(0, 2, 1, 3)   # [NB, bs, KVH, D]
    assert (kt[~written] == 0).all() and (vt[~written] == 0).all()


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_swiglu(cuda_device, dtype):
    """custom_swiglu.forward at T=4096, I=4864 (gate/up [T, 2*4864])."""
    from tiny_infra_b200 import custom_swiglu
    rng = np.random.default_rng(7)
    x = rng.standard_normal((4096, 2 * 4864)).astype(np.float32)
    xt = _to_dev(x, DT[dtype], cuda_device)
    out = custom_swiglu.forward(xt)
    ref = OK.swiglu(_f32(xt))
    tol = 2.0 ** -8 if dtype == "bf16" else 2.0 ** -11
    assert out.shape == (4096, 4864)
    assert (np.abs(_f32(out) - ref) <= tol * np.abs(ref) + 1e-6).all()
    with pytest.raises(RuntimeError):
        custom_swiglu.forward(xt[:, :12].contiguous())   # I = 6 is not a multiple of 8


@pytest.mark.parametrize("T", [4096, 4095, 37])
def test_rmsnorm(cuda_device, T):
    """RMSNorm over hidden 896 (eps 1e-6) on the float32 residual stream, bf16 output: large
    batches run two rows per warp (4095: the last pass has one row), small ones one."""
    from tiny_infra_b200 import _native as N
    rng = np.random.default_rng(8)
    H = 896
    x = (rng.standard_normal((T, H)) * 3).astype(np.float32)
    w = bf16_round(rng.standard_normal(H).astype(np.float32))
    xt = torch.from_numpy(x).to(cuda_device)
    wt = _to_dev(w, torch.bfloat16, cuda_device)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=cuda_device)
    N.check(N.lib().ti_rmsnorm(out.data_ptr(), xt.data_ptr(), N.TI_DTYPE_FP32, wt.data_ptr(),
                               1e-6, T, H, N.TI_DTYPE_BF16, torch.cuda.current_stream().cuda_stream))
    ref = OK.rmsnorm(x, w, 1e-6)
    # two bf16 roundings (normalised row, then the weight product), as in the reference
    tol = 2 * 2.0 ** -8
    assert (np.abs(_f32(out) - ref) <= tol * np.abs(ref) + 1e-5).all()


@pytest.mark.parametrize("T", [300, 40, 2048, 32, 17])
def test_qkv_rope_append_gemm(cuda_device, T):
    """QKV projection with RoPE and the KV append fused in the tcgen05 GEMM epilogue: q and the
    pool's k/v equal the float32 x W^T + b, rotated, rounded once to bf16 (one ulp allowed for
    accumulation order).  300, 40, 32 and 17 tokens run split-K over a cluster of 4 (17: the last
    rows of the 128-row tile past M), 2048 unsplit."""
    from tiny_infra_b200 import _native as N
    rng = np.random.default_rng(9)
    H, NH, KVH, D, bs = 896, 14, 2, 64, 16
    NB = (T + bs - 1) // bs + 48
    QKV = (NH + 2 * KVH) * D
    x = bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    w = bf16_round((rng.standard_normal((QKV, H)) * 0.03).astype(np.float32))
    b = bf16_round((rng.standard_normal(QKV) * 0.1).astype(np.float32))
    pos = rng.integers(0, 4096, T).astype(np.int32)
    slots = rng.permutation(NB * bs)[:T].astype(np.int64)
    slots[5] = -1
    cos, sin = OK.rope_table(4096, D, 1e6)
    dev = cuda_device
    tx, tw, tb = (_to_dev(a, torch.bfloat16, dev) for a in (x, w, b))
    d_slots, d_cos = torch.from_numpy(slots).to(dev), torch.from_numpy(cos).to(dev)
    d_sin, d_pos = torch.from_numpy(sin).to(dev), torch.from_numpy(pos).to(dev)
    q = torch.zeros(T, QKV, dtype=torch.bfloat16, device=dev)
    kc = torch.zeros(NB, KVH, bs, D, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    N.check(N.lib().ti_gemm_qkv_rope(
        tx.data_ptr(), H, tw.data_ptr(), H, tb.data_ptr(), T, H, NH, KVH, D, q.data_ptr(), QKV,
        kc.data_ptr(), vc.data_ptr(), d_slots.data_ptr(), d_cos.data_ptr(), d_sin.data_ptr(),
        d_pos.data_ptr(), bs, N.TI_DTYPE_BF16, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    y = x @ w.T + b
    rq = y[:, :NH * D].reshape(T, NH, D).copy()
    rk = y[:, NH * D:(NH + KVH) * D].reshape(T, KVH, D).copy()
    rv = y[:, (NH + KVH) * D:].reshape(T, KVH, D)
    OK.rope_inplace(rq, rk, cos, sin, pos)

    def close(got, ref):
        return (np.abs(got - ref) <= 2.0 ** -8 * np.abs(ref) + 1e-4).all()

    assert close(_f32(q)[:, :NH * D], rq.reshape(T, -1))
    live = slots >= 0
    blk, off = slots[live] // bs, slots[live] % bs
    assert close(_f32(kc)[blk, :, off, :], rk[live])
    assert close(_f32(vc)[blk, :, off, :], rv[live])
    written = np.zeros((NB, bs), bool)
    written[blk, off] = True
    assert (_f32(kc).transpose(0, 2, 1, 3)[~written] == 0).all()


def test_step_kernels_bound_their_indices(cuda_device):
    """ti_decode_prepare and ti_kv_scatter check slots, positions and block ids against the
    block table and the pool they are given: a row whose position lies past its table row, or
    whose slot is outside the table, becomes padding; a new block or a pool slot outside the pool
    is not written; each raises TI_DEVERR_BAD_INPUT and leaves the valid rows' results intact."""
    from tiny_infra_b200 import _native as N
    lib, dev = N.lib(), cuda_device
    s = torch.cuda.current_stream().cuda_stream
    slots_n, mb, nb, bs, H, V = 4, 3, 10, 16, 64, 32
    bt = torch.full((slots_n, mb), -1, dtype=torch.int32, device=dev)
    bt[0, 0] = 2
    seq = torch.tensor([5, 0, mb * bs, 0], dtype=torch.int32, device=dev)   # slot 2: past its row
    tokens = torch.tensor([1, 2, 3, 4], dtype=torch.int32, device=dev)
    rows_slots = torch.tensor([0, 1, 2, 9], dtype=torch.int32, device=dev)  # 9: outside the table
    new_block = torch.tensor([-1, nb + 5, 4, 6], dtype=torch.int32, device=dev)  # row 1: outside
    pos = torch.full((4,), -7, dtype=torch.int32, device=dev)
    smap = torch.full((4,), -7, dtype=torch.int64, device=dev)
    ctx = torch.full((4,), -7, dtype=torch.int32, device=dev)
    hid = torch.full((4, H), 3.0, dtype=torch.float32, device=dev)
    emb = torch.randn(V, H, device=dev).to(torch.bfloat16)
    N.device_status()
    N.check(lib.ti_decode_prepare(tokens.data_ptr(), rows_slots.data_ptr(), new_block.data_ptr(),
                                  seq.data_ptr(), bt.data_ptr(), bt.stride(0), slots_n, mb, nb, bs,
                                  pos.data_ptr(), smap.data_ptr(), ctx.data_ptr(), hid.data_ptr(),
                                  emb.data_ptr(), H, V, 4, N.TI_DTYPE_BF16, s))
    torch.cuda.synchronize()
    assert N.device_status() & N.TI_DEVERR_BAD_INPUT
    assert smap.tolist() == [2 * bs + 5, -1, -1, -1]
    assert ctx.tolist() == [6, 1, 0, 0] and pos.tolist()[:2] == [5, 0]
    assert bt[1].tolist() == [-1, -1, -1] and bt[2].tolist() == [-1, -1, -1]
    assert torch.equal(hid[0], emb[1].float()) and (hid[2:] == 0).all()
    kc = torch.zeros(nb, 2, bs, 64, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    k = torch.randn(3, 2, 64, device=dev).to(torch.bfloat16)
    v = torch.randn(3, 2, 64, device=dev).to(torch.bfloat16)
    sm = torch.tensor([3, nb * bs, -1], dtype=torch.int64, device=dev)     # second: outside
    N.check(lib.ti_kv_scatter(kc.data_ptr(), vc.data_ptr(), k.data_ptr(), k.stride(0), k.stride(1),
                              v.data_ptr(), v.stride(0), v.stride(1), sm.data_ptr(), 3, nb, 2, 64,
                              bs, N.TI_DTYPE_BF16, s))
    torch.cuda.synchronize()
    assert N.device_status() & N.TI_DEVERR_BAD_INPUT
    assert torch.equal(kc[0, :, 3], k[0]) and torch.equal(vc[0, :, 3], v[0])
    assert int((kc != 0).sum()) == int((k[0] != 0).sum())
    assert N.device_status() == 0
