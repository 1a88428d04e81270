"""Ragged causal prefill attention over the paged pool (ti_paged_prefill_attention) against the
oracle (oracle.kernels.paged_prefill_attention, fp32), for both kernels: the tcgen05 one
(TMEM accumulators, P split into bf16 hi + lo; each tile's keys split over a cluster of two CTAs
whose partials merge through distributed shared memory, or one CTA per tile with
TI_PREFILL_ATTN_SPLIT=0) and the mma.sync one (TI_PREFILL_ATTN_KERNEL=mma).

Cases: whole prompts from position 0, chunks starting at odd positions (chunked prefill),
partial 16-token query tiles, a long prefix (several hundred 64-key steps), and a pool whose
key norms grow along the sequence so that the rows' running maxima keep rising (the tcgen05
kernel then rescales O in TMEM).  Tolerance: |err| <= 2e-3 + 2^-8 |oracle|: half an ulp of a bf16
value is up to 2^-8 of it, and a query that attends to a handful of keys has outputs near 1-2
(the decode tests average over hundreds of keys, so their outputs stay small).
"""
import numpy as np
import pytest
import torch

from oracle import kernels as OK

pytestmark = pytest.mark.gpu


def _run(dev, lens, starts, seed, grow=0.0, NH=14, KVH=2, D=64):
    from tiny_infra_b200 import _native as N
    rng = np.random.default_rng(seed)
    bs = 16
    S = len(lens)
    nblk = [(s + n + bs - 1) // bs for s, n in zip(starts, lens)]
    NB = sum(nblk) + 8
    mb = max(nblk)
    perm = rng.permutation(NB)
    bt = np.full((S, mb), -1, np.int32)
    off = 0
    for i in range(S):
        bt[i, :nblk[i]] = perm[off:off + nblk[i]]
        off += nblk[i]
    T = int(sum(lens))
    q = rng.standard_normal((T, NH, D)).astype(np.float32)
    k = rng.standard_normal((NB, KVH, bs, D)).astype(np.float32)
    v = rng.standard_normal((NB, KVH, bs, D)).astype(np.float32)
    if grow:
        for i in range(S):          # key norm grows with the position: rising row maxima
            for lb in range(nblk[i]):
                pos = lb * bs + np.arange(bs)
                k[bt[i, lb]] *= (1.0 + grow * pos)[None, :, None]
    to = lambda x: torch.from_numpy(x).to(dev).to(torch.bfloat16)  # noqa: E731
    qt, kt, vt = to(q), to(k), to(v)
    out = torch.full_like(qt, 9.0)
    cu = np.zeros(S + 1, np.int32)
    cu[1:] = np.cumsum(lens)
    ts, tq = [], []
    for i in range(S):
        for q0 in range(0, lens[i], 16):
            ts.append(i)
            tq.append(q0)
    ai = lambda x: torch.from_numpy(np.asarray(x, np.int32)).to(dev)  # noqa: E731
    d_bt, d_rows, d_st, d_cu, d_ts, d_tq = (ai(bt), ai(np.arange(S)), ai(starts), ai(cu), ai(ts),
                                            ai(tq))
    N.check(N.lib().ti_paged_prefill_attention(
        out.data_ptr(), NH * D, qt.data_ptr(), NH * D, kt.data_ptr(), vt.data_ptr(), NB,
        d_bt.data_ptr(), d_bt.stride(0), d_rows.data_ptr(), d_st.data_ptr(), d_cu.data_ptr(),
        d_ts.data_ptr(), d_tq.data_ptr(), len(ts), NH, KVH, D, bs, N.TI_DTYPE_BF16,
        torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    rq, rk, rv = (x.float().cpu().numpy() for x in (qt, kt, vt))
    for i in range(S):
        ref = OK.paged_prefill_attention(rq[cu[i]:cu[i + 1]], rk, rv, bt[i], starts[i], bs)
        err = np.abs(got[cu[i]:cu[i + 1]] - ref)
        assert (err <= 2e-3 + 2.0 ** -8 * np.abs(ref)).all(), (i, float(err.max()))
    assert N.device_status() == 0


def _select(monkeypatch, kernel):
    """tc: the tcgen05 kernel with every tile split over a cluster of two CTAs (the default);
    tc1: the same kernel, one CTA per tile (TI_PREFILL_ATTN_SPLIT=0); mma: the mma.sync kernel."""
    if kernel == "mma":
        monkeypatch.setenv("TI_PREFILL_ATTN_KERNEL", "mma")
    if kernel == "tc1":
        monkeypatch.setenv("TI_PREFILL_ATTN_SPLIT", "0")


@pytest.mark.parametrize("kernel", ["tc", "tc1", "mma"])
def test_prefill_attention_ragged_chunks(cuda_device, monkeypatch, kernel):
    _select(monkeypatch, kernel)
    _run(cuda_device, [37, 16, 5, 130, 64, 1], [0, 100, 2047, 0, 513, 77], seed=1)


@pytest.mark.parametrize("kernel", ["tc", "tc1", "mma"])
def test_prefill_attention_long_prefix_and_rising_max(cuda_device, monkeypatch, kernel):
    _select(monkeypatch, kernel)
    _run(cuda_device, [48, 200], [20000, 0], seed=2)
    _run(cuda_device, [33, 160], [3000, 0], seed=3, grow=0.004)


def test_prefill_attention_group_of_eight(cuda_device):
    """Eight query heads per kv head fill all 128 MMA rows of the tcgen05 kernel."""
    _run(cuda_device, [40, 17], [0, 300], seed=4, NH=16, KVH=2)
