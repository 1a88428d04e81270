"""GPU parity of the device sampler (ti_sample) with the oracle's restatement of
``ContinuousBatcher._sample_next_token`` (engine/scheduler.py:104-156).

Candidates (temperature, then the top-k rule with its batch-level behaviour) come from the
oracle.  The top-p boundary -- the first token of the descending order whose cumulative
probability exceeds p -- is a float-rounding-sensitive decision (the oracle accumulates in
float32, the reference in the logits dtype, the kernel in 32.32 fixed point), so the check
recomputes it in float64 and accepts a kernel boundary up to 3 positions away; the drawn token
must then lie in the kept prefix and its CDF interval (normalized by that prefix's mass) must
contain u to 1e-6.  Greedy rows (temperature 0) must match exactly.
"""
import numpy as np
import pytest
import torch

from oracle import sampler as OS
from oracle.numerics import bf16_round

pytestmark = pytest.mark.gpu


class _Req:
    def __init__(self, t, k, p):
        self.temperature, self.top_k, self.p_value = t, k, p


def _check_row(cand_row, p, tok, u, slack=3, tol=1e-6):
    """cand_row: the row after temperature and top-k (-inf = removed), float32."""
    keep = np.nonzero(np.isfinite(cand_row))[0]
    order = keep[np.lexsort((keep, -cand_row[keep]))]
    w = np.exp(cand_row[order].astype(np.float64) - float(cand_row[order[0]]))
    c = np.cumsum(w)
    c /= c[-1]
    L = len(order) - 1
    if p < 1.0:
        over = np.nonzero(c > p)[0]
        L = int(over[0]) if len(over) else L
    hits = np.nonzero(order == tok)[0]
    assert len(hits) == 1, tok
    pos = int(hits[0])
    assert pos <= L + slack, (tok, pos, L)
    lo = c[pos - 1] if pos > 0 else 0.0
    hi = c[pos]
    for L2 in range(max(pos, L - slack), min(len(order), L + slack + 1)):
        z = c[L2]
        if lo / z - tol <= u <= hi / z + tol:
            return
    raise AssertionError((tok, pos, L, lo, hi, u))


def _run(logits_bf16, temps, ks, ps, us):
    from tiny_infra_b200 import sampler as S
    reqs = [_Req(t, k, p) for t, k, p in zip(temps, ks, ps)]
    return S.sample_next_token(logits_bf16, reqs, uniforms=us)


@pytest.mark.parametrize("V", [5000, 151936])
def test_mixed_parameters_match_oracle(cuda_device, V):
    rng = np.random.default_rng(V)
    B = 8
    logits = bf16_round((rng.standard_normal((B, V)) * 3.0).astype(np.float32))
    temps = [0.7, 1.0, 0.0, 1.3, 0.7, 0.5, 0.9, 0.7]
    ks = [50, 50, 50, 20, 0, 50, 50, 50]          # rows with 20 / 0 keep everything (quirk)
    ps = [0.9, 0.9, 0.9, 0.9, 0.5, 1.0, 0.95, 0.3]
    us = rng.random(B).astype(np.float32).tolist()
    dev = torch.from_numpy(logits).to(cuda_device, torch.bfloat16)
    toks = _run(dev, temps, ks, ps, us)
    cand = OS.filter_logits(logits, temps, ks, [1.0] * B)     # temperature + top-k only
    p_active = any(p < 1.0 for p in ps)
    for b in range(B):
        if temps[b] == 0.0:
            assert toks[b] == int(np.argmax(logits[b])), b
        else:
            _check_row(cand[b], ps[b] if p_active else 1.0, toks[b], us[b])


def test_distribution_matches_oracle(cuda_device):
    """4096 draws of one row (u on a uniform grid): the empirical distribution equals the
    oracle's filtered softmax (top-k 50, top-p 0.9, temperature 0.7)."""
    rng = np.random.default_rng(3)
    V, B = 2048, 4096
    row = bf16_round((rng.standard_normal(V) * 2.0).astype(np.float32))
    logits = np.tile(row, (B, 1))
    us = ((np.arange(B) + 0.5) / B).astype(np.float32)
    dev = torch.from_numpy(logits).to(cuda_device, torch.bfloat16)
    toks = np.array(_run(dev, [0.7] * B, [50] * B, [0.9] * B, us.tolist()))
    probs = OS.sample_probs(row[None, :], [0.7], [50], [0.9])[0]
    emp = np.bincount(toks, minlength=V) / B
    assert set(np.nonzero(emp)[0]) <= set(np.nonzero(probs > 0)[0])
    assert 0.5 * np.abs(emp - probs).sum() < 0.02


def test_edge_cases(cuda_device):
    rng = np.random.default_rng(5)
    V = 4096
    logits = bf16_round(rng.standard_normal((4, V)).astype(np.float32))
    logits[0, 100] = logits[0, 200] = 9.0          # tied maximum: greedy takes the lower index
    logits[1, :] = -np.inf
    logits[1, 7] = 0.0                              # one finite entry
    dev = torch.from_numpy(logits).to(cuda_device, torch.bfloat16)
    # greedy tie, single finite entry, top-p keeping only the first token, full distribution
    temps, ks, ps = [0.0, 0.8, 1.0, 0.6], [0, 0, 0, 0], [1.0, 1.0, 1e-4, 0.999]
    us = [0.5, 0.999, 0.999, 0.999999]
    toks = _run(dev, temps, ks, ps, us)
    assert toks[0] == 100
    assert toks[1] == 7
    assert toks[2] == int(np.argmax(logits[2]))
    _check_row(OS.filter_logits(logits, temps, ks, [1.0] * 4)[3], ps[3], toks[3], us[3])
    # top_k = 1 in every row: the cutoff applies to all rows, each keeps only its maximum
    toks = _run(dev, [1.0] * 4, [1] * 4, [1.0] * 4, [0.3, 0.6, 0.9, 0.0])
    assert toks[2:] == [int(np.argmax(logits[2])), int(np.argmax(logits[3]))]
    # u = 0 draws the largest kept value
    toks = _run(dev, [1.0] * 4, [0] * 4, [1.0] * 4, [0.0] * 4)
    assert toks[2:] == [int(np.argmax(logits[2])), int(np.argmax(logits[3]))]


def test_topk_fast_path_and_overflow(cuda_device):
    """Rows with a top-k cut of at most 512 take the compacted-candidate route; a row whose
    top-k keeps more than 4096 tied elements falls back to the radix selects.  Both must give
    the reference's answer: with 6000 equal maxima and k = 10 every tie is kept (x >= the 10th
    largest), each with weight exp(0), so u = 0.5 draws the 3001st tied index; k = 512 and
    k = 1 on a random row follow the oracle's kept set and CDF."""
    rng = np.random.default_rng(8)
    V = 8192
    logits = bf16_round(rng.standard_normal((3, V)).astype(np.float32))
    ties = np.sort(rng.choice(V, 6000, replace=False))
    logits[0, :] = -3.0
    logits[0, ties] = 1.0
    dev = torch.from_numpy(logits).to(cuda_device, torch.bfloat16)
    temps, ks, ps, us = [1.0, 0.9, 1.2], [10, 512, 1], [1.0, 0.95, 1.0], [0.5, 0.37, 0.8]
    # the batch rule keeps top-k only in rows whose k is the batch's largest: run rows alone
    toks = [_run(dev[i:i + 1], [temps[i]], [ks[i]], [ps[i]], [us[i]])[0] for i in range(3)]
    assert toks[0] == int(ties[3000])
    for i in (1, 2):
        cand = OS.filter_logits(logits[i:i + 1], [temps[i]], [ks[i]], [1.0])[0]
        _check_row(cand, ps[i], toks[i], us[i])


def test_seq_len_advance(cuda_device):
    from tiny_infra_b200 import sampler as S
    V = 1000
    logits = torch.randn(3, V, device=cuda_device).to(torch.bfloat16)
    sp = S.SamplingParams([0.0, 0.0, 0.0], [0, 0, 0], [1.0, 1.0, 1.0], [0.1, 0.2, 0.3], V)
    pd = torch.from_numpy(sp.packed()).to(cuda_device)
    out = torch.empty(3, dtype=torch.int32, device=cuda_device)
    slots = torch.tensor([2, -1, 0], dtype=torch.int32, device=cuda_device)
    seq = torch.tensor([5, 6, 7], dtype=torch.int32, device=cuda_device)
    S.launch_sample(logits, pd, out, slots, seq, 1)
    torch.cuda.synchronize()
    assert seq.tolist() == [6, 6, 8]
    assert out.tolist() == torch.argmax(logits.float(), dim=-1).tolist()
