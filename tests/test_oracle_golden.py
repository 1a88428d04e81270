"""Pin the oracle against golden vectors produced by the reference's own code
(tests/golden/make_golden.py, and make_kernel_golden.py for the CUDA kernels)."""
import hashlib
import json
import os

import numpy as np
import pytest

from oracle import kernels as OK
from oracle import sampler as OS
from oracle.cache import OracleKVCache
from oracle.model import OracleConfig, forward, init_weights


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def test_cache_ops_bit_exact(golden_dir):
    """Allocator, tables, lengths, free list and pool bytes equal the reference's after every
    call of a scripted sequence, including its ValueError / RuntimeError(OOM) / IndexError."""
    meta = json.load(open(os.path.join(golden_dir, "cache_ops.json")))
    arr = _load(golden_dir, "cache_ops.npz")
    c = meta["config"]
    mgr = OracleKVCache(c["max_batch_size"], c["max_seq_len"], c["num_layers"],
                        c["num_kv_heads"], c["head_dim"], c["block_size"])
    for i, rec in enumerate(meta["records"]):
        op, err = rec["op"], None
        if op[0] == "insert":
            try:
                for layer in range(c["num_layers"]):
                    mgr.allocate_and_insert(layer, np.array(op[1], np.int64), arr[f"k{i}"],
                                            arr[f"v{i}"])
            except (ValueError, RuntimeError) as e:
                err = type(e).__name__
        elif op[0] == "advance":
            mgr.seq_len[np.array(op[1])] += op[2]
        elif op[0] == "truncate_free":
            del mgr.free_blocks[op[1]:]
        elif op[0] == "free":
            try:
                mgr.free_batch_slot(op[1])
            except IndexError as e:
                err = type(e).__name__
        assert err == rec["error"], (i, op)
        assert mgr.block_tables.tolist() == rec["block_tables"], (i, op)
        assert mgr.seq_len.tolist() == rec["seq_len"], (i, op)
        assert mgr.free_blocks == rec["free_blocks"], (i, op)
        assert hashlib.sha256(mgr.key_cache.tobytes()).hexdigest() == rec["key_sha256"], (i, op)
        assert hashlib.sha256(mgr.value_cache.tobytes()).hexdigest() == rec["val_sha256"], (i, op)
    np.testing.assert_array_equal(mgr.key_cache, arr["key_final"])
    np.testing.assert_array_equal(mgr.value_cache, arr["val_final"])


def test_rope_table(golden_dir):
    """cos/sin tables of engine/scheduler.py:36-48 at 32768 positions (within 2 float32 ulp
    of the argument: numpy's and torch's pow/cos/sin may differ in the last bit)."""
    g = _load(golden_dir, "rope_table.npz")
    cos, sin = OK.rope_table(32768, 64, 1e6)
    rows = g["rows"]
    # |freq| reaches 32767 rad; one fp32 ulp of the argument there is ~0.004 rad.
    np.testing.assert_allclose(cos[rows], g["cos"], atol=8e-3, rtol=0)
    np.testing.assert_allclose(sin[rows], g["sin"], atol=8e-3, rtol=0)
    np.testing.assert_allclose(cos[:256], g["cos"][:256], atol=2e-5, rtol=0)
    np.testing.assert_allclose(sin[:256], g["sin"][:256], atol=2e-5, rtol=0)


@pytest.mark.parametrize("case", ["uniform_k", "mixed_k", "no_topp", "full_vocab", "ties"])
def test_sampler_distribution(golden_dir, case):
    """The distribution handed to torch.multinomial, and the greedy rows' tokens."""
    g = _load(golden_dir, "sampler.npz")
    logits, temps = g[f"{case}_logits"], g[f"{case}_temps"]
    ks, ps = g[f"{case}_topk"], g[f"{case}_topp"]
    probs = OS.sample_probs(logits, temps, ks, ps)
    ref = g[f"{case}_probs"]
    # Support must agree except possibly one boundary token per row (float summation order
    # of the top-p cumsum); probabilities agree to float32 rounding.  Where logits tie exactly
    # at the top-p boundary, the reference keeps whichever tied tokens torch.sort (unstable)
    # puts first; the restatement keeps the lowest indices, so there the kept sets may differ
    # among tokens of the boundary value only -- counts and probability values still agree.
    for b in range(probs.shape[0]):
        mine, theirs = probs[b] > 0, ref[b] > 0
        diff = np.count_nonzero(mine != theirs)
        if diff == 0:
            np.testing.assert_allclose(probs[b], ref[b], atol=2e-6, rtol=1e-4)
            continue
        boundary = logits[b][theirs].min()
        differing = np.nonzero(mine != theirs)[0]
        if np.all(logits[b][differing] == boundary):
            assert mine.sum() == theirs.sum()
            np.testing.assert_allclose(np.sort(probs[b][mine]), np.sort(ref[b][theirs]),
                                       atol=2e-6, rtol=1e-4)
        else:
            assert diff <= 1, (case, b, diff)
    tok = g[f"{case}_tokens"]
    greedy = OS.greedy(logits, temps, ks, ps)
    for b in range(len(temps)):
        if temps[b] == 0.0:
            assert greedy[b] == tok[b]
        else:
            assert ref[b, tok[b]] > 0   # the reference's sample lies in the support


def test_model_forward(golden_dir):
    """Qwen2ForCausalLM.forward (small config, fp32): two prefills and two decode steps."""
    from tests.golden.make_golden import SMALL
    g = _load(golden_dir, "model_forward.npz")
    cfg = OracleConfig(**SMALL)
    W = init_weights(cfg, seed=3, tied=False, bf16=False)
    cache = OracleKVCache(3, 64, cfg.num_layers, cfg.num_key_value_heads, cfg.head_dim, 16)
    cos, sin = OK.rope_table(64, cfg.head_dim, cfg.rope_theta)
    for i in range(int(g["num_calls"])):
        ids, idx = g[f"ids{i}"], g[f"idx{i}"]
        logits = forward(W, cfg, ids, idx, cache, cos, sin)
        cache.seq_len[idx] += ids.shape[1]
        np.testing.assert_allclose(logits, g[f"logits{i}"], atol=2e-5, rtol=1e-4)
    np.testing.assert_array_equal(cache.block_tables, g["block_tables"])
    np.testing.assert_array_equal(cache.seq_len, g["seq_len"])


def test_paged_attention_edge_cases():
    """ctx==0 leaves out untouched (attention.cu:62); a leading -1 entry gives NaN
    (attention.cu:90,150); a -1 after valid blocks truncates the context."""
    rng = np.random.default_rng(0)
    q = rng.standard_normal((3, 4, 8)).astype(np.float32)
    kc = rng.standard_normal((6, 2, 4, 8)).astype(np.float32)
    vc = rng.standard_normal((6, 2, 4, 8)).astype(np.float32)
    bt = np.array([[0, 1, 2], [-1, 3, 4], [5, -1, 1]], np.int32)
    out = np.full((3, 4, 8), 7.0, np.float32)
    OK.paged_attention(out, q, kc, vc, bt, np.array([0, 5, 12], np.int32), 4)
    assert (out[0] == 7.0).all()
    assert np.isnan(out[1]).all()
    ref = np.zeros((1, 4, 8), np.float32)
    OK.paged_attention(ref, q[2:3], kc, vc, bt[2:3], np.array([4], np.int32), 4)
    np.testing.assert_allclose(out[2], ref[0], rtol=1e-6)


def test_chunked_prefill_matches_whole_prefill():
    """Paged causal attention over earlier chunks equals the reference's whole-prompt SDPA."""
    rng = np.random.default_rng(1)
    S, NH, KVH, D, bs = 37, 4, 2, 8, 16
    q = rng.standard_normal((1, S, NH, D)).astype(np.float32)
    k = rng.standard_normal((1, S, KVH, D)).astype(np.float32)
    v = rng.standard_normal((1, S, KVH, D)).astype(np.float32)
    whole = OK.causal_self_attention(q, k, v)[0]
    kc = np.zeros((5, KVH, bs, D), np.float32)
    vc = np.zeros_like(kc)
    table = np.array([3, 0, 4, -1], np.int32)
    for t in range(S):
        kc[table[t // bs], :, t % bs] = k[0, t]
        vc[table[t // bs], :, t % bs] = v[0, t]
    parts = [OK.paged_prefill_attention(q[0, a:b], kc, vc, table, a, bs)
             for a, b in ((0, 10), (10, 31), (31, 37))]
    np.testing.assert_allclose(np.concatenate(parts), whole, atol=1e-5, rtol=1e-5)


def test_reference_kernels(golden_dir):
    """The oracle restatements of src/attention.cu, src/fused_rope.cu and src/fused_swiglu.cu
    against the reference kernels themselves, compiled from the reference sources
    (oracle/build_ref.py) and run on a B200 by tests/golden/make_kernel_golden.py.  The
    reference kernels compute in fp32 and store fp16: tolerance is fp16 rounding of the output
    (2^-11 relative) plus 1e-3 absolute for fp32 summation order (the reference sums q.k with
    a block tree reduction and uses __expf)."""
    path = os.path.join(golden_dir, "kernel_golden.npz")
    if not os.path.exists(path):
        pytest.skip("kernel_golden.npz not generated")
    from tests.golden.make_kernel_golden import inputs
    g = np.load(path)
    x = inputs()
    for name in ("attn64", "attn128"):
        q, k, v, bt, ctx = x[name]
        ref = g[f"{name}_out"].astype(np.float32)
        out = np.full(q.shape, 7.0, np.float32)
        OK.paged_attention(out, q.astype(np.float32), k.astype(np.float32),
                           v.astype(np.float32), bt, ctx, 16)
        live = ctx > 0
        assert (ref[~live] == 7.0).all()           # ctx == 0: untouched (attention.cu:62)
        np.testing.assert_allclose(out[live], ref[live], atol=1e-3, rtol=2.0 ** -10)
    rq, rk, pos = x["rope"]
    qf, kf = rq.astype(np.float32).copy(), rk.astype(np.float32).copy()
    cos, sin = OK.rope_table(4096, 64, 1e6)
    OK.rope_inplace(qf, kf, cos, sin, pos)
    np.testing.assert_allclose(qf, g["rope_q"].astype(np.float32), atol=1e-3, rtol=2.0 ** -10)
    np.testing.assert_allclose(kf, g["rope_k"].astype(np.float32), atol=1e-3, rtol=2.0 ** -10)
    sw = OK.swiglu(x["swiglu"].astype(np.float32))
    np.testing.assert_allclose(sw, g["swiglu_out"].astype(np.float32), atol=1e-3, rtol=2.0 ** -10)
