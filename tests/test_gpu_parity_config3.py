"""Parity of the full decode step at the full-model decode configuration: 24 layers, hidden 896,
14/2 heads, vocab 151936, tied random-init bf16 weights (std 0.02), 32 sequences with context
lengths seeded U[128, 2048] and the KV pool pre-filled with N(0,1) values.

The CUDA path runs with the deterministic residual reduction (``model.deterministic``: the
split-K slices of the O and down projections are summed in a fixed order), so every number
below is reproducible from run to run.  The oracle (``oracle.model``, the numpy restatement of
models/qwen_25.py) runs in float32 with bf16 storage at the points where the device stores
bf16 ("an fp32 reference in bf16").

* ``test_layer_outputs_config3``: one decode step of all 32 sequences; the float32 residual
  stream after EVERY one of the 24 layers must be within 2e-3 max-abs of the oracle's, and the
  block tables (including the step's new blocks) bit-exact.
* ``test_free_running_greedy_config3``: 8 of the sequences decode 64 greedy tokens
  free-running -- the engine (graph-captured ``DecodeEngine``) and the oracle each feed back
  their own tokens -- and the streams must be identical.  At most one sequence may diverge,
  and only at a step where the oracle's own top-2 logit margin is below twice its logit noise
  floor (a near-tie that bf16 storage cannot decide); the first divergence index and margin are
  reported.

With TI_PARITY_REPORT=<path> the measured per-layer errors and the stream report are written
there as JSON.
"""
import copy
import json
import os

import numpy as np
import pytest
import torch

from oracle import kernels as OK
from oracle import model as OM
from oracle.cache import OracleKVCache

pytestmark = pytest.mark.gpu

B, CTX_LO, CTX_HI = 32, 128, 2048
STEPS, FREE_SEQS = 64, 8
MAX_ABS = 2e-3                     # layer outputs: max-abs bar against the oracle
MAX_NEAR_TIE_SEQS = 1              # free-running: sequences allowed to diverge at a near-tie
REPORT = {}


def _report(key, value):
    REPORT[key] = value
    path = os.environ.get("TI_PARITY_REPORT")
    if path:
        with open(path, "w") as f:
            json.dump(REPORT, f, indent=1)


@pytest.fixture(scope="module")
def full_model(cuda_device):
    from tiny_infra_b200.config import QwenConfig
    from tiny_infra_b200.qwen2 import Qwen2ForCausalLM
    cfg = QwenConfig()
    sd = Qwen2ForCausalLM.random_state_dict(cfg, seed=0, tied=True, device=cuda_device)
    model = Qwen2ForCausalLM(cfg, device=cuda_device).load_reference_state_dict(sd)
    model.deterministic = True
    W = {k: v.float().cpu().numpy() for k, v in sd.items()}
    W["lm_head.weight"] = W["model.embed_tokens.weight"]
    del sd
    return cfg, model, W


def _prefilled(cfg, cuda_device, n, extra, seed):
    """KV cache with ``n`` sequences at seeded lengths U[128, 2048], N(0,1) KV in every layer,
    and the oracle's mirror of it (same block tables, same FIFO free list, same pool values)."""
    from tiny_infra_b200.cache_manager import KVCacheManager
    rng = np.random.default_rng(seed)
    ctx = rng.integers(CTX_LO, CTX_HI + 1, n).astype(np.int32)
    max_seq = CTX_HI + extra + 16
    nb = int(sum((int(c) + extra + 15) // 16 for c in ctx)) + 8
    kv = KVCacheManager(n, max_seq, cfg.num_layers, cfg.num_key_value_heads, cfg.head_dim,
                        device=cuda_device, num_blocks=nb)
    slots = list(range(n))
    kv.plan_tokens(slots, [int(c) for c in ctx])
    g = torch.Generator(device=cuda_device)
    g.manual_seed(seed + 100)
    for li in range(cfg.num_layers):
        kv.key_cache[li].normal_(generator=g)
        kv.value_cache[li].normal_(generator=g)
    kv.advance_device(slots, [int(c) for c in ctx])
    oc = OracleKVCache(n, max_seq, cfg.num_layers, cfg.num_key_value_heads, cfg.head_dim,
                       allocate_pool=False, num_blocks=nb)
    oc.key_cache = kv.key_cache.float().cpu().numpy()
    oc.value_cache = kv.value_cache.float().cpu().numpy()
    oc.block_tables[:] = kv.block_tables.cpu().numpy()
    oc.free_blocks = [int(b) for b in kv.free_blocks]
    oc.seq_len[:] = kv.seq_len.cpu().numpy()
    np.testing.assert_array_equal(oc.seq_len, ctx)
    return kv, oc, ctx, rng


def test_layer_outputs_config3(full_model, cuda_device):
    cfg, model, W = full_model
    kv, oc, ctx, rng = _prefilled(cfg, cuda_device, B, 8, seed=3)
    slots = list(range(B))
    tokens = rng.integers(0, cfg.vocab_size, B)
    cos, sin = model.rope_tables(kv.max_seq_len)
    ocos, osin = OK.rope_table(kv.max_seq_len, cfg.head_dim, cfg.rope_theta)

    pb = model.plan(kv, slots, [1] * B, tokens)
    layers = []
    model.forward_packed(pb, kv, cos, sin, rows="last", layer_out=layers)
    got = [h.cpu().numpy() for h in layers]

    ref = {}
    OM.forward(W, OM.OracleConfig(), tokens[:, None], np.array(slots), oc, ocos, osin,
               device_rounding="bf16", layer_hook=lambda li, h: ref.__setitem__(li, h[:, 0].copy()))
    np.testing.assert_array_equal(kv.block_tables.cpu().numpy(), oc.block_tables)

    rows = []
    for li in range(cfg.num_layers):
        err = np.abs(got[li] - ref[li])
        i = np.unravel_index(int(np.argmax(err)), err.shape)
        rows.append({"layer": li, "max_abs": float(err.max()),
                     "rms": float(np.sqrt(np.mean(err ** 2))),
                     "over_bar": int((err > MAX_ABS).sum()),
                     "ref_max_abs": float(np.abs(ref[li]).max()),
                     "ref_rms": float(np.sqrt(np.mean(ref[li] ** 2))),
                     "worst": [int(i[0]), int(i[1])]})
    for r in rows:
        print("layer {layer:2d}: max-abs {max_abs:.3e} rms {rms:.3e} (|ref| max {ref_max_abs:.3f}, "
              "rms {ref_rms:.3f}) elements over {bar}: {over_bar}".format(bar=MAX_ABS, **r))
    _report("layer_outputs", {"config": f"{B} seqs, ctx U[{CTX_LO},{CTX_HI}] seed 3, "
                                        "24 layers, N(0,1) KV, deterministic residual",
                              "bar_max_abs": MAX_ABS, "layers": rows})
    bad = [r for r in rows if r["max_abs"] > MAX_ABS]
    assert not bad, bad


def _logit_noise_floor(W, ids, slots, cache, cos, sin):
    """Largest change of the oracle's logits when its float32 values are perturbed by 2e-6
    relative before each bf16 rounding (accumulation-order noise), on copies of the cache."""
    import oracle.model as OMm
    cfg = OM.OracleConfig()
    base = OM.forward(W, cfg, ids, np.asarray(slots), copy.deepcopy(cache), cos, sin,
                      device_rounding="bf16")
    orig = OMm.round_to
    rng = np.random.default_rng(321)
    OMm.round_to = lambda x, dt: orig(np.asarray(x, np.float32) * (
        1 + rng.standard_normal(np.shape(x)).astype(np.float32) * 2e-6), dt)
    try:
        pert = OM.forward(W, cfg, ids, np.asarray(slots), copy.deepcopy(cache), cos, sin,
                          device_rounding="bf16")
    finally:
        OMm.round_to = orig
    return float(np.abs(base - pert).max())


def test_free_running_greedy_config3(full_model, cuda_device):
    from tiny_infra_b200.engine import DecodeEngine
    cfg, model, W = full_model
    kv, oc, ctx, rng = _prefilled(cfg, cuda_device, FREE_SEQS, STEPS + 8, seed=7)
    slots = list(range(FREE_SEQS))
    first = rng.integers(0, cfg.vocab_size, FREE_SEQS)
    eng = DecodeEngine(model, kv)
    ocos, osin = OK.rope_table(kv.max_seq_len, cfg.head_dim, cfg.rope_theta)
    # the near-tie bar: the oracle's logit noise floor on the first step's inputs (measured on
    # copies of the cache, before the streams start)
    tau = 2 * _logit_noise_floor(W, first[:, None], slots, oc, ocos, osin)

    g_tok, o_tok = first.copy(), first.copy()
    g_hist, o_hist, margins = [], [], []
    for step in range(STEPS):
        g_tok = eng.step(slots, g_tok)
        lg = OM.forward(W, OM.OracleConfig(), o_tok[:, None], np.array(slots), oc, ocos, osin,
                        device_rounding="bf16")[:, 0]
        oc.seq_len[np.array(slots)] += 1
        o_tok = np.argmax(lg, axis=-1)
        srt = np.sort(lg, axis=-1)
        g_hist.append(np.asarray(g_tok).copy())
        o_hist.append(o_tok.copy())
        margins.append(srt[:, -1] - srt[:, -2])
        np.testing.assert_array_equal(kv.block_tables.cpu().numpy(), oc.block_tables)
    np.testing.assert_array_equal(kv.seq_len.cpu().numpy(), oc.seq_len)
    g_hist, o_hist, margins = np.array(g_hist), np.array(o_hist), np.array(margins)

    seqs = []
    for i in range(FREE_SEQS):
        diff = np.nonzero(g_hist[:, i] != o_hist[:, i])[0]
        d = int(diff[0]) if len(diff) else None
        seqs.append({"seq": i, "ctx": int(ctx[i]), "first_divergence": d,
                     "oracle_margin_at_divergence": None if d is None else float(margins[d, i]),
                     "identical_tokens": STEPS if d is None else d,
                     "min_oracle_margin_before": float(margins[:STEPS if d is None else d + 1,
                                                               i].min())})
        print(seqs[-1])
    diverged = [s for s in seqs if s["first_divergence"] is not None]
    _report("free_running", {"config": f"{FREE_SEQS} seqs, ctx U[{CTX_LO},{CTX_HI}] seed 7, "
                                       f"{STEPS} greedy steps each, engine vs oracle each "
                                       "feeding back its own tokens",
                             "tau_near_tie": tau, "max_near_tie_seqs": MAX_NEAR_TIE_SEQS,
                             "identical_sequences": FREE_SEQS - len(diverged),
                             "sequences": seqs})
    assert len(diverged) <= MAX_NEAR_TIE_SEQS, diverged
    for s in diverged:
        assert s["oracle_margin_at_divergence"] < tau, (s, tau)
