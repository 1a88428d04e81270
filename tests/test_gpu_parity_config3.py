"""Parity of the decode step at the full-model decode configuration: 24 layers, hidden 896,
14/2 heads, vocab 151936, tied random-init bf16 weights (std 0.02), 32 sequences with context
lengths seeded U[128, 2048] and the KV pool pre-filled with N(0,1) values.

The CUDA path runs with the deterministic residual reduction (``model.deterministic``), so
every number here is reproducible from run to run.  The oracle (``oracle.model``, the numpy
restatement of models/qwen_25.py) runs in float32 with bf16 storage at the points where the
device stores bf16 ("an fp32 reference in bf16").

What this random-init model does to tiny differences sets what can be asserted.  Perturbing
the oracle's own float32 values by 2e-6 relative before each bf16 rounding (the size of
float32 accumulation-order differences) moves its residual stream by ~2e-3 max-abs after one
layer and by ~6e-2 after 24 (bf16 rounding flips of the activations, amplified layer by
layer), and makes most of its free-running greedy streams diverge within 64 tokens.  No bf16
implementation whose float32 sums run in another order can therefore stay within 2e-3 of the
oracle over 24 chained layers.  The tests below hold the 2e-3 bar where it is meaningful --
each layer given the oracle's own input -- and prove the rest stage by stage:

* ``test_layer_outputs_config3``: for each of the 24 layers, the GPU runs the layer on the
  oracle's input stream and every intermediate it stores is compared with what the oracle
  computes from the GPU's own previous intermediate (``decoder_layer(given=...)``): bf16
  tensors identical or one bf16 ulp apart (rounding flips, at most 1 % of the elements), the
  float32 stream to float32 accumulation precision.  The layer's output must then be within
  2e-3 max-abs of the oracle's, except at most 0.1 % of the elements, which the stage checks
  attribute to flips; the chained 24-layer stream is compared as well and must stay within
  twice the oracle's own noise floor.  Block tables are bit-exact.
* ``test_free_running_greedy_config3``: 8 sequences decode 64 greedy tokens free-running --
  the graph-captured ``DecodeEngine`` and the oracle each feed back their own tokens.  Every
  divergence must come at a step where the oracle's own top-2 margin is below twice its logit
  noise floor, and the engine must keep at least half as many identical tokens as the oracle
  keeps against itself under the 2e-6 perturbation (the same seeds, the same 8 x 64 steps).

With TI_PARITY_REPORT=<path> the measured numbers are written there as JSON.
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
MAX_ABS = 2e-3                 # per-layer bar against the oracle, each layer on the same input
MAX_OVER_FRAC = 1e-3           # layer-output elements allowed over it (flip-attributed)
MAX_FLIP_FRAC = 1e-2           # bf16 stage elements allowed one ulp away
REPORT = {}
BF16_STAGES = ("xn1", "q", "k", "v", "attn", "xn2", "act")
F32_STAGES = ("h_mid", "h_out")


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


def _bf16_ulp(x):
    """Spacing of bf16 values at |x| (2^(exponent - 7)); the smallest normal spacing at 0."""
    e = np.floor(np.log2(np.maximum(np.abs(x), 2.0 ** -126)))
    return np.exp2(e - 7).astype(np.float32)


def _gpu_layer(model, pb, kv, cos, sin, li, h_in):
    """Layer ``li`` on the GPU from the float32 stream ``h_in`` [B, H]; every stored stage."""
    cfg = model.config
    NH, KVH, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    got = {}

    def trace(layer, stage, tb):
        src = {"xn1": "xn", "qkv": "qkv", "attn": "attn", "h_mid": "hidden", "xn2": "xn",
               "act": "act", "h_out": "hidden"}[stage]
        got[stage] = tb[src].clone()

    model.forward_packed(pb, kv, cos, sin, first_layer=li, num_layers=li + 1,
                         hidden_in=torch.from_numpy(h_in), trace=trace, return_hidden=True)
    torch.cuda.synchronize()
    out = {k: v.float().cpu().numpy() for k, v in got.items()}
    out["q"] = out.pop("qkv")[:, :NH * D].reshape(-1, 1, NH, D)
    slot = pb.slot_mapping.long()
    blk, off = slot // kv.block_size, slot % kv.block_size
    out["k"] = kv.key_cache[li][blk, :, off].float().cpu().numpy().reshape(-1, 1, KVH, D)
    out["v"] = kv.value_cache[li][blk, :, off].float().cpu().numpy().reshape(-1, 1, KVH, D)
    return out


def test_layer_outputs_config3(full_model, cuda_device):
    cfg, model, W = full_model
    ocfg = OM.OracleConfig()
    kv, oc, ctx, rng = _prefilled(cfg, cuda_device, B, 8, seed=3)
    slots = np.arange(B)
    tokens = rng.integers(0, cfg.vocab_size, B)
    cos, sin = model.rope_tables(kv.max_seq_len)
    ocos, osin = OK.rope_table(kv.max_seq_len, cfg.head_dim, cfg.rope_theta)
    pb = model.plan(kv, list(slots), [1] * B, tokens)     # the step's new blocks (host FIFO)
    pos = OM.positions(oc, slots, 1)
    h = OM.embed(W, tokens[:, None])
    noise_cache = copy.deepcopy(oc)

    rows, over_total = [], 0
    chain_ref = []
    for li in range(cfg.num_layers):
        ref = {}
        h_next = OM.decoder_layer(W, ocfg, li, h, pos, slots, oc, ocos, osin,
                                  device_rounding="bf16", record=ref)
        got = _gpu_layer(model, pb, kv, cos, sin, li, h[:, 0].copy())
        sub = {}                     # each stage from the GPU's own previous stage
        OM.decoder_layer(W, ocfg, li, h, pos, slots, oc, ocos, osin, device_rounding="bf16",
                         record=sub, given={k: got[k] for k in BF16_STAGES + ("h_mid",)})
        row = {"layer": li}
        for st in BF16_STAGES:
            g, r = got[st].reshape(-1), sub[st].reshape(-1)
            d = np.abs(g - r)
            # one bf16 step at the larger of the two values, plus the float32 error of a value
            # that a sum produced by cancellation (relative to the stage's rms)
            rms = float(np.sqrt(np.mean(r.astype(np.float64) ** 2)))
            tol = _bf16_ulp(np.maximum(np.abs(g), np.abs(r))) * 1.0001 + 1e-5 * rms
            bad = np.nonzero(d > tol)[0]
            assert len(bad) == 0, (li, st, [(int(i), float(g[i]), float(r[i])) for i in bad[:8]])
            row[f"{st}_flips"] = int((d > 0).sum())
            assert row[f"{st}_flips"] <= MAX_FLIP_FRAC * d.size, (li, st, row[f"{st}_flips"])
        for st in F32_STAGES:
            g, r = got[st].reshape(-1), sub[st].reshape(-1)
            rms = float(np.sqrt(np.mean(r.astype(np.float64) ** 2)))
            row[f"{st}_f32_err"] = float(np.abs(g - r).max())
            assert row[f"{st}_f32_err"] <= 1e-4 * rms + 1e-6, (li, st, row[f"{st}_f32_err"], rms)
        err = np.abs(got["h_out"].reshape(B, -1) - ref["h_out"].reshape(B, -1))
        row.update(max_abs=float(err.max()), rms=float(np.sqrt(np.mean(err ** 2))),
                   over_bar=int((err > MAX_ABS).sum()),
                   ref_rms=float(np.sqrt(np.mean(ref["h_out"] ** 2))))
        over_total += row["over_bar"]
        assert row["over_bar"] <= MAX_OVER_FRAC * err.size, row
        rows.append(row)
        chain_ref.append(h_next[:, 0].copy())
        h = h_next
        print(row)
    np.testing.assert_array_equal(kv.block_tables.cpu().numpy(), oc.block_tables)

    # the chained 24 layers on the GPU against the oracle's chain and its own noise floor
    chain = []
    model.forward_packed(pb, kv, cos, sin, return_hidden=True,
                         trace=lambda li, st, tb: chain.append(tb["hidden"].clone())
                         if st == "h_out" else None)
    import oracle.model as OMm
    orig, prng = OMm.round_to, np.random.default_rng(321)
    OMm.round_to = lambda x, dt: orig(np.asarray(x, np.float32) * (
        1 + prng.standard_normal(np.shape(x)).astype(np.float32) * 2e-6), dt)
    pert = []
    try:
        OM.forward(W, ocfg, tokens[:, None], slots, noise_cache, ocos, osin,
                   device_rounding="bf16", layer_hook=lambda li, hh: pert.append(hh[:, 0].copy()))
    finally:
        OMm.round_to = orig
    chained = []
    for li in range(cfg.num_layers):
        e = float(np.abs(chain[li].cpu().numpy() - chain_ref[li]).max())
        floor = float(np.abs(pert[li] - chain_ref[li]).max())
        chained.append({"layer": li, "gpu_max_abs": e, "oracle_noise_max_abs": floor})
        print(chained[-1])
    _report("layer_outputs", {
        "config": f"{B} seqs, ctx U[{CTX_LO},{CTX_HI}] seed 3, 24 layers, N(0,1) KV, "
                  "deterministic residual; each layer on the oracle's input",
        "bar_max_abs": MAX_ABS, "elements_over_bar_total": over_total,
        "elements_per_layer": B * cfg.hidden_size, "layers": rows, "chained": chained})
    for c in chained:
        assert c["gpu_max_abs"] <= max(MAX_ABS, 2 * c["oracle_noise_max_abs"]), c


def _free_run(W, cache, first, slots, cos, sin, steps, noisy=False):
    """Greedy oracle stream, optionally with the 2e-6 perturbation; returns tokens and margins."""
    import oracle.model as OMm
    orig = OMm.round_to
    if noisy:
        prng = np.random.default_rng(321)
        OMm.round_to = lambda x, dt: orig(np.asarray(x, np.float32) * (
            1 + prng.standard_normal(np.shape(x)).astype(np.float32) * 2e-6), dt)
    toks, hist, margins = first.copy(), [], []
    try:
        for _ in range(steps):
            lg = OM.forward(W, OM.OracleConfig(), toks[:, None], np.asarray(slots), cache, cos,
                            sin, device_rounding="bf16")[:, 0]
            cache.seq_len[np.asarray(slots)] += 1
            toks = np.argmax(lg, axis=-1)
            srt = np.sort(lg, axis=-1)
            hist.append(toks.copy())
            margins.append(srt[:, -1] - srt[:, -2])
    finally:
        OMm.round_to = orig
    return np.array(hist), np.array(margins)


def _logit_noise_floor(W, ids, slots, cache, cos, sin):
    """Largest change of the oracle's logits under the 2e-6 perturbation (copies of the cache)."""
    import oracle.model as OMm
    cfg = OM.OracleConfig()
    base = OM.forward(W, cfg, ids, np.asarray(slots), copy.deepcopy(cache), cos, sin,
                      device_rounding="bf16")
    orig, prng = OMm.round_to, np.random.default_rng(321)
    OMm.round_to = lambda x, dt: orig(np.asarray(x, np.float32) * (
        1 + prng.standard_normal(np.shape(x)).astype(np.float32) * 2e-6), dt)
    try:
        pert = OM.forward(W, cfg, ids, np.asarray(slots), copy.deepcopy(cache), cos, sin,
                          device_rounding="bf16")
    finally:
        OMm.round_to = orig
    return float(np.abs(base - pert).max())


def _first_divergence(a, b):
    d = np.nonzero(a != b)[0]
    return int(d[0]) if len(d) else None


def test_free_running_greedy_config3(full_model, cuda_device):
    from tiny_infra_b200.engine import DecodeEngine
    cfg, model, W = full_model
    kv, oc, ctx, rng = _prefilled(cfg, cuda_device, FREE_SEQS, STEPS + 8, seed=7)
    slots = list(range(FREE_SEQS))
    first = rng.integers(0, cfg.vocab_size, FREE_SEQS)
    ocos, osin = OK.rope_table(kv.max_seq_len, cfg.head_dim, cfg.rope_theta)
    tau = 2 * _logit_noise_floor(W, first[:, None], slots, oc, ocos, osin)
    noisy_cache = copy.deepcopy(oc)

    eng = DecodeEngine(model, kv)
    g_tok, g_hist = first.copy(), []
    for _ in range(STEPS):
        g_tok = eng.step(slots, g_tok)
        g_hist.append(np.asarray(g_tok).copy())
    g_hist = np.array(g_hist)
    o_hist, margins = _free_run(W, oc, first, slots, ocos, osin, STEPS)
    np.testing.assert_array_equal(kv.block_tables.cpu().numpy(), oc.block_tables)
    np.testing.assert_array_equal(kv.seq_len.cpu().numpy(), oc.seq_len)
    n_hist, _ = _free_run(W, noisy_cache, first, slots, ocos, osin, STEPS, noisy=True)

    seqs = []
    for i in range(FREE_SEQS):
        d = _first_divergence(g_hist[:, i], o_hist[:, i])
        dn = _first_divergence(n_hist[:, i], o_hist[:, i])
        seqs.append({"seq": i, "ctx": int(ctx[i]), "engine_first_divergence": d,
                     "oracle_margin_at_divergence": None if d is None else float(margins[d, i]),
                     "engine_identical_tokens": STEPS if d is None else d,
                     "perturbed_oracle_first_divergence": dn,
                     "perturbed_oracle_identical_tokens": STEPS if dn is None else dn})
        print(seqs[-1])
    eng_same = sum(s["engine_identical_tokens"] for s in seqs)
    orc_same = sum(s["perturbed_oracle_identical_tokens"] for s in seqs)
    _report("free_running", {
        "config": f"{FREE_SEQS} seqs, ctx U[{CTX_LO},{CTX_HI}] seed 7, {STEPS} greedy steps, "
                  "engine and oracle each feeding back their own tokens",
        "tau_near_tie": tau, "engine_identical_tokens": eng_same,
        "perturbed_oracle_identical_tokens": orc_same, "tokens": FREE_SEQS * STEPS,
        "engine_identical_sequences": sum(s["engine_first_divergence"] is None for s in seqs),
        "perturbed_oracle_identical_sequences":
            sum(s["perturbed_oracle_first_divergence"] is None for s in seqs),
        "sequences": seqs})
    for s in seqs:
        if s["engine_first_divergence"] is not None:
            assert s["oracle_margin_at_divergence"] < tau, (s, tau)
    assert eng_same >= orc_same // 2, (eng_same, orc_same)
