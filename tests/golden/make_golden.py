"""Generate golden vectors by running the reference project's own Python code on the CPU.

Run where the reference checkout is available (a CUDA machine need not have it):

    python tests/golden/make_golden.py --ref <reference checkout>

The reference's ``models/qwen_25.py`` imports three native modules (``engine.ops.custom_*``)
whose prebuilt binaries are absent from the reference checkout.  This script registers a
shim ``engine.ops`` package whose three functions call the oracle's float32 restatements of
``src/attention.cu``, ``src/fused_rope.cu`` and ``src/fused_swiglu.cu``; those restatements
are pinned separately against the reference kernels themselves (make_kernel_golden.py).
Everything else -- the allocator, the scheduler, the sampler, the model's layer structure, the
RoPE table -- is the reference's own code.

Outputs (small, committed): cache_ops.json/.npz, rope_table.npz, sampler.npz, model_forward.npz,
scheduler_trace.json.
"""
from __future__ import annotations

import argparse
import asyncio
import hashlib
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import kernels as OK  # noqa: E402
from oracle.model import OracleConfig, init_weights  # noqa: E402


def install_ops_shim() -> None:
    """Register ``engine.ops.custom_{paged_attn,rope,swiglu}`` backed by the oracle."""
    import engine  # the reference package (sys.path set by the caller)

    ops = types.ModuleType("engine.ops")
    ops.__path__ = []

    pa = types.ModuleType("engine.ops.custom_paged_attn")

    def launch_paged_attention(out, q, k_cache, v_cache, block_tables, context_lens, block_size):
        o = out.detach().cpu().numpy().astype(np.float32)
        OK.paged_attention(o, q.detach().cpu().numpy(), k_cache.detach().cpu().numpy(),
                           v_cache.detach().cpu().numpy(), block_tables.cpu().numpy(),
                           context_lens.cpu().numpy(), int(block_size))
        out.copy_(torch.from_numpy(o).to(out.dtype))

    pa.launch_paged_attention = launch_paged_attention

    rp = types.ModuleType("engine.ops.custom_rope")

    def apply_inplace(q, k, cos, sin, pos_ids):
        qn = q.detach().cpu().numpy().astype(np.float32).copy()
        kn = k.detach().cpu().numpy().astype(np.float32).copy()
        OK.rope_inplace(qn, kn, cos.cpu().numpy(), sin.cpu().numpy(),
                        pos_ids.cpu().numpy().astype(np.int64))
        q.copy_(torch.from_numpy(qn).to(q.dtype))
        k.copy_(torch.from_numpy(kn).to(k.dtype))

    rp.apply_inplace = apply_inplace

    sw = types.ModuleType("engine.ops.custom_swiglu")
    sw.forward = lambda x: torch.from_numpy(OK.swiglu(x.detach().cpu().numpy())).to(x.dtype)

    ops.custom_paged_attn, ops.custom_rope, ops.custom_swiglu = pa, rp, sw
    sys.modules["engine.ops"] = ops
    sys.modules["engine.ops.custom_paged_attn"] = pa
    sys.modules["engine.ops.custom_rope"] = rp
    sys.modules["engine.ops.custom_swiglu"] = sw
    engine.ops = ops


# ---------------------------------------------------------------------------------------------
def cache_ops(out_dir: str) -> None:
    """Run a scripted sequence of KVCacheManager calls; record tables, lengths, free list and
    pool contents after every call (engine/cache_manager.py)."""
    from engine.cache_manager import KVCacheManager

    rng = np.random.default_rng(11)
    L, KVH, D, bs = 2, 2, 8, 16
    mgr = KVCacheManager(max_batch_size=4, max_seq_len=64, num_layers=L, num_kv_heads=KVH,
                         head_dim=D, block_size=bs, device=torch.device("cpu"),
                         dtype=torch.float32)
    script = [
        ("insert", [0], 25), ("advance", [0], 25),
        ("insert", [1], 12), ("advance", [1], 12),
        ("insert", [2], 33), ("advance", [2], 33),
        ("insert", [0, 1, 2], 1), ("advance", [0, 1, 2], 1),
        ("free", 0),
        ("insert", [3], 40), ("advance", [3], 40),
        ("insert", [1, 3, 2], 1), ("advance", [1, 3, 2], 1),
        ("insert", [0], 16), ("advance", [0], 16),
        ("free", 2),
        ("insert", [2], 70),          # position 64 >= max_seq_len -> ValueError mid-insert
        ("free", 2),
        ("insert", [1], 4), ("advance", [1], 4),
        ("insert", [2], 50), ("advance", [2], 50),
        ("truncate_free", 2),         # shrink the public free list to two blocks
        ("insert", [0, 1], 30),       # runs out of free blocks -> RuntimeError (OOM)
        ("free", 1), ("free", 3), ("free", 0), ("free", 2),
        ("insert", [], 1),            # empty batch -> ValueError
        ("free", 4),                  # out of range -> IndexError
    ]
    records, arrays = [], {}
    for i, op in enumerate(script):
        err = None
        if op[0] == "insert":
            _, idx, n = op
            k = rng.standard_normal((len(idx), KVH, n, D)).astype(np.float32)
            v = rng.standard_normal((len(idx), KVH, n, D)).astype(np.float32)
            arrays[f"k{i}"], arrays[f"v{i}"] = k, v
            try:
                for layer in range(L):
                    mgr.allocate_and_insert(layer, torch.tensor(idx, dtype=torch.int32),
                                            torch.from_numpy(k), torch.from_numpy(v))
            except Exception as e:  # noqa: BLE001 - the exception type is what we record
                err = type(e).__name__
        elif op[0] == "advance":
            _, idx, n = op
            mgr.seq_len[torch.tensor(idx, dtype=torch.long)] += n
        elif op[0] == "truncate_free":
            del mgr.free_blocks[op[1]:]
        elif op[0] == "free":
            try:
                mgr.free_batch_slot(op[1])
            except Exception as e:  # noqa: BLE001
                err = type(e).__name__
        records.append({"op": list(op), "error": err,
                        "block_tables": mgr.block_tables.tolist(),
                        "seq_len": mgr.seq_len.tolist(),
                        "free_blocks": list(mgr.free_blocks)})
        records[-1]["key_sha256"] = hashlib.sha256(mgr.key_cache.numpy().tobytes()).hexdigest()
        records[-1]["val_sha256"] = hashlib.sha256(mgr.value_cache.numpy().tobytes()).hexdigest()
    arrays["key_final"] = mgr.key_cache.numpy().copy()
    arrays["val_final"] = mgr.value_cache.numpy().copy()
    with open(os.path.join(out_dir, "cache_ops.json"), "w") as f:
        json.dump({"config": {"max_batch_size": 4, "max_seq_len": 64, "num_layers": L,
                              "num_kv_heads": KVH, "head_dim": D, "block_size": bs},
                   "records": records}, f)
    np.savez_compressed(os.path.join(out_dir, "cache_ops.npz"), **arrays)


def rope_table(out_dir: str) -> None:
    """``ContinuousBatcher._init_rope_cache`` (engine/scheduler.py:36-48) at 32768 positions;
    rows 0..255 and every 97th row are stored."""
    from engine.scheduler import ContinuousBatcher

    fake_cache = types.SimpleNamespace(max_batch_size=1, max_seq_len=32768, head_dim=64,
                                       device=torch.device("cpu"))
    b = ContinuousBatcher(model=None, kv_cache=fake_cache)
    rows = np.unique(np.concatenate([np.arange(256), np.arange(0, 32768, 97), [32767]]))
    np.savez_compressed(os.path.join(out_dir, "rope_table.npz"), rows=rows,
                        cos=b.cos_cache.numpy()[rows], sin=b.sin_cache.numpy()[rows])


def sampler(out_dir: str) -> None:
    """``_sample_next_token`` (engine/scheduler.py:104-156): the distribution handed to
    ``torch.multinomial`` (captured by patching it) and the final tokens of greedy rows."""
    from engine.scheduler import ContinuousBatcher, GenerationRequest

    fake_cache = types.SimpleNamespace(max_batch_size=8, max_seq_len=16, head_dim=64,
                                       device=torch.device("cpu"))
    b = ContinuousBatcher(model=None, kv_cache=fake_cache)
    rng = np.random.default_rng(5)
    V = 1000
    cases = {
        "uniform_k": ([0.7, 0.7, 1.0, 0.0, 1.3], [50, 50, 50, 50, 50], [0.9, 0.9, 0.5, 0.9, 1.0]),
        "mixed_k": ([0.7, 1.0, 0.0, 0.5], [20, 50, 5, 50], [0.9, 1.0, 0.9, 0.8]),
        "no_topp": ([0.7, 1.2, 0.0], [20, 20, 20], [1.0, 1.0, 1.0]),
        "full_vocab": ([0.8, 0.0, 1.0], [0, 0, 0], [0.95, 0.95, 0.7]),
        "ties": ([1.0, 0.0], [3, 3], [0.9, 0.9]),
    }
    out = {}
    real_multinomial = torch.multinomial
    for name, (temps, ks, ps) in cases.items():
        B = len(temps)
        logits = rng.standard_normal((B, 1, V)).astype(np.float32) * 3.0
        if name == "ties":
            logits[:, 0, :] = np.round(logits[:, 0, :])
        reqs = [GenerationRequest([1], 1, temperature=t, p_value=p, top_k=k)
                for t, k, p in zip(temps, ks, ps)]
        captured = {}

        def fake_multinomial(probs, num_samples=1, **kw):
            captured["probs"] = probs.detach().clone()
            return real_multinomial(probs, num_samples, **kw)

        torch.multinomial = fake_multinomial
        try:
            toks = b._sample_next_token(torch.from_numpy(logits), reqs)
        finally:
            torch.multinomial = real_multinomial
        out[f"{name}_logits"] = logits[:, 0, :]
        out[f"{name}_temps"] = np.array(temps, np.float32)
        out[f"{name}_topk"] = np.array(ks, np.int64)
        out[f"{name}_topp"] = np.array(ps, np.float32)
        out[f"{name}_probs"] = captured["probs"].numpy()
        out[f"{name}_tokens"] = np.array(toks, np.int64)
    np.savez_compressed(os.path.join(out_dir, "sampler.npz"), **out)


SMALL = dict(vocab_size=300, hidden_size=256, num_layers=2, num_attention_heads=4,
             num_key_value_heads=2, intermediate_size=512)


def _small_reference_model(seed: int):
    from models.config import QwenConfig
    from models.qwen_25 import Qwen2ForCausalLM

    cfg = QwenConfig(**SMALL)
    ocfg = OracleConfig(**SMALL)
    W = init_weights(ocfg, seed=seed, tied=False, bf16=False)
    model = Qwen2ForCausalLM(cfg)
    model.load_state_dict({k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in W.items()},
                          strict=True)
    return model.eval(), cfg


def model_forward(out_dir: str) -> None:
    """``Qwen2ForCausalLM.forward`` (models/qwen_25.py) with a small config in fp32: two prefills
    then two batched decode steps, with the scheduler's seq_len updates in between."""
    from engine.cache_manager import KVCacheManager
    from engine.scheduler import ContinuousBatcher

    model, cfg = _small_reference_model(seed=3)
    kv = KVCacheManager(max_batch_size=3, max_seq_len=64, num_layers=cfg.num_layers,
                        num_kv_heads=cfg.num_key_value_heads, head_dim=64, block_size=16,
                        device=torch.device("cpu"), dtype=torch.float32)
    sched = ContinuousBatcher(model, kv)
    cos, sin = sched.cos_cache, sched.sin_cache
    rng = np.random.default_rng(9)
    calls = [([0], rng.integers(0, cfg.vocab_size, (1, 20))),
             ([2], rng.integers(0, cfg.vocab_size, (1, 7))),
             ([0, 2], rng.integers(0, cfg.vocab_size, (2, 1))),
             ([0, 2], rng.integers(0, cfg.vocab_size, (2, 1)))]
    out = {"num_calls": np.array(len(calls))}
    with torch.no_grad():
        for i, (idx, ids) in enumerate(calls):
            bi = torch.tensor(idx, dtype=torch.int32)
            logits = model(torch.from_numpy(ids.astype(np.int32)), bi, kv, cos, sin)
            kv.seq_len[bi] += ids.shape[1]
            out[f"ids{i}"] = ids.astype(np.int64)
            out[f"idx{i}"] = np.array(idx, np.int64)
            out[f"logits{i}"] = logits.numpy()
    out["block_tables"] = kv.block_tables.numpy()
    out["seq_len"] = kv.seq_len.numpy()
    np.savez_compressed(os.path.join(out_dir, "model_forward.npz"), **out)


class _TraceModel:
    """Deterministic stand-in model for the scheduler trace: writes layer-0 KV through the
    cache manager (so block allocation happens exactly as with the real model) and returns
    logits whose argmax is a fixed function of the last input token and its position."""

    def __init__(self, vocab: int, eos: int):
        self.vocab, self.eos = vocab, eos

    def __call__(self, input_ids, batch_indices, kv_cache, cos, sin):
        B, S = input_ids.shape
        start = kv_cache.seq_len[batch_indices.long()]
        z = torch.zeros(B, kv_cache.num_kv_heads, S, kv_cache.head_dim)
        for layer in range(kv_cache.num_layers):
            kv_cache.allocate_and_insert(layer, batch_indices, z, z)
        last = input_ids[:, -1].long()
        pos = start.long() + S - 1
        nxt = (last * 7 + pos * 3 + 1) % self.vocab
        logits = torch.zeros(B, S, self.vocab)
        logits[torch.arange(B), -1, nxt] = 5.0
        return logits


def scheduler_trace(out_dir: str) -> None:
    """Drive ``ContinuousBatcher._fill_active_slots`` / ``_step_generation`` by hand with
    staggered arrivals and greedy requests; record every step (engine/scheduler.py:89-281)."""
    from engine.cache_manager import KVCacheManager
    from engine.scheduler import ContinuousBatcher, _END_OF_STREAM

    vocab, eos = 97, 13
    kv = KVCacheManager(max_batch_size=3, max_seq_len=48, num_layers=2, num_kv_heads=2,
                        head_dim=8, block_size=16, device=torch.device("cpu"),
                        dtype=torch.float32)
    sched = ContinuousBatcher(_TraceModel(vocab, eos), kv, eos_token_id=eos)
    rng = np.random.default_rng(21)
    arrivals = {0: 2, 1: 1, 3: 2, 6: 1, 9: 2}       # step -> number of new requests
    requests, specs, steps = [], [], []

    async def drive():
        from engine.scheduler import GenerationRequest
        for step in range(40):
            for _ in range(arrivals.get(step, 0)):
                plen = int(rng.integers(3, 40))
                prompt = [int(x) for x in rng.integers(0, vocab, plen)]
                mnt = int(rng.integers(1, 12))
                req = GenerationRequest(prompt, mnt, temperature=0.0, p_value=0.9, top_k=20)
                requests.append(req)
                specs.append({"prompt": prompt, "max_new_tokens": mnt})
                await sched.requests_queue.put(req)
            sched._fill_active_slots()
            slots_before = [requests.index(r) if r is not None else None
                            for r in sched.active_slots]
            if any(r is not None for r in sched.active_slots):
                sched._step_generation()
            emitted = {}
            for ri, r in enumerate(requests):
                toks = []
                while not r.token_queue.empty():
                    t = r.token_queue.get_nowait()
                    toks.append("END" if t is _END_OF_STREAM else int(t))
                if toks:
                    emitted[ri] = toks
            steps.append({"step": step, "slots": slots_before, "emitted": emitted,
                          "block_tables": kv.block_tables.tolist(), "seq_len": kv.seq_len.tolist(),
                          "free_blocks": list(kv.free_blocks)})

    asyncio.run(drive())
    with open(os.path.join(out_dir, "scheduler_trace.json"), "w") as f:
        json.dump({"vocab": vocab, "eos": eos,
                   "cache": {"max_batch_size": 3, "max_seq_len": 48, "num_layers": 2,
                             "num_kv_heads": 2, "head_dim": 8, "block_size": 16},
                   "arrivals": {str(k): v for k, v in arrivals.items()},
                   "requests": specs, "steps": steps,
                   "final": [r.generated_tokens for r in requests]}, f)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=None, help="reference checkout (default: $TINY_INFRA_REF)")
    ap.add_argument("--out", default=HERE)
    a = ap.parse_args()
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from oracle.build_ref import reference_root
    ref = reference_root(a.ref)
    if ref is None:
        ap.error("no reference checkout: pass --ref or set TINY_INFRA_REF")
    sys.path.insert(0, ref)
    torch.manual_seed(0)
    install_ops_shim()
    import builtins
    real_print = builtins.print
    builtins.print = lambda *x, **k: None    # the reference prints on every slot change
    try:
        cache_ops(a.out)
        rope_table(a.out)
        sampler(a.out)
        model_forward(a.out)
        scheduler_trace(a.out)
    finally:
        builtins.print = real_print
    print("golden vectors written to", a.out)


if __name__ == "__main__":
    main()
