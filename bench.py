"""Decode throughput of the Qwen2.5-0.5B continuous-batching hot path on B200.

Workload (one engine replica per GPU, weak scaling): 256 ragged sequences per GPU, context
lengths seeded uniform in [128, 2048], KV pool pre-filled with N(0,1) values, random-init bf16
weights (std 0.02, tied embeddings), greedy decoding.  A step is one decode step for all 256
sequences: block-table update, 24 layers, final norm, lm_head + argmax, seq_len advance.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
  python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...

Prints one JSON line (rank 0).  `value` is device-timed with inputs resident in HBM (tokens fed
back on the device, no host round trip between steps); `e2e` is the same metric through the
public per-step API (`DecodeEngine.step`: host token lists in and out, pinned H2D/D2H copies and
a sync every step).  `--impl reference` times the oracle (numpy restatement of the reference's
CPU PyTorch path) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time


def _cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# The CPU arms (the reference arm, and the cpu_baseline leg) run the numpy oracle, whose BLAS
# reads its thread count when numpy is first imported; torchrun exports OMP_NUM_THREADS=1 to
# every rank.  Rank 0 does all the CPU work (the other ranks only wait), so it gets every host
# core before numpy loads.
if os.environ.get("RANK", "0") == "0":
    for _v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[_v] = str(_cores())

import numpy as np  # noqa: E402

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "decode tokens/sec @256 ragged seqs per B200 (1/2/4/8); paged-attn HBM GB/s"
SEQS = 256
CTX_LO, CTX_HI = 128, 2048
CPU_SAMPLE_SEQS = 32
WINDOW = 16          # decode steps between context-length resets (stationary workload)
REF_MAX_SECONDS = 60.0   # reference arm: cap on the timed oracle steps' work


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--seqs", type=int, default=SEQS,
                    help="decode workload: sequences per GPU (256: the headline; 32: the "
                         "full-model decode configuration of 32 sequences)")
    ap.add_argument("--workload", choices=["decode", "serving", "long"], default="decode",
                    help="decode: the 256-sequence decode step (the headline metric); serving: "
                         "a Poisson request stream through the continuous batcher")
    ap.add_argument("--requests", type=int, default=1024, help="serving: number of requests")
    ap.add_argument("--rate", type=float, default=64.0, help="serving: arrivals per second")
    ap.add_argument("--lm-head", choices=["bf16", "int8"], default="bf16",
                    help="decode workload: the greedy lm_head's weights (int8: weight-only "
                         "int8 copy with per-row scales)")
    ap.add_argument("--kernel", choices=["attention", "gate_up", "rmsnorm", "sampler",
                                         "prefill_gemm", "prefill_attention", "lm_head",
                                         "lm_head_int8", "qkv", "o_proj", "down"], default=None,
                    help="time one kernel alone instead of the decode step")
    ap.add_argument("--case", choices=["256", "config1", "long"], default="256",
                    help="attention case: one layer of the 256-sequence workload, or the "
                         "8-sequence ctx U[1,512] paged-attention op")
    ap.add_argument("--rows", type=int, default=4096,
                    help="rmsnorm kernel: rows per launch (4096: a prefill chunk; 256: one decode "
                         "step's batch)")
    return ap.parse_args()


def _dist():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def _config(world, extra=None):
    c = {"workload": f"qwen2.5-0.5b decode step, {SEQS} ragged seqs/GPU, ctx U[128,2048], "
                     "greedy, random-init bf16 weights (std 0.02, tied), KV pre-filled N(0,1)",
         "seqs_per_gpu": SEQS, "ctx_range": [CTX_LO, CTX_HI], "block_size": 16,
         "parallelism": f"replicas x{world} (no collectives)",
         "context_window": f"lengths reset to the sampled ctx every {WINDOW} steps: each step "
                           f"decodes at ctx + 0..{WINDOW - 1}; timed steps replayed as one "
                           f"CUDA graph per {WINDOW}-step window",
         "l2": "inputs larger than L2 (~4.4 GB read per step), no flush"}
    if extra:
        c.update(extra)
    return c


def _peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _traffic_from_profiles():
    """DRAM bytes per launch of the attention kernel from the committed ncu summary, scaled to
    this workload's algorithmic bytes when the capture was a smaller case."""
    p = os.path.join(REPO, "profiles", "paged_attention_decode_256seqs.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":")[1].split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled in the background during a timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.5)
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        mhz, mx, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                mhz.append(float(f[1]))
                mx = float(f[2])
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(mhz)) if mhz else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(mhz),
                "power_w_max": max(power) if power else None}


# ---------------------------------------------------------------------------------------------
def build_workload(device, seed, steps_total, lm_head="bf16"):
    """Engine replica with SEQS sequences at their sampled context lengths, KV pre-filled."""
    import torch
    from tiny_infra_b200.cache_manager import KVCacheManager
    from tiny_infra_b200.config import QwenConfig
    from tiny_infra_b200.engine import DecodeEngine
    from tiny_infra_b200.qwen2 import Qwen2ForCausalLM

    cfg = QwenConfig()
    rng = np.random.default_rng(seed)
    ctx = rng.integers(CTX_LO, CTX_HI + 1, SEQS).astype(np.int32)
    max_seq = CTX_HI + steps_total + 16
    blocks = int(sum((int(c) + steps_total + 15) // 16 for c in ctx)) + 64
    sd = Qwen2ForCausalLM.random_state_dict(cfg, seed=seed, tied=True, device=device)
    model = Qwen2ForCausalLM(cfg, device=device).load_reference_state_dict(sd)
    if lm_head == "int8":
        model.quantize_lm_head_int8()
    kv = KVCacheManager(SEQS, max_seq, cfg.num_layers, cfg.num_key_value_heads, cfg.head_dim,
                        device=device, num_blocks=blocks)
    slots = list(range(SEQS))
    kv.plan_tokens(slots, [int(c) for c in ctx])            # reference allocation order
    g = torch.Generator(device=device)
    g.manual_seed(seed + 1)
    for li in range(cfg.num_layers):                         # N(0,1) K/V everywhere
        kv.key_cache[li].normal_(generator=g)
        kv.value_cache[li].normal_(generator=g)
    kv.advance_device(slots, ctx)
    engine = DecodeEngine(model, kv)
    first = torch.from_numpy(rng.integers(0, cfg.vocab_size, SEQS).astype(np.int32)).to(device)
    return cfg, sd, model, kv, engine, slots, ctx, first


def attention_roofline(engine, kv, cfg, ctx, reps, peak_gbs):
    """Time the paged-attention kernel alone (layer 0 of this workload) with CUDA events on its
    stream; achieved = algorithmic bytes per launch / mean launch time."""
    import torch
    from tiny_infra_b200 import _native as N
    D, NH, KVH = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    lib = N.lib()
    n = len(ctx)
    q = torch.randn(n, NH * D, device=kv.device, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    slots = torch.arange(n, dtype=torch.int32, device=kv.device)
    lens = torch.from_numpy(np.asarray(ctx, np.int32) + WINDOW // 2).to(kv.device)
    s = torch.cuda.current_stream().cuda_stream
    # as in the decode step: the batch's plan once, then the planned attention per layer
    N.check(lib.ti_paged_attention_plan(
        kv.block_tables.data_ptr(), kv.block_tables.stride(0), slots.data_ptr(), lens.data_ptr(),
        n, NH, KVH, D, kv.max_blocks_per_seq, kv.total_physical_blocks, engine.plan.data_ptr(),
        engine.plan.numel(), s))

    def launch():
        N.check(lib.ti_paged_attention_decode_planned(
            out.data_ptr(), NH * D, q.data_ptr(), NH * D, kv.key_cache[0].data_ptr(),
            kv.value_cache[0].data_ptr(), kv.total_physical_blocks, kv.block_tables.data_ptr(),
            kv.block_tables.stride(0), slots.data_ptr(), lens.data_ptr(), n, NH, KVH, D,
            kv.block_size, kv.max_blocks_per_seq, N.TI_DTYPE_BF16, engine.ws.data_ptr(),
            engine.ws.numel(), engine.plan.data_ptr(), s))

    for _ in range(5):
        launch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        launch()
    e1.record()
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / reps / 1e3
    tot = int(lens.sum().item())
    algo = tot * KVH * D * 2 * 2 + 2 * n * NH * D * 2      # K+V of every context token, q, out
    achieved = algo / t / 1e9
    return {"bound": "hbm", "kernel": "attn::decode_kernel_v5 (planned) + merge_pieces_kernel (paged decode attention)",
            "achieved": round(achieved, 1), "peak": peak_gbs, "unit": "GB/s",
            "frac": round(achieved / peak_gbs, 4), "traffic": _traffic_from_profiles(),
            "algorithmic_bytes_per_launch": algo, "us_per_launch": round(t * 1e6, 2)}


# ---------------------------------------------------------------------------------------------
def oracle_sample(sd, kv, ctx, seed):
    """The oracle (CPU restatement of the reference path) set up on CPU_SAMPLE_SEQS of the
    workload's sequences: fp32 copies of the weights and of those sequences' KV."""
    import torch
    from oracle import kernels as OK
    from oracle import model as OM
    from oracle.cache import OracleKVCache

    cfg = OM.OracleConfig()
    W = {k: v.float().cpu().numpy() for k, v in sd.items()}
    W["lm_head.weight"] = W["model.embed_tokens.weight"]
    n = CPU_SAMPLE_SEQS
    bs = 16
    need = [(int(c) + 1 + bs - 1) // bs + 1 for c in ctx[:n]]
    cache = OracleKVCache(n, int(max(ctx[:n])) + 64, cfg.num_layers, cfg.num_key_value_heads,
                          cfg.head_dim, bs, num_blocks=int(sum(need)) + 8)
    bt = kv.block_tables[:n].cpu().numpy()
    k_dev, v_dev = [], []
    nxt = 0
    for i in range(n):
        nb = (int(ctx[i]) + bs - 1) // bs
        phys = torch.from_numpy(bt[i, :nb].astype(np.int64)).to(kv.device)
        k_dev.append(kv.key_cache[:, phys])
        v_dev.append(kv.value_cache[:, phys])
        cache.block_tables[i, :nb] = np.arange(nxt, nxt + nb)
        nxt += nb
    cache.key_cache[:, :nxt] = torch.cat(k_dev, 1).float().cpu().numpy()
    cache.value_cache[:, :nxt] = torch.cat(v_dev, 1).float().cpu().numpy()
    cache.free_blocks = list(range(nxt, cache.total_physical_blocks))
    cache.seq_len[:] = ctx[:n]
    cos, sin = OK.rope_table(cache.max_seq_len, cfg.head_dim, cfg.rope_theta)
    tokens = np.random.default_rng(seed).integers(0, cfg.vocab_size, n)
    return W, cfg, cache, cos, sin, tokens


def oracle_decode_steps(state, steps, min_seconds=0.0, max_seconds=None, ctx0=None):
    """Run oracle decode steps (greedy, tokens fed back); returns (steps run, seconds).  With
    ``ctx0`` the lengths go back to it every WINDOW steps (the GPU arm's stationary contexts);
    ``max_seconds`` stops early (at least one step)."""
    from oracle import model as OM
    W, cfg, cache, cos, sin, tokens = state
    n = len(tokens)
    idx = np.arange(n)
    t0 = time.perf_counter()
    done = 0
    while done < steps or (time.perf_counter() - t0) < min_seconds:
        if ctx0 is not None and done % WINDOW == 0:
            cache.seq_len[idx] = ctx0
        logits = OM.forward(W, cfg, tokens[:, None], idx, cache, cos, sin)
        cache.seq_len[idx] += 1
        tokens = np.argmax(logits[:, -1], axis=-1)
        done += 1
        if min_seconds and done >= 2 and (time.perf_counter() - t0) >= min_seconds:
            break
        if max_seconds is not None and (time.perf_counter() - t0) >= max_seconds:
            break
    state[5][:] = tokens
    return done, time.perf_counter() - t0


def _blas_threads():
    """Threads the numpy BLAS actually runs with (threadpoolctl), else the host core count."""
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 0) for i in threadpool_info() if i.get("user_api") == "blas"]
        return int(max(n)) if n else _cores()
    except Exception:  # threadpoolctl missing or unable to inspect the library
        return _cores()


# ---------------------------------------------------------------------------------------------
def run_reference(a, rank, world):
    """CPU reference arm: the oracle restatement of the reference's PyTorch path on the host
    cores, same metric and workload (a bounded sample of it per step)."""
    if rank != 0:
        return 0
    import torch
    torch.set_num_threads(_cores())
    from oracle import model as OM
    from oracle.cache import OracleKVCache
    from oracle import kernels as OK
    cfg = OM.OracleConfig()
    W = OM.init_weights(cfg, seed=a.seed, tied=True, bf16=True)
    rng = np.random.default_rng(a.seed)
    ctx = rng.integers(CTX_LO, CTX_HI + 1, SEQS).astype(np.int32)[:CPU_SAMPLE_SEQS]
    n = CPU_SAMPLE_SEQS
    steps_total = a.warmup + a.steps
    cache = OracleKVCache(n, CTX_HI + steps_total + 16, cfg.num_layers, cfg.num_key_value_heads,
                          cfg.head_dim, 16, allocate_pool=False,
                          num_blocks=int(sum((int(c) + steps_total + 15) // 16 for c in ctx)) + 8)
    shape = (cfg.num_layers, cache.total_physical_blocks, cfg.num_key_value_heads, 16,
             cfg.head_dim)
    kr = np.random.default_rng(a.seed + 1)
    cache.key_cache = kr.standard_normal(shape, dtype=np.float32)
    cache.value_cache = kr.standard_normal(shape, dtype=np.float32)
    for i, c in enumerate(ctx):          # FIFO allocation of each context's blocks
        nb = (int(c) + 15) // 16
        for lb in range(nb):
            cache.block_tables[i, lb] = cache.free_blocks.pop(0)
    cache.seq_len[:] = ctx
    cos, sin = OK.rope_table(cache.max_seq_len, cfg.head_dim, cfg.rope_theta)
    state = [W, cfg, cache, cos, sin, rng.integers(0, cfg.vocab_size, n)]
    # warm-up bounded to 2 steps, timed steps to REF_MAX_SECONDS of work (the run has to end
    # within minutes: one oracle step of 32 sequences takes ~1 s); contexts reset every WINDOW
    # steps as in the GPU arm
    oracle_decode_steps(state, min(a.warmup, 2), ctx0=ctx)
    done, secs = oracle_decode_steps(state, a.steps, max_seconds=REF_MAX_SECONDS, ctx0=ctx)
    value = n * done / secs
    line = {"metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
            "steps": done, "warmup": min(a.warmup, 2), "ms_per_step": round(secs / done * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": _config(1, {"sample": f"{n} of the {SEQS} sequences per step"}),
            "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": _blas_threads(),
                             "kind": "port",
                             "sample": f"{n} sequences of the workload per decode step, "
                                       f"{done} steps, numpy fp32 restatement of the reference path"},
            "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_ours(a, rank, world, local):
    import torch
    import torch.distributed as dist
    from tiny_infra_b200 import _native as N
    from tiny_infra_b200 import replicas

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        # replicas: the only cross-rank steps are the barrier and the max over ranks of the
        # timed region, host-side work for gloo (no NCCL: the data path has no collective)
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    steps_total = a.warmup + a.steps
    # the engine is built for warm-up + timed + e2e steps, and at least one context window
    cfg, sd, model, kv, engine, slots, ctx, first = build_workload(
        device, a.seed + rank, max(2 * steps_total + 4, WINDOW + 4), a.lm_head)
    peak, peak_kind = _peaks()

    # ---- device-resident decode (value) ----
    # Stationary contexts: every WINDOW steps each sequence's length goes back to its sampled
    # value, so every timed step decodes at ctx0 + 0..WINDOW-1 (the configured distribution)
    # instead of drifting by the number of steps.  The block allocations of one window are
    # planned once (re-applying them is idempotent).
    ctx0_dev = kv.seq_len[:SEQS].clone()
    plan = engine.plan_steps(slots, WINDOW)
    rows = plan.shape[1]
    engine.d_in[1, :SEQS].copy_(torch.arange(SEQS, dtype=torch.int32))
    engine.d_in[0, :SEQS].copy_(first)
    sampler = ClockSampler(local)
    sampler.start()

    def resident_step(k):
        if k % WINDOW == 0:
            kv.seq_len[:SEQS].copy_(ctx0_dev)
        engine.d_in[2, :rows].copy_(plan[k % WINDOW])
        engine._replay(rows)
        engine.d_in[0, :SEQS].copy_(engine.next_tok[:SEQS])

    # warm-up (also captures the one-step graph)
    for k in range(a.warmup):
        resident_step(k)
    torch.cuda.synchronize()

    # The timed steps run as whole windows: one CUDA graph holds a window's WINDOW steps
    # (length reset, each step's new blocks, all its kernels, the token feedback), so the host
    # issues one replay per window instead of four calls per step.  Every step does the same
    # work as a one-step replay.
    def window_graph(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for k in range(n):
                if k == 0:
                    kv.seq_len[:SEQS].copy_(ctx0_dev)
                engine.d_in[2, :rows].copy_(plan[k])
                engine._launch(rows)
                engine.d_in[0, :SEQS].copy_(engine.next_tok[:SEQS])
        return g

    full, rem = divmod(a.steps, WINDOW)
    g_full = window_graph(WINDOW) if full else None
    g_rem = window_graph(rem) if rem else None
    for g in (g_full, g_rem):            # first replay uploads the graph (untimed)
        if g is not None:
            g.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(full):
        g_full.replay()
    if g_rem is not None:
        g_rem.replay()
    e1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    secs = replicas.max_over_ranks(e0.elapsed_time(e1) / 1e3)
    launches = engine.launches_per_step.get((rows, False, False), 0) * a.steps
    value = world * SEQS * a.steps / secs

    # ---- e2e through the public per-step API (host tokens in/out) ----
    # same stationary contexts: host and device lengths go back to ctx0 every WINDOW steps (the
    # allocator then hands out fresh blocks for the window's block boundary; the pool has room)
    ctx0_host = np.asarray(ctx, np.int32)
    slots_np = np.asarray(slots, np.int32)      # host ints, converted once (a list costs ~13 us)

    def e2e_step(k, toks):
        if k % WINDOW == 0:
            kv.alloc.seq_len[:SEQS] = ctx0_host
            kv.seq_len[:SEQS].copy_(ctx0_dev)
        return engine.step(slots_np, toks)

    toks = engine.next_tok[:SEQS].cpu().numpy()
    for k in range(2):
        toks = e2e_step(k, toks)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2 = [torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)]
    e2[0].record()
    for k in range(a.steps):
        toks = e2e_step(k, toks)
    e2[1].record()
    torch.cuda.synchronize()
    esecs = replicas.max_over_ranks(e2[0].elapsed_time(e2[1]) / 1e3)
    e2e = world * SEQS * a.steps / esecs

    roof = attention_roofline(engine, kv, cfg, ctx, 50, peak) if rank == 0 else None
    status = N.device_status()

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        torch.set_num_threads(_cores())
        st = list(oracle_sample(sd, kv, ctx, a.seed))
        oracle_decode_steps(st, 1, ctx0=ctx[:CPU_SAMPLE_SEQS])
        done, csecs = oracle_decode_steps(st, 2, min_seconds=10.0, ctx0=ctx[:CPU_SAMPLE_SEQS])
        cpu = {"value": round(CPU_SAMPLE_SEQS * done / csecs, 2), "unit": "tokens/s",
               "cores": _blas_threads(), "kind": "port",
               "sample": f"{CPU_SAMPLE_SEQS} of the {SEQS} sequences, {done} greedy decode steps, "
                         "numpy fp32 restatement of the reference path (oracle/)"}
    if world > 1:
        dist.barrier()
    engine.graphs.clear()
    del g_full, g_rem
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return 0
    kv_bytes = int(ctx.sum() + SEQS * (WINDOW + 1) / 2) * cfg.num_layers * 2 * 2 * 64 * 2
    step_bytes = model.weight_bytes() + kv_bytes
    ms = secs / a.steps * 1e3
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights, random token ids, N(0,1) KV)",
        "config": _config(world, {"global_batch": SEQS * world,
                                  **({"lm_head": "weight-only int8 (per-row scales), greedy"}
                                     if a.lm_head == "int8" else {})}),
        "e2e": {"value": round(e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": 3 * SEQS * 4,
                "d2h_bytes_per_step": SEQS * 4,
                "api": "tiny_infra_b200.engine.DecodeEngine.step (host lists in/out)"},
        "roofline": roof,
        "step_roofline": {"bytes_per_step": step_bytes,
                          "achieved_gbs": round(step_bytes / (secs / a.steps) / 1e9, 1),
                          "peak_gbs": peak, "frac": round(step_bytes / (secs / a.steps) / 1e9 / peak, 4),
                          "peak_kind": peak_kind},
        "cpu_baseline": cpu, "clocks": clocks, "gpu_launches": int(launches),
        "device_status": status,
    }
    print(json.dumps(line), flush=True)
    return _status_rc(status)


def _status_rc(status: int) -> int:
    """Exit code of a measured run: a kernel that raised a device status bit skipped work, so
    its line is not a measurement."""
    if status:
        print(f"bench: device status 0x{status:x} raised during the run: the line above is "
              "not a valid measurement", file=sys.stderr, flush=True)
        return 1
    return 0


def _kernel_line_flops(a, metric_value, t, flops, workload, data, extra_cfg=None):
    """JSON line of a tensor-bound kernel mode: TFLOP/s of its algorithmic FLOPs against the
    measured bf16 GEMM peak (burst: the kernel is timed alone)."""
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    peak, kind = (float(json.load(open(p))["bf16_tflops"]), "measured") if os.path.exists(p) \
        else (1590.0, "fallback")
    tfs = flops / t / 1e12
    cfg = {"workload": workload, "l2": "weights cycled over buffers larger than L2, no flush"}
    cfg.update(extra_cfg or {})
    print(json.dumps({
        "metric": metric_value, "value": round(tfs, 1), "unit": "TFLOP/s",
        "n_gpus": 1, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(t * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": data, "config": cfg,
        "roofline": {"bound": "tensor", "achieved": round(tfs, 1), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(tfs / peak, 4), "peak_kind": kind,
                     "algorithmic_flops_per_launch": int(flops)}}), flush=True)


def _kernel_line(a, metric_value, t, algo, workload, data, extra_cfg=None):
    peak, kind = _peaks()
    gbs = algo / t / 1e9
    cfg = {"workload": workload, "l2": "inputs larger than L2 (distinct buffers per launch), no flush"}
    cfg.update(extra_cfg or {})
    print(json.dumps({
        "metric": metric_value, "value": round(gbs, 1), "unit": "GB/s",
        "n_gpus": 1, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(t * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": data, "config": cfg,
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs / peak, 4), "peak_kind": kind,
                     "algorithmic_bytes_per_launch": int(algo)}}), flush=True)


def _time_launches(fn, n_buffers, steps, warmup):
    """Average device time of `steps` back-to-back launches cycling over n_buffers inputs.
    The launches are captured in one CUDA graph and replayed (as the decode step runs them),
    so the host's per-call cost (ctypes, argument checks) stays out of the device timeline;
    events on the replay stream bracket the timed replay, after one untimed replay."""
    import torch
    for i in range(max(warmup, n_buffers)):
        fn(i % n_buffers)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(steps):
            fn(i % n_buffers)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    del graph
    return e0.elapsed_time(e1) / 1e3 / steps


def run_attention_kernel(a):
    """Paged decode attention alone: the 256-sequence workload (ctx U[128,2048]) or the
    8-sequence op of ctx U[1,512] over a 512-block pool; HBM GB/s of one layer's launch (the
    attention kernel and its split-K merge), cycling over 8 layers' pools."""
    import torch
    from tiny_infra_b200 import custom_paged_attn
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(a.seed)
    B, lo, hi, NB = {"256": (SEQS, CTX_LO, CTX_HI, None), "config1": (8, 1, 512, 512),
                     "long": (SEQS, 8192, 32768, None)}[a.case]
    NH, KVH, D, bs = 14, 2, 64, 16
    ctx = rng.integers(lo, hi + 1, B).astype(np.int32)
    need = int(sum((int(c) + bs - 1) // bs for c in ctx))
    NB = NB or need + 64
    mb = (hi + bs - 1) // bs
    perm = rng.permutation(NB)
    bt = np.full((B, mb), -1, np.int32)
    off = 0
    for b in range(B):
        n = (int(ctx[b]) + bs - 1) // bs
        bt[b, :n] = perm[off:off + n]
        off += n
    layers = {"256": 8, "config1": 64, "long": 2}[a.case]   # > 126 MB of KV in every case
    g = torch.Generator(device=dev)
    g.manual_seed(a.seed)
    q = torch.randn(B, NH, D, device=dev, generator=g).to(torch.bfloat16)
    ks = [torch.randn(NB, KVH, bs, D, device=dev, generator=g).to(torch.bfloat16)
          for _ in range(layers)]
    vs = [torch.randn(NB, KVH, bs, D, device=dev, generator=g).to(torch.bfloat16)
          for _ in range(layers)]
    out = torch.empty_like(q)
    btt, ct = torch.from_numpy(bt).to(dev), torch.from_numpy(ctx).to(dev)
    t = _time_launches(lambda i: custom_paged_attn.launch_paged_attention(
        out, q, ks[i], vs[i], btt, ct, bs), layers, a.steps, a.warmup)
    algo = int(ctx.sum()) * KVH * D * 2 * 2 + 2 * B * NH * D * 2
    _kernel_line(a, "paged-attn HBM GB/s", t, algo,
                 f"paged decode attention, {B} seqs, ctx U[{lo},{hi}], 14/2 heads, D=64, "
                 f"pool {NB} blocks x 16, {layers} layers cycled",
                 "synthetic (N(0,1) q/k/v, random block permutation)")
    return 0


def run_gate_up_kernel(a):
    """The decode step's gate/up projection alone (256 tokens x 896 -> 2 x 4864, SwiGLU fused),
    cycling over 24 layers' weights; GB/s of its algorithmic bytes (weights + activations in,
    SwiGLU output)."""
    import torch
    from tiny_infra_b200 import _native as N
    dev = torch.device("cuda:0")
    M, H, I, L = SEQS, 896, 4864, 24
    g = torch.Generator(device=dev)
    g.manual_seed(a.seed)
    x = torch.randn(M, H, device=dev, generator=g).to(torch.bfloat16)
    ws = [(torch.randn(2 * I, H, device=dev, generator=g) * 0.02).to(torch.bfloat16)
          for _ in range(L)]
    act = torch.empty(M, I, device=dev, dtype=torch.bfloat16)
    lib = N.lib()

    def launch(i):
        N.check(lib.ti_gemm(N.TI_EPI_SWIGLU16, x.data_ptr(), H, ws[i].data_ptr(), H, M, 2 * I, H,
                            act.data_ptr(), I, None, None, None, N.TI_DTYPE_BF16, 0, 1,
                            torch.cuda.current_stream().cuda_stream))
    t = _time_launches(launch, L, a.steps, a.warmup)
    algo = 2 * I * H * 2 + M * H * 2 + M * I * 2
    _kernel_line(a, "gate_up GEMM HBM GB/s", t, algo,
                 f"gate/up projection + SwiGLU (rows interleaved in groups of 8, 144-wide "
                 f"tiles), M={M}, N={2 * I}, K={H}, {L} layers' weights cycled", "synthetic (N(0,1) activations, N(0,0.02) weights)")
    return 0


def run_lm_head_kernel(a, int8):
    """The greedy lm_head alone at 256 decode rows: 151936 x 896 weights (bf16, or the int8 copy
    with per-row scales) times the final normed hidden rows, per-tile argmax in the epilogue;
    two weight copies cycled (2 x 272 MB or 2 x 136 MB > L2).  GB/s of the weight bytes (+ the
    activations and the argmax partials)."""
    import torch
    from tiny_infra_b200 import _native as N
    dev = torch.device("cuda:0")
    M, H, V, L = SEQS, 896, 151936, 2
    g = torch.Generator(device=dev)
    g.manual_seed(a.seed)
    x = torch.randn(M, H, device=dev, generator=g).to(torch.bfloat16)
    ws = [(torch.randn(V, H, device=dev, generator=g) * 0.02).to(torch.bfloat16) for _ in range(L)]
    nt = V // 128
    val = torch.empty(M, nt, device=dev, dtype=torch.float32)
    idx = torch.empty(M, nt, device=dev, dtype=torch.int32)
    lib = N.lib()
    st = lambda: torch.cuda.current_stream().cuda_stream  # noqa: E731
    if int8:
        qs, ss = [], []
        for w in ws:
            q = torch.empty(V, H, dtype=torch.int8, device=dev)
            sc = torch.empty(V, dtype=torch.float32, device=dev)
            N.check(lib.ti_quantize_rows_int8(w.data_ptr(), H, V, H, q.data_ptr(), H,
                                              sc.data_ptr(), N.TI_DTYPE_BF16, st()))
            qs.append(q)
            ss.append(sc)
        del ws

        def launch(i):
            N.check(lib.ti_lm_head_argmax_int8(x.data_ptr(), H, qs[i].data_ptr(), H,
                                               ss[i].data_ptr(), M, V, H, val.data_ptr(),
                                               idx.data_ptr(), N.TI_DTYPE_BF16, st()))
        wbytes = V * H + V * 4
    else:
        def launch(i):
            N.check(lib.ti_gemm(N.TI_EPI_ARGMAX, x.data_ptr(), H, ws[i].data_ptr(), H, M, V, H,
                                None, 0, None, val.data_ptr(), idx.data_ptr(), N.TI_DTYPE_BF16,
                                128, 1, st()))
        wbytes = V * H * 2
    t = _time_launches(launch, L, a.steps, a.warmup)
    algo = wbytes + M * H * 2 + M * nt * 8
    kind = "weight-only int8 (per-row scales)" if int8 else "bf16"
    _kernel_line(a, f"lm_head ({kind}) HBM GB/s", t, algo,
                 f"greedy lm_head, {M} rows x {H} -> {V} vocab, {kind} weights, per-tile argmax "
                 f"epilogue, {L} weight copies cycled",
                 "synthetic (N(0,1) hidden rows, N(0,0.02) weights)")
    return 0


def run_projection_kernel(a):
    """One decode-step projection alone at 256 tokens, weight copies cycled (> L2): qkv
    (896 -> 1152 with bias, RoPE and the KV-append write into a paged pool), o_proj (896 -> 896)
    or down (4864 -> 896), both adding into the float32 residual stream (split-K red.add, as in
    the decode step).  GB/s of the algorithmic bytes: weights, activations in, output."""
    import torch
    from tiny_infra_b200 import _native as N
    dev = torch.device("cuda:0")
    M, H, I, NH, KVH, D = SEQS, 896, 4864, 14, 2, 64
    g = torch.Generator(device=dev)
    g.manual_seed(a.seed)
    lib = N.lib()
    st = lambda: torch.cuda.current_stream().cuda_stream  # noqa: E731
    K, Nout = {"qkv": (H, (NH + 2 * KVH) * D), "o_proj": (NH * D, H), "down": (I, H)}[a.kernel]
    L = -(-320 * 2 ** 20 // (Nout * K * 2))      # weight copies: > 2.5 x L2 in every cycle
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    ws = [(torch.randn(Nout, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
          for _ in range(L)]
    if a.kernel == "qkv":
        bias = (torch.randn(Nout, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        nb = M + 16
        kc = torch.zeros(nb, KVH, 16, D, device=dev, dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        slot = torch.arange(M, device=dev, dtype=torch.int64) * 16     # one block per token
        pos = torch.randint(0, 2048, (M,), device=dev, dtype=torch.int32, generator=g)
        inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, device=dev).float() / D))
        fr = torch.outer(torch.arange(4096, device=dev, dtype=torch.float32), inv)
        cos, sin = fr.cos().contiguous(), fr.sin().contiguous()
        q = torch.empty(M, NH * D, device=dev, dtype=torch.bfloat16)

        def launch(i):
            N.check(lib.ti_gemm_qkv_rope(x.data_ptr(), K, ws[i].data_ptr(), K, bias.data_ptr(), M,
                                         H, NH, KVH, D, q.data_ptr(), NH * D, kc.data_ptr(),
                                         vc.data_ptr(), slot.data_ptr(), cos.data_ptr(),
                                         sin.data_ptr(), pos.data_ptr(), 16, N.TI_DTYPE_BF16,
                                         st()))
        out_bytes = M * Nout * 2
        what = "QKV projection + bias + RoPE + KV append (cluster split-K)"
    else:
        hidden = torch.zeros(M, Nout, device=dev, dtype=torch.float32)
        bn, split = (64, 7) if a.kernel == "o_proj" else (128, 16)

        def launch(i):
            N.check(lib.ti_gemm(N.TI_EPI_RESIDUAL, x.data_ptr(), K, ws[i].data_ptr(), K, M, Nout,
                                K, hidden.data_ptr(), Nout, None, None, None, N.TI_DTYPE_BF16,
                                bn, split, st()))
        out_bytes = M * Nout * 4 * 2                  # residual read-modify-write (float32)
        what = f"{a.kernel} projection + residual add (block_n {bn}, split-K red.add)"
    t = _time_launches(launch, L, max(a.steps, L), a.warmup)
    algo = Nout * K * 2 + M * K * 2 + out_bytes
    _kernel_line(a, f"{a.kernel} GEMM HBM GB/s", t, algo,
                 f"{what}, M={M}, N={Nout}, K={K}, {L} weight copies cycled (> L2), "
                 f"{max(a.steps, L)} launches timed",
                 "synthetic (N(0,1) activations, N(0,0.02) weights)")
    return 0


def run_rmsnorm_kernel(a):
    """RMSNorm of the fused-elementwise workload: 4096 tokens x hidden 896 (``--rows``: 256 for
    one decode step's batch), float32 residual stream in, bf16 out, eps 1e-6, cycling over
    enough inputs to exceed L2 (>= 147 MB); GB/s of its algorithmic bytes (x read once, out
    written once, the weight)."""
    import torch
    from tiny_infra_b200 import _native as N
    dev = torch.device("cuda:0")
    T, H = a.rows, 896
    L = max(12, -(-160 * 2 ** 20 // (T * H * 4)))
    g = torch.Generator(device=dev)
    g.manual_seed(a.seed)
    xs = [torch.randn(T, H, device=dev, generator=g) for _ in range(L)]
    w = torch.randn(H, device=dev, generator=g).to(torch.bfloat16)
    outs = [torch.empty(T, H, device=dev, dtype=torch.bfloat16) for _ in range(L)]
    lib = N.lib()

    def launch(i):
        N.check(lib.ti_rmsnorm(outs[i].data_ptr(), xs[i].data_ptr(), N.TI_DTYPE_FP32, w.data_ptr(),
                               1e-6, T, H, N.TI_DTYPE_BF16, torch.cuda.current_stream().cuda_stream))
    t = _time_launches(launch, L, a.steps, a.warmup)
    _kernel_line(a, "rmsnorm HBM GB/s", t, T * H * 4 + T * H * 2 + H * 2,
                 f"RMSNorm, {T} tokens x {H}, fp32 in / bf16 out, {L} inputs cycled",
                 "synthetic (N(0,1) residual stream and weight)")
    return 0


def run_sampler_kernel(a):
    """Device sampler on one decode step's logits: 256 rows x 151936 (bf16), temperature 0.7,
    top-k 50, top-p 0.9 (the serving configuration's sampling), two logits buffers cycled
    (156 MB > L2); GB/s of one read of the logits."""
    import torch
    from tiny_infra_b200 import sampler as S
    dev = torch.device("cuda:0")
    R, V, L = 256, 151936, 2
    g = torch.Generator(device=dev)
    g.manual_seed(a.seed)
    logits = [(torch.randn(R, V, device=dev, generator=g) * 3.0).to(torch.bfloat16)
              for _ in range(L)]
    rng = np.random.default_rng(a.seed)
    sp = S.SamplingParams([0.7] * R, [50] * R, [0.9] * R, rng.random(R).tolist(), V)
    pd = torch.from_numpy(sp.packed()).to(dev)
    out = torch.empty(R, dtype=torch.int32, device=dev)
    t = _time_launches(lambda i: S.launch_sample(logits[i], pd, out), L, a.steps, a.warmup)
    _kernel_line(a, "sampler HBM GB/s", t, R * V * 2 + R * 16 + R * 4,
                 f"temperature / top-k / top-p sampling, {R} rows x {V} bf16 logits, "
                 f"T 0.7, k 50, p 0.9, {L} logits buffers cycled",
                 "synthetic (N(0,3) logits, seeded uniforms)")
    return 0


def run_prefill_gemm_kernel(a):
    """gate/up + SwiGLU at prefill size: 4096 tokens x 896 -> 2 x 4864 (71.4 GFLOP, the packed
    token count of the fused-elementwise workload), 24 layers' weights cycled; TFLOP/s on the
    tcgen05 tensor pipe against the measured bf16 GEMM peak."""
    import torch
    from tiny_infra_b200 import _native as N
    dev = torch.device("cuda:0")
    M, H, I, L = 4096, 896, 4864, 24
    g = torch.Generator(device=dev)
    g.manual_seed(a.seed)
    x = torch.randn(M, H, device=dev, generator=g).to(torch.bfloat16)
    ws = [(torch.randn(2 * I, H, device=dev, generator=g) * 0.02).to(torch.bfloat16)
          for _ in range(L)]
    act = torch.empty(M, I, device=dev, dtype=torch.bfloat16)
    lib = N.lib()

    def launch(i):
        N.check(lib.ti_gemm(N.TI_EPI_SWIGLU16, x.data_ptr(), H, ws[i].data_ptr(), H, M, 2 * I, H,
                            act.data_ptr(), I, None, None, None, N.TI_DTYPE_BF16, 0, 1,
                            torch.cuda.current_stream().cuda_stream))
    t = _time_launches(launch, L, a.steps, a.warmup)
    _kernel_line_flops(a, "prefill gate_up GEMM TFLOP/s", t, 2.0 * M * 2 * I * H,
                       f"gate/up projection + SwiGLU (rows interleaved in groups of 8, 256-wide "
                       f"tiles), M={M}, N={2 * I}, K={H}, {L} layers' weights cycled",
                       "synthetic (N(0,1) activations, N(0,0.02) weights)")
    return 0


def run_prefill_attention_kernel(a):
    """Ragged causal prefill attention over the paged pool, the fused-elementwise packing: 4096
    new tokens in 16 sequences of seeded lengths, each chunk at a seeded start position so that
    its tokens lie in [0, 32768), attending to every earlier position of its sequence; 14/2
    heads, D 64, bf16, one layer (its KV > L2).  TFLOP/s of the causal QK^T and PV products."""
    import torch
    from tiny_infra_b200 import _native as N
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(a.seed)
    S_, T, NH, KVH, D, bs = 16, 4096, 14, 2, 64, 16
    cut = np.sort(rng.choice(np.arange(1, T), S_ - 1, replace=False))
    lens = np.diff(np.concatenate([[0], cut, [T]])).astype(np.int32)
    start = np.array([rng.integers(0, 32768 - n + 1) for n in lens], np.int32)
    nblk = (start + lens + bs - 1) // bs
    NB = int(nblk.sum()) + 16
    mb = int(nblk.max())
    perm = rng.permutation(NB)
    bt = np.full((S_, mb), -1, np.int32)
    off = 0
    for i in range(S_):
        bt[i, :nblk[i]] = perm[off:off + nblk[i]]
        off += int(nblk[i])
    cu = np.zeros(S_ + 1, np.int32)
    cu[1:] = np.cumsum(lens)
    ts, tq, work = [], [], []
    for i in range(S_):
        for q0 in range(0, int(lens[i]), 16):
            ts.append(i)
            tq.append(q0)
            work.append(int(start[i]) + min(q0 + 16, int(lens[i])))
    order = np.argsort(-np.asarray(work, np.int64), kind="stable")   # as the model orders them
    ts, tq = [ts[o] for o in order], [tq[o] for o in order]
    g = torch.Generator(device=dev)
    g.manual_seed(a.seed)
    q = torch.randn(T, NH, D, device=dev, generator=g).to(torch.bfloat16)
    kc = torch.randn(NB, KVH, bs, D, device=dev, generator=g).to(torch.bfloat16)
    vc = torch.randn(NB, KVH, bs, D, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty_like(q)
    as_dev = lambda x: torch.from_numpy(np.ascontiguousarray(x, np.int32)).to(dev)  # noqa: E731
    d_bt, d_start, d_cu = as_dev(bt), as_dev(start), as_dev(cu)
    d_ts, d_tq, d_rows = as_dev(ts), as_dev(tq), as_dev(np.arange(S_))
    lib = N.lib()

    def launch(_):
        N.check(lib.ti_paged_prefill_attention(
            out.data_ptr(), NH * D, q.data_ptr(), NH * D, kc.data_ptr(), vc.data_ptr(), NB,
            d_bt.data_ptr(), d_bt.stride(0), d_rows.data_ptr(), d_start.data_ptr(), d_cu.data_ptr(),
            d_ts.data_ptr(), d_tq.data_ptr(), len(ts), NH, KVH, D, bs, N.TI_DTYPE_BF16,
            torch.cuda.current_stream().cuda_stream))
    t = _time_launches(launch, 1, a.steps, a.warmup)
    keys = sum(int(s0) * int(n) + int(n) * (int(n) + 1) // 2 for s0, n in zip(start, lens))
    flops = 4.0 * keys * D * NH                     # QK^T and PV, 2 FLOP per MAC
    _kernel_line_flops(a, "prefill attention TFLOP/s", t, flops,
                       f"ragged causal prefill attention, {T} tokens in {S_} sequences, starts "
                       f"in [0, 32768), 14/2 heads, D=64, paged pool of {NB} blocks",
                       "synthetic (N(0,1) q/k/v, random block permutation)",
                       {"kv_bytes_unique": int(nblk.sum()) * KVH * bs * D * 2 * 2,
                        "l2": "one layer's pool; its unique KV fits L2 after the first touch "
                              "(compute-bound kernel), no flush"})
    return 0


def run_serving(a):
    """A stream of generation requests through ContinuousBatcher (one GPU): Poisson arrivals
    (--rate per second, seeded), prompt ids U[0, 151936), prompt lengths U[32, 1024], output
    lengths U[16, 512], temperature 0.7 / top-k 50 / top-p 0.9, 256 slots, prefill chunked to
    2048 tokens per tick.  Reports output tokens per second over the whole run (first arrival
    to last completion) and latency statistics."""
    import asyncio
    import time

    import torch
    from tiny_infra_b200.cache_manager import KVCacheManager
    from tiny_infra_b200.config import QwenConfig
    from tiny_infra_b200.qwen2 import Qwen2ForCausalLM
    from tiny_infra_b200.scheduler import ContinuousBatcher

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    cfg = QwenConfig()
    sd = Qwen2ForCausalLM.random_state_dict(cfg, seed=a.seed, tied=True)
    model = Qwen2ForCausalLM(cfg).load_reference_state_dict(sd)
    kv = KVCacheManager(SEQS, 1024 + 512 + 16, cfg.num_layers, cfg.num_key_value_heads,
                        cfg.head_dim, device=dev)
    sched = ContinuousBatcher(model, kv, eos_token_id=None, prefill_chunk_tokens=2048)
    rng = np.random.default_rng(a.seed)
    n = a.requests
    gaps = rng.exponential(1.0 / a.rate, n)
    arrive = np.cumsum(gaps) - gaps[0]
    plen = rng.integers(32, 1025, n)
    olen = rng.integers(16, 513, n)
    prompts = [rng.integers(0, cfg.vocab_size, int(k)).tolist() for k in plen]

    async def warm():
        loop = asyncio.create_task(sched.run_loop())
        await asyncio.gather(*[sched.generate(prompts[i][:64], 4) for i in range(4)])
        loop.cancel()

    asyncio.run(warm())                   # graphs and kernels set up outside the measurement
    ttft, done_at, ntok = [None] * n, [None] * n, [0] * n

    async def one(i, t0):
        await asyncio.sleep(max(0.0, t0 + arrive[i] - time.perf_counter()))
        start = time.perf_counter()
        async for _ in sched.generate_stream(prompts[i], int(olen[i]), temperature=0.7,
                                             p_value=0.9, top_k=50):
            if ntok[i] == 0:
                ttft[i] = time.perf_counter() - start
            ntok[i] += 1
        done_at[i] = time.perf_counter() - start

    async def main():
        loop = asyncio.create_task(sched.run_loop())
        t0 = time.perf_counter()
        await asyncio.gather(*[one(i, t0) for i in range(n)])
        secs = time.perf_counter() - t0
        loop.cancel()
        return secs

    secs = asyncio.run(main())
    torch.cuda.synchronize()
    total = int(sum(ntok))
    lat = np.array(done_at)
    tt = np.array(ttft)
    per_tok = (lat - tt) / np.maximum(np.array(ntok) - 1, 1)
    print(json.dumps({
        "metric": "serving output tokens/s (Poisson stream, continuous batching)",
        "value": round(total / secs, 1), "unit": "tokens/s", "n_gpus": 1,
        "higher_is_better": True, "dtype": "bf16", "vs_baseline": None,
        "data": "synthetic (random-init weights, random prompt ids, seeded arrivals and lengths)",
        "config": {"workload": f"{n} requests, Poisson {a.rate}/s, prompt U[32,1024], output "
                               "U[16,512], temp 0.7 / top-k 50 / top-p 0.9, 256 slots, "
                               "prefill chunks of 2048 tokens",
                   "wall_s": round(secs, 2), "output_tokens": total,
                   "arrival_span_s": round(float(arrive[-1]), 2)},
        "latency": {"ttft_ms_p50": round(float(np.median(tt)) * 1e3, 1),
                    "ttft_ms_p90": round(float(np.percentile(tt, 90)) * 1e3, 1),
                    "per_token_ms_p50": round(float(np.median(per_tok)) * 1e3, 2),
                    "per_token_ms_p90": round(float(np.percentile(per_tok, 90)) * 1e3, 2)}}),
          flush=True)
    return 0


def run_long(a, rank, world, local):
    """Long-context decode across replicas: 2048 requests (--requests) partitioned round robin
    over the N ranks, contexts U[8192, 32768] (KV pre-filled N(0,1)), 128 greedy output tokens
    each, 256 slots per replica; each replica decodes its share in batches of up to 256
    requests.  value = all ranks' generated tokens / the max over ranks of the device time of
    the decode steps (weak scaling: the request count is fixed, so per-GPU work shrinks as N
    grows -- "scaling": "strong")."""
    import torch
    import torch.distributed as dist
    from tiny_infra_b200 import _native as N
    from tiny_infra_b200 import replicas
    from tiny_infra_b200.cache_manager import KVCacheManager
    from tiny_infra_b200.config import QwenConfig
    from tiny_infra_b200.engine import DecodeEngine
    from tiny_infra_b200.qwen2 import Qwen2ForCausalLM

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=900))
    LO, HI, OUT, SLOTS = 8192, 32768, 128, 256
    total_req = a.requests if a.requests != 1024 else 2048
    rng = np.random.default_rng(a.seed)
    ctx_all = rng.integers(LO, HI + 1, total_req).astype(np.int32)
    mine = replicas.partition(total_req, world, rank)
    ctx_mine = ctx_all[mine]
    cfg = QwenConfig()
    sd = Qwen2ForCausalLM.random_state_dict(cfg, seed=a.seed, tied=True, device=device)
    model = Qwen2ForCausalLM(cfg, device=device).load_reference_state_dict(sd)
    max_seq = HI + OUT + 16
    blocks = SLOTS * ((max_seq + 15) // 16)          # every slot at the longest context
    kv = KVCacheManager(SLOTS, max_seq, cfg.num_layers, cfg.num_key_value_heads, cfg.head_dim,
                        device=device, num_blocks=blocks)
    g = torch.Generator(device=device)
    g.manual_seed(a.seed + 1 + rank)
    for li in range(cfg.num_layers):
        kv.key_cache[li].normal_(generator=g)
        kv.value_cache[li].normal_(generator=g)
    engine = DecodeEngine(model, kv)

    def load_batch(ctx):
        n = len(ctx)
        slots = list(range(n))
        for sl in range(SLOTS):
            if kv.seq_len_host(sl) or kv.alloc.block_tables[sl, 0] >= 0:
                kv.free_batch_slot(sl)
        kv.plan_tokens(slots, [int(c) for c in ctx])
        kv.advance_device(slots, [int(c) for c in ctx])
        plan = engine.plan_steps(slots, OUT)
        first = torch.from_numpy(rng.integers(0, cfg.vocab_size, n).astype(np.int32)).to(device)
        return slots, plan, first

    def run_batch(slots, plan, first, steps):
        n = len(slots)
        rows = plan.shape[1]
        engine.d_in[1, :n].copy_(torch.arange(n, dtype=torch.int32))
        engine.d_in[1, n:rows] = -1
        engine.d_in[0, :n].copy_(first)
        for k in range(steps):
            engine.d_in[2, :rows].copy_(plan[k])
            engine._replay(rows)
            engine.d_in[0, :n].copy_(engine.next_tok[:n])

    # warm-up (graph capture) on the first batch, then every batch timed from its start
    sl, pl, fi = load_batch(ctx_mine[:SLOTS])
    run_batch(sl, pl, fi, max(1, a.warmup))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local)
    sampler.start()
    secs, tokens, kv_tok = 0.0, 0, 0
    for b0 in range(0, len(ctx_mine), SLOTS):
        ctx = ctx_mine[b0:b0 + SLOTS]
        sl, pl, fi = load_batch(ctx)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        run_batch(sl, pl, fi, OUT)
        e1.record()
        torch.cuda.synchronize()
        secs += e0.elapsed_time(e1) / 1e3
        tokens += len(ctx) * OUT
        kv_tok += int(ctx.sum()) * OUT + len(ctx) * OUT * (OUT + 1) // 2
    clocks = sampler.stop()
    status = N.device_status()
    tsecs = replicas.max_over_ranks(secs)
    all_tokens = total_req * OUT
    steps = -(-len(ctx_mine) // SLOTS) * OUT
    if world > 1:
        dist.barrier()
    engine.graphs.clear()
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return 0
    peak, peak_kind = _peaks()
    step_bytes = model.weight_bytes() + kv_tok / steps * cfg.num_layers * 2 * 2 * 64 * 2
    print(json.dumps({
        "metric": "long-context decode tokens/s (2048 requests, ctx U[8192,32768], 128 tokens)",
        "value": round(all_tokens / tsecs, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": max(1, a.warmup), "ms_per_step": round(tsecs / steps * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights, random token ids, N(0,1) KV)",
        "config": {"workload": f"{total_req} requests round robin over {world} replica(s), ctx "
                               f"U[{LO},{HI}], {OUT} greedy tokens, {SLOTS} slots per replica, "
                               "KV pre-filled (no prefill)",
                   "parallelism": f"replicas x{world} (no collectives)",
                   "l2": "inputs far larger than L2 (~65 GB of KV per step), no flush"},
        "step_roofline": {"bytes_per_step": int(step_bytes),
                          "achieved_gbs": round(step_bytes / (tsecs / steps) / 1e9, 1),
                          "peak_gbs": peak, "peak_kind": peak_kind,
                          "frac": round(step_bytes / (tsecs / steps) / 1e9 / peak, 4)},
        "clocks": clocks, "device_status": status}), flush=True)
    return _status_rc(status)


def main():
    global SEQS, METRIC
    a = _args()
    rank, world, local = _dist()
    if a.seqs != SEQS:
        SEQS = a.seqs
        METRIC = f"decode tokens/sec @{SEQS} ragged seqs per B200; paged-attn HBM GB/s"
    if a.workload == "serving":
        return run_serving(a) if rank == 0 else 0
    if a.workload == "long":
        return run_long(a, rank, world, local)
    if a.kernel == "attention":
        return run_attention_kernel(a) if rank == 0 else 0
    if a.kernel == "rmsnorm":
        return run_rmsnorm_kernel(a) if rank == 0 else 0
    if a.kernel in ("qkv", "o_proj", "down"):
        return run_projection_kernel(a) if rank == 0 else 0
    if a.kernel in ("lm_head", "lm_head_int8"):
        return run_lm_head_kernel(a, a.kernel == "lm_head_int8") if rank == 0 else 0
    if a.kernel == "sampler":
        return run_sampler_kernel(a) if rank == 0 else 0
    if a.kernel == "prefill_gemm":
        return run_prefill_gemm_kernel(a) if rank == 0 else 0
    if a.kernel == "prefill_attention":
        return run_prefill_attention_kernel(a) if rank == 0 else 0
    if a.kernel == "gate_up":
        return run_gate_up_kernel(a) if rank == 0 else 0
    if a.impl == "reference":
        return run_reference(a, rank, world)
    return run_ours(a, rank, world, local)


if __name__ == "__main__":
    sys.exit(main())
