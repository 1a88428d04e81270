"""Record the outputs of the reference project's own CUDA kernels on seeded inputs.

Runs on a machine with a B200, with the reference kernels prebuilt from the reference sources by
``oracle/build_ref.py`` (into ``oracle/_ref``):

    python tests/golden/make_kernel_golden.py --out tests/golden/kernel_golden.npz

Inputs are regenerated from the seeds in :func:`inputs` (numpy PCG64, stable across
versions), so the fixture stores only the reference kernels' fp16 outputs.  The CPU test
``tests/test_oracle_golden.py::test_reference_kernels`` checks the oracle against them.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))


def attention_inputs(seed: int, B: int, NH: int, KVH: int, D: int, NB: int, ctx_hi: int,
                     special: bool):
    """Paged-attention inputs with each sequence's block table a slice of one random
    permutation of the pool (distinct blocks), fp16-representable values."""
    bs = 16
    rng = np.random.default_rng(seed)
    ctx = rng.integers(1, ctx_hi + 1, B).astype(np.int32)
    max_blocks = (ctx_hi + bs - 1) // bs
    perm = rng.permutation(NB)
    bt = np.full((B, max_blocks), -1, np.int32)
    off = 0
    for b in range(B):
        n = (int(ctx[b]) + bs - 1) // bs
        bt[b, :n] = perm[off:off + n]
        off += n
    if special:
        ctx[0] = 0                      # untouched row
        bt[1, 1:] = -1                  # context truncated at the first -1
        ctx[1] = max(ctx[1], 40)
    q = rng.standard_normal((B, NH, D)).astype(np.float16)
    k = rng.standard_normal((NB, KVH, bs, D)).astype(np.float16)
    v = rng.standard_normal((NB, KVH, bs, D)).astype(np.float16)
    return q, k, v, bt, ctx


def inputs():
    rng = np.random.default_rng(2024)
    attn64 = attention_inputs(101, 8, 14, 2, 64, 512, 512, special=False)
    attn128 = attention_inputs(102, 6, 8, 2, 128, 64, 96, special=True)
    T, NH, KVH, D = 64, 14, 2, 64
    rq = rng.standard_normal((T, NH, D)).astype(np.float16)
    rk = rng.standard_normal((T, KVH, D)).astype(np.float16)
    pos = rng.integers(0, 4096, T).astype(np.int32)
    sw = (rng.standard_normal((64, 512)) * 2.0).astype(np.float16)
    return {"attn64": attn64, "attn128": attn128, "rope": (rq, rk, pos), "swiglu": sw}


def main() -> None:
    import torch
    from oracle import kernels as OK
    from oracle.build_ref import load_ref

    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default="tests/golden/kernel_golden.npz")
    a = ap.parse_args()
    dev = torch.device("cuda:0")
    pa, rp, sw = (load_ref("custom_paged_attn"), load_ref("custom_rope"),
                  load_ref("custom_swiglu"))
    x = inputs()
    out = {}
    for name in ("attn64", "attn128"):
        q, k, v, bt, ctx = x[name]
        qt = torch.from_numpy(q).to(dev)
        o = torch.full_like(qt, 7.0)    # ctx == 0 rows must stay 7
        pa.launch_paged_attention(o, qt, torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev),
                                  torch.from_numpy(bt).to(dev), torch.from_numpy(ctx).to(dev), 16)
        torch.cuda.synchronize()
        out[f"{name}_out"] = o.cpu().numpy()
    rq, rk, pos = x["rope"]
    cos, sin = OK.rope_table(4096, 64, 1e6)
    qt, kt = torch.from_numpy(rq).to(dev), torch.from_numpy(rk).to(dev)
    rp.apply_inplace(qt, kt, torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev),
                     torch.from_numpy(pos).to(dev))
    torch.cuda.synchronize()
    out["rope_q"], out["rope_k"] = qt.cpu().numpy(), kt.cpu().numpy()
    out["swiglu_out"] = sw.forward(torch.from_numpy(x["swiglu"]).to(dev)).cpu().numpy()
    os.makedirs(os.path.dirname(os.path.abspath(a.out)), exist_ok=True)
    np.savez_compressed(a.out, **out)
    print("wrote", a.out, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
