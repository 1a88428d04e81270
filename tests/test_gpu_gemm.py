"""GPU parity of the tcgen05 projection GEMM and its fused epilogues against a float32 matmul
of the same bf16/fp16-representable operands.

Tolerance: fp32 accumulation in a different order, then one rounding of the output dtype:
|err| <= 2^-8 |ref| + 1e-3 * rms(ref) (bf16 outputs); float32 outputs (residual epilogue):
|err| <= 1e-4 * rms(ref) + 1e-6.
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle.numerics import bf16_round

pytestmark = pytest.mark.gpu


def _dev(x, dt=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda().to(dt)


def _gemm(epi, A, B, M, N, K, out=None, ldo=0, bias=None, aux_val=None, aux_idx=None,
          block_n=128, split_k=1):
    from tiny_infra_b200 import _native as N_
    N_.check(N_.lib().ti_gemm(
        epi, A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0), M, N, K,
        out.data_ptr() if out is not None else None, ldo,
        bias.data_ptr() if bias is not None else None,
        aux_val.data_ptr() if aux_val is not None else None,
        aux_idx.data_ptr() if aux_idx is not None else None,
        N_.dtype_code(A.dtype), block_n, split_k, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert N_.device_status() == 0


def _operands(seed, M, N, K, wstd=0.05):
    rng = np.random.default_rng(seed)
    a = bf16_round(rng.standard_normal((M, K)).astype(np.float32))
    b = bf16_round((rng.standard_normal((N, K)) * wstd).astype(np.float32))
    return a, b


def _close_bf16(got, ref):
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2))) + 1e-12
    err = np.abs(got - ref)
    assert (err <= 2.0 ** -8 * np.abs(ref) + 1e-3 * rms).all(), float(err.max())


@pytest.mark.parametrize("M,N,K,bn", [(256, 1152, 896, 64), (256, 1152, 896, 128),
                                      (37, 256, 128, 64), (4096, 1152, 896, 128),
                                      (300, 512, 896, 256)])
def test_store_bias(cuda_device, M, N, K, bn):
    from tiny_infra_b200 import _native as N_
    a, b = _operands(M * 7 + N, M, N, K)
    bias = bf16_round(np.random.default_rng(1).standard_normal(N).astype(np.float32) * 0.1)
    A, B, Bi = _dev(a), _dev(b), _dev(bias)
    out = torch.full((M, N), 9.0, dtype=torch.bfloat16, device="cuda")
    _gemm(N_.TI_EPI_STORE, A, B, M, N, K, out=out, ldo=N, bias=Bi, block_n=bn)
    _close_bf16(out.float().cpu().numpy(), a @ b.T + bias)


def test_store_fp16(cuda_device):
    from tiny_infra_b200 import _native as N_
    M, N, K = 200, 384, 640
    rng = np.random.default_rng(3)
    a = rng.standard_normal((M, K)).astype(np.float16).astype(np.float32)
    b = (rng.standard_normal((N, K)) * 0.05).astype(np.float16).astype(np.float32)
    A, B = _dev(a, torch.float16), _dev(b, torch.float16)
    out = torch.empty((M, N), dtype=torch.float16, device="cuda")
    _gemm(N_.TI_EPI_STORE, A, B, M, N, K, out=out, ldo=N)
    ref = a @ b.T
    err = np.abs(out.float().cpu().numpy() - ref)
    assert (err <= 2.0 ** -11 * np.abs(ref) + 1e-3).all()


@pytest.mark.parametrize("bn", [64, 128])
def test_swiglu_epilogue(cuda_device, bn):
    """gate/up projection with SwiGLU fused in the epilogue (weights interleaved per tile;
    block_n 64 stores 64-byte output rows)."""
    from tiny_infra_b200 import _native as N_
    M, I, K = 256, 1024, 896
    rng = np.random.default_rng(4)
    a = bf16_round(rng.standard_normal((M, K)).astype(np.float32))
    wg = bf16_round((rng.standard_normal((I, K)) * 0.05).astype(np.float32))
    wu = bf16_round((rng.standard_normal((I, K)) * 0.05).astype(np.float32))
    h = bn // 2
    inter = np.concatenate([np.concatenate([wg[j:j + h], wu[j:j + h]]) for j in range(0, I, h)])
    out = torch.empty((M, I), dtype=torch.bfloat16, device="cuda")
    _gemm(N_.TI_EPI_SWIGLU, _dev(a), _dev(inter), M, 2 * I, K, out=out, ldo=I, block_n=bn)
    g, u = a @ wg.T, a @ wu.T
    _close_bf16(out.float().cpu().numpy(), g / (1 + np.exp(-g)) * u)


@pytest.mark.parametrize("M,I,dt", [(256, 4864, "bf16"), (200, 4864, "bf16"), (129, 4864, "bf16"),
                                    (100, 1032, "bf16"), (256, 1032, "bf16"),
                                    (4096, 4864, "bf16"), (300, 1032, "bf16"), (1, 4864, "bf16"),
                                    (32, 4864, "bf16"), (37, 4864, "bf16"), (64, 4864, "fp16"),
                                    (17, 1032, "bf16"), (256, 4864, "fp16"), (4096, 1032, "fp16")])
def test_swiglu16_epilogue(cuda_device, M, I, dt):
    """gate/up + SwiGLU with gate/up rows interleaved in groups of 8 (TI_EPI_SWIGLU16), the
    model's layout: the library picks 80-, 144- or 256-wide tiles by M (80 at M <= 128 and
    2I = 2064: a ragged last tile of 64 columns; 144 at M = 200 / 256 and 2I = 9728: a last tile
    of 80; 256 above 256 rows, ragged at 2I = 2064).  At M <= 32 / 64 the activation box is 32 /
    64 rows and the ring holds all 14 K blocks (the MMA's rows past M read the rest of the stage
    and are dropped).  Output columns past I stay untouched."""
    from tiny_infra_b200 import _native as N_
    K = 896
    tdt = torch.bfloat16 if dt == "bf16" else torch.float16
    rnd = bf16_round if dt == "bf16" else (lambda x: x.astype(np.float16).astype(np.float32))
    rng = np.random.default_rng(M + I)
    a = rnd(rng.standard_normal((M, K)).astype(np.float32))
    wg = rnd((rng.standard_normal((I, K)) * 0.05).astype(np.float32))
    wu = rnd((rng.standard_normal((I, K)) * 0.05).astype(np.float32))
    inter = np.stack([wg.reshape(I // 8, 8, K), wu.reshape(I // 8, 8, K)], axis=1).reshape(2 * I, K)
    out = torch.full((M, I + 8), 7.0, dtype=tdt, device="cuda")
    _gemm(N_.TI_EPI_SWIGLU16, _dev(a, tdt), _dev(inter, tdt), M, 2 * I, K, out=out, ldo=I + 8,
          block_n=0)
    g, u = a @ wg.T, a @ wu.T
    got = out.float().cpu().numpy()
    _close_bf16(got[:, :I], g / (1 + np.exp(-g)) * u)
    assert (got[:, I:] == 7.0).all()


@pytest.mark.parametrize("M,split,bn", [(256, 1, 64), (256, 2, 64), (256, 3, 64), (256, 5, 64),
                                        (256, 8, 128), (256, 16, 128), (129, 10, 128),
                                        (200, 5, 64)])
def test_residual_split_k(cuda_device, M, split, bn):
    """x_f32 += A W^T with each split-K slice adding its partial tile into x (red.add); a second
    run agrees up to the fp32 rounding of the (varying) order of the slices' additions.  129-256
    rows run on CTA pairs (M = 256 MMAs over two SMs; at 129 / 200 the odd CTA's rows are
    mostly or partly past M)."""
    from tiny_infra_b200 import _native as N_
    N, K = 896, 4864
    a, b = _operands(5, M, N, K, wstd=0.02)
    x0 = np.random.default_rng(6).standard_normal((M, N)).astype(np.float32)
    x = torch.from_numpy(x0).cuda()
    _gemm(N_.TI_EPI_RESIDUAL, _dev(a), _dev(b), M, N, K, out=x, ldo=N, block_n=bn, split_k=split)
    ref = x0 + a @ b.T
    rms = float(np.sqrt(np.mean(ref ** 2)))
    got = x.cpu().numpy()
    assert np.abs(got - ref).max() <= 1e-4 * rms + 1e-6
    x2 = torch.from_numpy(x0).cuda()
    _gemm(N_.TI_EPI_RESIDUAL, _dev(a), _dev(b), M, N, K, out=x2, ldo=N, block_n=bn, split_k=split)
    # each of the `split` red.adds into an element rounds once (half an ulp of the running sum,
    # bounded by |x| + rms), in an order that varies between runs
    diff = np.abs(x2.cpu().numpy() - got)
    assert (diff <= split * 2.0 ** -23 * (np.abs(got) + rms)).all(), float(diff.max())


@pytest.mark.parametrize("M,N,K,split,bn", [(256, 896, 4864, 16, 128), (256, 896, 896, 7, 64),
                                            (32, 896, 4864, 16, 128), (37, 896, 896, 2, 64),
                                            (300, 896, 4864, 8, 128)])
def test_residual_deterministic(cuda_device, M, N, K, split, bn):
    """TI_EPI_RESIDUAL_DET: the K slices are summed in a fixed order on a cluster before one
    add per element, so two runs give bit-identical x, within the residual tolerance of the
    float32 reference."""
    from tiny_infra_b200 import _native as N_
    a, b = _operands(M + K, M, N, K, wstd=0.02)
    x0 = np.random.default_rng(6).standard_normal((M, N)).astype(np.float32)
    outs = []
    for _ in range(2):
        x = torch.from_numpy(x0).cuda()
        _gemm(N_.TI_EPI_RESIDUAL_DET, _dev(a), _dev(b), M, N, K, out=x, ldo=N, block_n=bn,
              split_k=split)
        outs.append(x.cpu().numpy())
    ref = x0 + a @ b.T
    rms = float(np.sqrt(np.mean(ref ** 2)))
    assert np.abs(outs[0] - ref).max() <= 1e-4 * rms + 1e-6
    np.testing.assert_array_equal(outs[0], outs[1])


@pytest.mark.parametrize("bn,split", [(64, 2), (64, 4), (64, 8), (128, 2), (128, 4), (128, 8)])
def test_cluster_split_k_store_and_swiglu(cuda_device, bn, split):
    """STORE (+bias) and SwiGLU epilogues on split-K tiles reduced through distributed shared
    memory; M = 200 leaves a partial M tile, K = 640 leaves split 8 with three empty splits."""
    from tiny_infra_b200 import _native as N_
    M, N, K = 200, 512, 640
    a, b = _operands(11 + bn + split, M, N, K)
    bias = bf16_round(np.random.default_rng(12).standard_normal(N).astype(np.float32) * 0.1)
    out = torch.full((M, N), 9.0, dtype=torch.bfloat16, device="cuda")
    _gemm(N_.TI_EPI_STORE, _dev(a), _dev(b), M, N, K, out=out, ldo=N, bias=_dev(bias),
          block_n=bn, split_k=split)
    _close_bf16(out.float().cpu().numpy(), a @ b.T + bias)
    # SwiGLU: tile columns [0, bn/2) gate, [bn/2, bn) up
    I, h = N // 2, bn // 2
    wg, wu = b[:I], b[I:]
    inter = np.concatenate([np.concatenate([wg[j:j + h], wu[j:j + h]]) for j in range(0, I, h)])
    act = torch.full((M, I), 9.0, dtype=torch.bfloat16, device="cuda")
    _gemm(N_.TI_EPI_SWIGLU, _dev(a), _dev(inter), M, N, K, out=act, ldo=I, block_n=bn,
          split_k=split)
    g, u = a @ wg.T, a @ wu.T
    _close_bf16(act.float().cpu().numpy(), g / (1 + np.exp(-g)) * u)


def test_argmax_epilogue(cuda_device):
    """Per-tile (max, first argmax) of each row; reduced over tiles it is the row argmax.
    Exact ties are planted to check the lowest-index rule."""
    from tiny_infra_b200 import _native as N_
    M, N, K, bn = 130, 32768, 896, 128
    a, b = _operands(7, M, N, K)
    b[5000] = b[123]                 # duplicate rows -> identical logits in columns 123, 5000
    a[0] = bf16_round(b[123] * 64.0)  # ... and make them row 0's maximum
    A, B = _dev(a), _dev(b)
    nt = N // bn
    val = torch.empty((M, nt), dtype=torch.float32, device="cuda")
    idx = torch.empty((M, nt), dtype=torch.int32, device="cuda")
    logits = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    _gemm(N_.TI_EPI_ARGMAX, A, B, M, N, K, out=logits, ldo=N, aux_val=val, aux_idx=idx, block_n=bn)
    ref = a @ b.T
    v, ix = val.cpu().numpy(), idx.cpu().numpy()
    t = np.argmax(v, axis=1)
    got = ix[np.arange(M), t]
    want = np.argmax(ref, axis=1)
    # where the top two logits are within accumulation noise the order may legitimately differ
    srt = np.sort(ref, axis=1)
    clear = (srt[:, -1] - srt[:, -2]) > 1e-3
    assert (got[clear] == want[clear]).all()
    np.testing.assert_allclose(v.max(axis=1), ref.max(axis=1), rtol=1e-5, atol=1e-4)
    _close_bf16(logits.float().cpu().numpy(), ref)
    assert got[0] == 123             # exact tie across tiles: lowest index wins
    assert (ix >= 0).all() and (ix < N).all()


@pytest.mark.parametrize("M", [1, 16, 32, 37, 64, 130, 256])
def test_argmax_persistent_lm_head(cuda_device, M):
    """Greedy lm_head without logits: up to 64 tokens the weight-streaming kernel (gemv.cu:
    tokens resident, weights as the MMA's M), above the persistent GEMM (both 128-row halves per
    CTA, two TMEM buffers): per-tile (max, first argmax) equal to the float32 reference; ties
    planted within a tile and across tiles resolve to the lowest index."""
    from tiny_infra_b200 import _native as N_
    N, K, bn = 151936, 896, 128
    a, b = _operands(M + 3, M, N, K)
    b[140000] = b[77]
    b[78] = b[77]
    a[M - 1] = bf16_round(b[77] * 64.0)
    nt = N // bn
    val = torch.empty((M, nt), dtype=torch.float32, device="cuda")
    idx = torch.empty((M, nt), dtype=torch.int32, device="cuda")
    _gemm(N_.TI_EPI_ARGMAX, _dev(a), _dev(b), M, N, K, aux_val=val, aux_idx=idx, block_n=bn)
    ref = a @ b.T
    v, ix = val.cpu().numpy(), idx.cpu().numpy()
    np.testing.assert_allclose(v, ref.reshape(M, nt, bn).max(axis=2), rtol=1e-5, atol=1e-4)
    got = ix[np.arange(M), np.argmax(v, axis=1)]
    srt = np.sort(ref, axis=1)
    clear = (srt[:, -1] - srt[:, -2]) > 1e-3
    assert (got[clear] == np.argmax(ref, axis=1)[clear]).all()
    assert got[M - 1] == 77
    assert (ix >= 0).all() and (ix < N).all()


def test_pairs_at_decode_sizes(cuda_device):
    """The SwiGLU16 and residual cases again with CTA pairs (M = 256 MMAs on two SMs) for every
    batch above 128 rows (TI_GEMM_PAIR=1; by default only batches above 256 rows use them), in
    a child process because the library reads the switch once."""
    if os.environ.get("TI_GEMM_PAIR") == "1":
        pytest.skip("this process already runs with pairs at every size")
    env = dict(os.environ, TI_GEMM_PAIR="1")
    r = subprocess.run([sys.executable, "-m", "pytest", os.path.abspath(__file__), "-q", "-x",
                        "-m", "gpu", "-k", "swiglu16 or residual_split"],
                       env=env, capture_output=True, text=True, timeout=900,
                       cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
