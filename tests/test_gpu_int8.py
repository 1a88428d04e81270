"""GPU parity of the weight-only INT8 lm_head against its numpy definition (oracle/quant.py):

* ti_quantize_rows_int8: int8 values and scales bit-exact on the tied lm_head of the model's
  dimensions (151936 x 896, random-init bf16 weights) and on rows with zeros and ties;
* ti_lm_head_argmax_int8 (+ ti_argmax_finish): the greedy token of every row equals the argmax of
  the float32 logits of the dequantised weights, except where the oracle's own top-2 gap is below
  1e-5 of the logit scale (float32 accumulation order), at 1 / 32 / 37 / 256 rows; every
  (row, tile) maximum within 1e-5 of the logit scale of the oracle's;
* the graph-captured DecodeEngine with the int8 lm_head: a greedy step of a 2-layer model gives
  the oracle's tokens with the dequantised lm_head.
"""
import numpy as np
import pytest
import torch

from oracle import kernels as OK
from oracle import model as OM
from oracle import quant as OQ
from oracle.cache import OracleKVCache
from oracle.numerics import bf16_round

pytestmark = pytest.mark.gpu
V, H = 151936, 896


def _quantize(w_dev):
    from tiny_infra_b200 import _native as N_
    rows, cols = w_dev.shape
    q = torch.empty(rows, cols, dtype=torch.int8, device=w_dev.device)
    s = torch.empty(rows, dtype=torch.float32, device=w_dev.device)
    N_.check(N_.lib().ti_quantize_rows_int8(w_dev.data_ptr(), cols, rows, cols, q.data_ptr(), cols,
                                            s.data_ptr(), N_.TI_DTYPE_BF16,
                                            torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return q, s


def test_quantize_rows_bit_exact(cuda_device):
    rng = np.random.default_rng(0)
    w = bf16_round((rng.standard_normal((V, H)) * 0.02).astype(np.float32))
    w[3] = 0.0                                   # all-zero row: scale 1, q 0
    w[5, :8] = np.float32(0.25)                  # ties of |w| at the maximum
    w[7, 0] = -w[7].__abs__().max() * 2          # a negative maximum
    q, s = _quantize(torch.from_numpy(w).to(cuda_device, torch.bfloat16))
    rq, rs = OQ.quantize_rows_int8(w)
    np.testing.assert_array_equal(s.cpu().numpy(), rs)
    np.testing.assert_array_equal(q.cpu().numpy(), rq)


@pytest.mark.parametrize("M", [1, 32, 37, 256])
def test_lm_head_argmax_int8(cuda_device, M):
    from tiny_infra_b200 import _native as N_
    rng = np.random.default_rng(M)
    w = bf16_round((rng.standard_normal((V, H)) * 0.02).astype(np.float32))
    x = bf16_round(rng.standard_normal((M, H)).astype(np.float32))
    q, s = _quantize(torch.from_numpy(w).to(cuda_device, torch.bfloat16))
    nt = V // 128
    val = torch.full((M, nt), 7.0, dtype=torch.float32, device=cuda_device)
    idx = torch.full((M, nt), -1, dtype=torch.int32, device=cuda_device)
    tok = torch.zeros(M, dtype=torch.int32, device=cuda_device)
    xd = torch.from_numpy(x).to(cuda_device, torch.bfloat16)
    st = torch.cuda.current_stream().cuda_stream
    lib = N_.lib()
    N_.check(lib.ti_lm_head_argmax_int8(xd.data_ptr(), H, q.data_ptr(), H, s.data_ptr(), M, V, H,
                                        val.data_ptr(), idx.data_ptr(), N_.TI_DTYPE_BF16, st))
    N_.check(lib.ti_argmax_finish(val.data_ptr(), idx.data_ptr(), nt, M, tok.data_ptr(), None,
                                  None, 0, st))
    torch.cuda.synchronize()
    assert N_.device_status() == 0
    ref = OQ.int8_logits(x, q.cpu().numpy(), s.cpu().numpy())
    scale = float(np.abs(ref).max())
    tiles = ref.reshape(M, nt, 128)
    np.testing.assert_allclose(val.cpu().numpy(), tiles.max(axis=2), rtol=0, atol=1e-5 * scale)
    got = tok.cpu().numpy()
    want = ref.argmax(axis=1)
    srt = np.sort(ref, axis=1)
    clear = (srt[:, -1] - srt[:, -2]) > 1e-5 * scale
    np.testing.assert_array_equal(got[clear], want[clear])
    assert clear.sum() >= M - 1


def test_engine_greedy_step_int8_lm_head(cuda_device):
    from tiny_infra_b200.cache_manager import KVCacheManager
    from tiny_infra_b200.config import QwenConfig
    from tiny_infra_b200.engine import DecodeEngine
    from tiny_infra_b200.qwen2 import Qwen2ForCausalLM
    L, S = 2, 64
    cfg = QwenConfig(num_layers=L, vocab_size=V)
    sd = Qwen2ForCausalLM.random_state_dict(cfg, seed=2, tied=True)
    model = Qwen2ForCausalLM(cfg).load_reference_state_dict(sd).quantize_lm_head_int8()
    model.deterministic = True
    kv = KVCacheManager(4, S, L, cfg.num_key_value_heads, cfg.head_dim)
    eng = DecodeEngine(model, kv)
    W = {k: v.float().cpu().numpy() for k, v in sd.items()}
    q = model.weights["lm_head_q"].cpu().numpy()
    sc = model.weights["lm_head_scale"].cpu().numpy()
    W["lm_head.weight"] = (q.astype(np.float32) * sc[:, None]).astype(np.float32)
    oc = OracleKVCache(4, S, L, cfg.num_key_value_heads, cfg.head_dim)
    ocfg = OM.OracleConfig(num_layers=L, vocab_size=V)
    cos, sin = OK.rope_table(S, cfg.head_dim, cfg.rope_theta)
    rng = np.random.default_rng(9)
    slots = [0, 1, 2, 3]
    for slot in slots:
        p = rng.integers(0, V, 5 + 3 * slot)
        pb = model.plan(kv, [slot], [len(p)], p)
        model.forward_packed(pb, kv, eng.cos, eng.sin, rows="last")
        kv.advance_device([slot], len(p))
        OM.forward(W, ocfg, p[None], np.array([slot]), oc, cos, sin, device_rounding="bf16",
                   last_only=True)
        oc.seq_len[slot] += len(p)
    first = rng.integers(0, V, 4)
    toks = eng.step(slots, first)
    ol = OM.forward(W, ocfg, first[:, None], np.array(slots), oc, cos, sin,
                    device_rounding="bf16")[:, 0]
    near = 0
    for i in range(4):
        srt = np.sort(ol[i])
        if int(toks[i]) != int(np.argmax(ol[i])):
            assert srt[-1] - srt[-2] < 0.05, (i, float(srt[-1] - srt[-2]))
            near += 1
    assert near <= 1
    np.testing.assert_array_equal(kv.block_tables.cpu().numpy(), oc.block_tables)
