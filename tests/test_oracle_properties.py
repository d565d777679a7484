"""CPU: the oracle against the properties the reference's own CPU tests assert, restated on
seeded inputs of this project's generator.

- the per-token / per-tensor scale formula and the int8 range (tests/test_quant.py:17-38);
- the round-trip error bound of symmetric quantisation (tests/test_quant.py:41-50);
- outlier saturation (tests/test_quant.py:53-64);
- dequantisation broadcasts one scale per (block, kv-head, token) (tests/test_quant.py:67-82);
- the scatter + dequantise round trip of the INT8 cache builder (tests/test_quant.py:85-111);
- paged attention equals dense attention over the contiguous K/V (test_paged_decode_attn.py:
  55-77).
"""

import math

import numpy as np
import pytest

import gen
import pa_oracle


def test_per_token_scale_formula_and_range():
    x = gen.Gen(20).normal((4, 7, 128)).astype(np.float32)
    q, s = pa_oracle.quantize_per_token(x, "f32")
    expect = np.maximum(np.abs(x).max(axis=-1), np.float32(1e-8)) / np.float32(127)  # fp32
    assert s.shape == (4, 7) and q.dtype == np.int8
    assert np.array_equal(s, expect.astype(np.float32))
    assert np.abs(q.astype(np.int32)).max() <= 127


def test_per_tensor_scale_formula_and_range():
    x = gen.Gen(21).normal((4, 7, 128)).astype(np.float32)
    q, s = pa_oracle.quantize_per_tensor(x, "f32")
    assert np.float32(s) == np.float32(max(np.abs(x).max(), np.float32(1e-8)) / np.float32(127))
    assert q.dtype == np.int8 and np.abs(q.astype(np.int32)).max() <= 127


def test_per_token_round_trip_bound():
    x = gen.Gen(22).normal((8, 256)).astype(np.float32)
    q, s = pa_oracle.quantize_per_token(x, "f32")
    dq = q.astype(np.float32) * s[:, None]
    # |error| <= scale / 2 per element (round to nearest), hence a small norm-relative error.
    assert (np.abs(dq - x) <= s[:, None] / 2 * (1 + 1e-6)).all()
    assert np.linalg.norm(dq - x) / np.linalg.norm(x) < 0.02


def test_outlier_saturates_and_drives_its_token_scale():
    x = gen.Gen(23).normal((2, 64)).astype(np.float32)
    x[0, 0] = 1000.0
    q, s = pa_oracle.quantize_per_token(x, "f32")
    assert np.abs(q.astype(np.int32)).max() <= 127
    assert q[0, 0] == 127
    assert s[0] > s[1]


def test_dequantize_broadcasts_per_token_scales():
    g = gen.Gen(24)
    nb, kvh, d, bs, x = 2, 2, 8, 4, 2
    kc = (g.randint(-127, 128, (nb, kvh, d // x, bs, x))).astype(np.int8)
    vc = (g.randint(-127, 128, (nb, kvh, d, bs))).astype(np.int8)
    ks = g.uniform((nb, kvh, bs)).astype(np.float32)
    vs = g.uniform((nb, kvh, bs)).astype(np.float32)
    kd, vd = pa_oracle.dequantize_kv(kc, vc, ks, vs)
    assert kd.shape == kc.shape and vd.shape == vc.shape
    for (b, h, c, t, w) in [(1, 0, 2, 3, 1), (0, 1, 0, 0, 0), (1, 1, 3, 2, 1)]:
        assert kd[b, h, c, t, w] == np.float32(kc[b, h, c, t, w]) * ks[b, h, t]
    for (b, h, e, t) in [(1, 1, 5, 2), (0, 0, 7, 3)]:
        assert vd[b, h, e, t] == np.float32(vc[b, h, e, t]) * vs[b, h, t]


def test_int8_cache_round_trip_within_half_a_step():
    c = gen.decode_case(seed=25, num_seqs=2, num_heads=4, num_kv_heads=2,
                        context_lens=[40, 33])
    k = c["k"].astype(np.float32)
    v = c["v"].astype(np.float32)
    lens, bt, nb = c["context_lens"], c["block_table"], c["num_blocks"]
    kq, ksc = pa_oracle.quantize_per_token(k, "f32")
    vq, vsc = pa_oracle.quantize_per_token(v, "f32")
    kc, vc = pa_oracle.scatter_paged_cache(kq, vq, lens, bt, nb)
    kd, vd = pa_oracle.dequantize_kv(kc, vc, pa_oracle.scatter_scales(ksc, lens, bt, nb, 2),
                                     pa_oracle.scatter_scales(vsc, lens, bt, nb, 2))
    for b in range(2):
        n = int(lens[b])
        kg, vg = pa_oracle.gather_seq(kd, vd, bt, n, b)           # [n, KVH, D]
        tol_k = np.abs(k[b, :n]).max(axis=-1, keepdims=True) / 127 / 2 + 1e-6
        tol_v = np.abs(v[b, :n]).max(axis=-1, keepdims=True) / 127 / 2 + 1e-6
        assert (np.abs(kg - k[b, :n]) <= tol_k).all()
        assert (np.abs(vg - v[b, :n]) <= tol_v).all()


@pytest.mark.parametrize("heads", [(8, 8), (8, 2), (12, 2)])
def test_paged_attention_equals_dense_attention(heads):
    H, KVH = heads
    lens = [1, 17, 130]
    c = gen.decode_case(seed=26, num_seqs=3, num_heads=H, num_kv_heads=KVH, context_lens=lens)
    kc, vc = pa_oracle.scatter_paged_cache(c["k"], c["v"], c["context_lens"], c["block_table"],
                                           c["num_blocks"])
    out = pa_oracle.paged_decode_attention(c["q"], kc, vc, c["block_table"], c["context_lens"])
    G = H // KVH
    for b, n in enumerate(lens):
        for h in range(H):
            kk = c["k"][b, :n, h // G].astype(np.float64)        # dense [n, D]
            vv = c["v"][b, :n, h // G].astype(np.float64)
            s = kk @ c["q"][b, h].astype(np.float64) / math.sqrt(128)
            p = np.exp(s - s.max())
            ref = (p / p.sum()) @ vv
            np.testing.assert_allclose(out[b, h], ref, atol=1e-5, rtol=1e-5)
