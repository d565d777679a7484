"""CPU: pin the numpy oracle to golden vectors produced by the reference implementation
(tests/golden/make_golden.py). Bit-exact for quantisation, 1e-5 for attention."""

import os

import numpy as np
import pytest

import gen
import pa_oracle

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    return np.load(os.path.join(GOLD, name))


def test_scale_table_f16_exhaustive():
    g = _load("scale_tables.npz")
    amax = g["f16_bits"].view(np.float16).astype(np.float32)
    s = pa_oracle.scale_from_amax(amax, "f16")
    assert np.array_equal(s.view(np.uint32), g["f16_scale"].view(np.uint32))


def test_scale_table_bf16_exhaustive():
    g = _load("scale_tables.npz")
    amax = (g["bf16_bits"].astype(np.uint32) << 16).view(np.float32)
    s = pa_oracle.scale_from_amax(amax, "bf16")
    assert np.array_equal(s.view(np.uint32), g["bf16_scale"].view(np.uint32))


@pytest.mark.parametrize("dt", ["16", "32", "bf16"])
def test_quantize_per_token_rows(dt):
    g = _load("quant_rows.npz")
    if dt == "16":
        x, dtype = g["x16"], "f16"
    elif dt == "32":
        x, dtype = g["x32"], "f32"
    else:
        x, dtype = (g["xbf16_bits"].astype(np.uint32) << 16).view(np.float32), "bf16"
    q, s = pa_oracle.quantize_per_token(x, dtype)
    assert np.array_equal(q, g["q" + dt])
    assert np.array_equal(s.view(np.uint32), g["s" + dt].view(np.uint32))


def test_quantize_edge_semantics():
    """The edge rows: zero row -> (0, scale 0); fp16 subnormal row -> scale 0 and +-127;
    exact .5 ties round to even; inf -> scale inf, values 0."""
    g = _load("quant_rows.npz")
    q, s = g["q16"], g["s16"]
    assert s[0] == 0 and not q[0].any()
    assert s[1] == 0 and list(q[1, :4]) == [127, 0, -127, 127]
    assert s[3] == 1.0 and list(q[3, 1:9]) == [0, 2, 2, 0, -2, -2, 126, -126]
    assert np.isinf(s[7]) and not q[7].any()


def test_quantize_per_tensor():
    g = _load("quant_rows.npz")
    q, s = pa_oracle.quantize_per_tensor(g["xt"], "f16")
    assert np.array_equal(q, g["qt"]) and np.float32(s) == g["st"]
    q0, s0 = pa_oracle.quantize_per_tensor(np.zeros((3, 128), np.float16), "f16")
    assert np.array_equal(q0, g["qz"]) and np.float32(s0) == g["sz"]


def _cfg1():
    lens = gen.Gen(1).randint(64, 513, (4,))
    c = gen.decode_case(seed=101, num_seqs=4, num_heads=12, num_kv_heads=2, context_lens=lens,
                        num_blocks=256)
    return c


def test_decode_cfg1_fp16():
    g = _load("decode_cfg1.npz")
    c = _cfg1()
    assert gen.sha256_arrays(c["q"], c["k"], c["v"], c["context_lens"],
                             c["block_table"]) == str(g["input_sha"]), "input generator drift"
    kc, vc = pa_oracle.scatter_paged_cache(c["k"], c["v"], c["context_lens"], c["block_table"],
                                           c["num_blocks"])
    out = pa_oracle.paged_decode_attention(c["q"], kc, vc, c["block_table"], c["context_lens"])
    np.testing.assert_allclose(out, g["out_f16"], atol=1e-5, rtol=1e-5)
    out_loop = pa_oracle.paged_decode_attention_loop(c["q"], kc, vc, c["block_table"],
                                                     c["context_lens"])
    np.testing.assert_allclose(out_loop, g["out_f16"], atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("mode", ["per_token", "per_tensor"])
def test_decode_cfg1_int8(mode):
    g = _load("decode_cfg1.npz")
    c = _cfg1()
    k, v, lens, bt, nb = c["k"], c["v"], c["context_lens"], c["block_table"], c["num_blocks"]
    if mode == "per_token":
        kq, ks = pa_oracle.quantize_per_token(k, "f16")
        vq, vs = pa_oracle.quantize_per_token(v, "f16")
    else:
        kq, a = pa_oracle.quantize_per_tensor(k, "f16")
        vq, b = pa_oracle.quantize_per_tensor(v, "f16")
        ks = np.full(k.shape[:-1], a, np.float32)
        vs = np.full(v.shape[:-1], b, np.float32)
    assert gen.sha256_arrays(kq, vq, ks, vs) == str(g[f"kq_{mode}_sha"])
    kc, vc = pa_oracle.scatter_paged_cache(kq, vq, lens, bt, nb)
    kd, vd = pa_oracle.dequantize_kv(kc, vc, pa_oracle.scatter_scales(ks, lens, bt, nb, 2),
                                     pa_oracle.scatter_scales(vs, lens, bt, nb, 2))
    out = pa_oracle.paged_decode_attention(c["q"], kd, vd, bt, lens)
    np.testing.assert_allclose(out, g[f"out_{mode}"], atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("variant", ["fp16", "int8_per_token", "int8_per_tensor"])
def test_bridge_cache_writes(variant):
    g = _load("bridge_cache.npz")
    k, v = g["k"], g["v"]
    c = pa_oracle.BridgeCacheOracle(2, 128, 40, variant=variant)
    c.prefill(k[:-1], v[:-1])
    assert c.decode_append(k[-1], v[-1]) == k.shape[0]
    assert np.array_equal(c.k_cache, g[f"{variant}_k"])
    assert np.array_equal(c.v_cache, g[f"{variant}_v"])
    if variant != "fp16":
        assert np.array_equal(c.k_scales.view(np.uint32), g[f"{variant}_ks"].view(np.uint32))
        assert np.array_equal(c.v_scales.view(np.uint32), g[f"{variant}_vs"].view(np.uint32))


def test_split_partials_merge_to_full_decode():
    """Property: LSE-merging 512-token split partials equals the one-pass decode."""
    c = gen.decode_case(seed=5, num_seqs=2, num_heads=8, num_kv_heads=2,
                        context_lens=[1300, 700])
    kc, vc = pa_oracle.scatter_paged_cache(c["k"], c["v"], c["context_lens"], c["block_table"],
                                           c["num_blocks"])
    sc = 1 / np.sqrt(128)
    parts = pa_oracle.split_partials(c["q"], kc, vc, c["block_table"], c["context_lens"], sc)
    merged = pa_oracle.lse_merge([p[0] for p in parts], [p[1] for p in parts],
                                 [p[2] for p in parts])
    full = pa_oracle.paged_decode_attention(c["q"], kc, vc, c["block_table"], c["context_lens"],
                                            scale=sc)
    np.testing.assert_allclose(merged, full, atol=1e-6, rtol=1e-6)
