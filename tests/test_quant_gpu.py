"""GPU parity of the cache-write kernels: bit-exact INT8 values and scales against the
oracle (which the golden vectors pin to the reference quantizer), FP16 copies, the bulk
prefill scatter, per-tensor scales and the bridge cache."""

import os

import numpy as np
import pytest
import torch

import gen
import pa_oracle
from pa_testlib import to_cuda

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _ops():
    from pa_b200 import ops
    return ops


def _caches(nb, kvh, bs=16, int8=True):
    dt = torch.int8 if int8 else torch.float16
    kc = torch.zeros(nb, kvh, 16, bs, 8, dtype=dt, device="cuda")
    vc = torch.zeros(nb, kvh, 128, bs, dtype=dt, device="cuda")
    ks = torch.zeros(nb, kvh, bs, dtype=torch.float32, device="cuda")
    vs = torch.zeros(nb, kvh, bs, dtype=torch.float32, device="cuda")
    return kc, vc, ks, vs


def _oracle_rows(k, v, slots, nb, kvh, bs, in_dtype, k_fix=None, v_fix=None):
    """Oracle cache after writing rows k, v [N, KVH, D] at slots (negative skipped)."""
    if k_fix is None:
        kq, ksc = pa_oracle.quantize_per_token(k, in_dtype)
        vq, vsc = pa_oracle.quantize_per_token(v, in_dtype)
    else:
        kq = pa_oracle.quantize_with_scale(k.astype(np.float32), k_fix)
        vq = pa_oracle.quantize_with_scale(v.astype(np.float32), v_fix)
        ksc = np.full(k.shape[:-1], k_fix, np.float32)
        vsc = np.full(v.shape[:-1], v_fix, np.float32)
    kc = np.zeros((nb, kvh, 16, bs, 8), np.int8)
    vc = np.zeros((nb, kvh, 128, bs), np.int8)
    ks = np.zeros((nb, kvh, bs), np.float32)
    vs = np.zeros((nb, kvh, bs), np.float32)
    for n, s in enumerate(slots):
        if s < 0:
            continue
        b, o = s // bs, s % bs
        kc[b, :, :, o, :] = kq[n].reshape(kvh, 16, 8)
        vc[b, :, :, o] = vq[n]
        ks[b, :, o] = ksc[n]
        vs[b, :, o] = vsc[n]
    return kc, vc, ks, vs


def _bits_equal(a, b):
    a = a.cpu().numpy() if hasattr(a, "cpu") else a
    if a.dtype == np.float32:
        return np.array_equal(a.view(np.uint32), np.asarray(b, np.float32).view(np.uint32))
    return np.array_equal(a, b)


@pytest.mark.parametrize("source", ["golden16", "golden32", "goldenbf16", "outlier"])
def test_quantize_rows_bit_exact(source):
    gold = np.load(os.path.join(GOLD, "quant_rows.npz"))
    if source == "golden16":
        x, dtype, tdt = gold["x16"], "f16", torch.float16
    elif source == "golden32":
        x, dtype, tdt = gold["x32"], "f32", torch.float32
    elif source == "goldenbf16":
        x = (gold["xbf16_bits"].astype(np.uint32) << 16).view(np.float32)
        dtype, tdt = "bf16", torch.bfloat16
    else:
        g = gen.Gen(3)
        x = gen.kv_values(g, (300, 1, 128), "lognormal_outlier")[:, 0].astype(np.float16)
        dtype, tdt = "f16", torch.float16
    R = x.shape[0] - x.shape[0] % 2
    x = x[:R]
    kvh, bs = 2, 16
    N = R // kvh
    k = x.reshape(N, kvh, 128)
    v = np.ascontiguousarray(k[::-1])
    nb = (N + bs - 1) // bs + 3
    slots = gen.Gen(4).permutation(nb * bs)[:N].astype(np.int32)
    slots[1] = -1  # padding token: skipped
    kc, vc, ks, vs = _caches(nb, kvh, bs)
    tk = torch.from_numpy(np.ascontiguousarray(k)).to(tdt).cuda() if tdt == torch.bfloat16 \
        else torch.from_numpy(np.ascontiguousarray(k)).cuda()
    tv = torch.from_numpy(np.ascontiguousarray(v)).to(tdt).cuda() if tdt == torch.bfloat16 \
        else torch.from_numpy(np.ascontiguousarray(v)).cuda()
    _ops().quantize_into_cache(tk, tv, kc, vc, ks, vs, torch.from_numpy(slots).cuda(), bs)
    okc, ovc, oks, ovs = _oracle_rows(k, v, slots, nb, kvh, bs, dtype)
    assert _bits_equal(kc, okc) and _bits_equal(vc, ovc)
    assert _bits_equal(ks, oks) and _bits_equal(vs, ovs)


def test_quantize_matches_golden_directly():
    """Kernel scales/values for the golden fp16 rows equal the reference's, element for
    element (no oracle in between)."""
    gold = np.load(os.path.join(GOLD, "quant_rows.npz"))
    x = gold["x16"]
    N = x.shape[0]
    kc, vc, ks, vs = _caches(N, 1, 16)
    slots = (np.arange(N, dtype=np.int32) * 16)  # token n -> block n, offset 0
    tx = torch.from_numpy(x.reshape(N, 1, 128)).cuda()
    _ops().quantize_into_cache(tx, tx, kc, vc, ks, vs, torch.from_numpy(slots).cuda(), 16)
    got_q = kc[:, 0, :, 0, :].reshape(N, 128).cpu().numpy()
    got_s = ks[:, 0, 0].cpu().numpy()
    assert np.array_equal(got_q, gold["q16"])
    assert np.array_equal(got_s.view(np.uint32), gold["s16"].view(np.uint32))
    got_v = vc[:, 0, :, 0].cpu().numpy()
    assert np.array_equal(got_v, gold["q16"])


def test_quantize_fixed_scale():
    g = gen.Gen(12)
    k = gen.kv_values(g, (40, 2, 128), "lognormal_outlier").astype(np.float16)
    v = gen.kv_values(g, (40, 2, 128), "normal").astype(np.float16)
    sk, sv = np.float32(0.37), np.float32(0.021)
    slots = np.arange(40, dtype=np.int32) + 5
    kc, vc, ks, vs = _caches(4, 2)
    tk, tv = to_cuda(k, v)
    _ops().quantize_into_cache(tk, tv, kc, vc, ks, vs, torch.from_numpy(slots).cuda(), 16,
                               k_scale=torch.tensor(sk, device="cuda"),
                               v_scale=torch.tensor(sv, device="cuda"))
    okc, ovc, oks, ovs = _oracle_rows(k, v, slots, 4, 2, 16, "f16", sk, sv)
    assert _bits_equal(kc, okc) and _bits_equal(vc, ovc)
    assert _bits_equal(ks, oks) and _bits_equal(vs, ovs)


def test_out_of_range_slot_flagged():
    ops = _ops()
    ops.read_status()
    k = torch.randn(3, 2, 128, dtype=torch.float16, device="cuda")
    kc, vc, ks, vs = _caches(2, 2)
    slots = torch.tensor([0, 999, 5], dtype=torch.int32, device="cuda")
    ops.quantize_into_cache(k, k, kc, vc, ks, vs, slots, 16)
    torch.cuda.synchronize()
    assert ops.read_status() & 256  # PA_ERR_SLOT


def test_fp16_write_into_cache():
    g = gen.Gen(13)
    k = gen.kv_values(g, (50, 4, 128), "normal")
    v = gen.kv_values(g, (50, 4, 128), "normal")
    slots = gen.Gen(14).permutation(64)[:50].astype(np.int32)
    kc, vc, _, _ = _caches(4, 4, int8=False)
    tk, tv = to_cuda(k, v)  # fp32 input: rounded to fp16 by the kernel
    _ops().write_into_cache(tk, tv, kc, vc, torch.from_numpy(slots).cuda(), 16)
    ok = np.zeros((4, 4, 16, 16, 8), np.float16)
    ov = np.zeros((4, 4, 128, 16), np.float16)
    for n, s in enumerate(slots):
        ok[s // 16, :, :, s % 16, :] = k[n].astype(np.float16).reshape(4, 16, 8)
        ov[s // 16, :, :, s % 16] = v[n].astype(np.float16)
    assert np.array_equal(kc.cpu().numpy().view(np.uint16), ok.view(np.uint16))
    assert np.array_equal(vc.cpu().numpy().view(np.uint16), ov.view(np.uint16))


@pytest.mark.parametrize("bs", [16, 32, 64])
@pytest.mark.parametrize("int8", [True, False])
def test_prefill_scatter(bs, int8):
    lens = [1, 33, 200, 64]
    c = gen.decode_case(15, 4, 8, 2, lens, block_size=bs, dist="lognormal_outlier",
                        num_blocks=40)
    k, v, cl, bt, nb = c["k"], c["v"], c["context_lens"], c["block_table"], c["num_blocks"]
    kc, vc, ks, vs = _caches(nb, 2, bs, int8)
    tk, tv, tbt, tcl = to_cuda(k, v, bt, cl)
    kw = dict(k_scales=ks, v_scales=vs) if int8 else {}
    _ops().prefill_into_cache(tk, tv, kc, vc, tbt, tcl, bs, **kw)
    if int8:
        kq, ksc = pa_oracle.quantize_per_token(k, "f16")
        vq, vsc = pa_oracle.quantize_per_token(v, "f16")
        okc, ovc = pa_oracle.scatter_paged_cache(kq, vq, cl, bt, nb, bs)
        oks = pa_oracle.scatter_scales(ksc, cl, bt, nb, 2, bs)
        ovs = pa_oracle.scatter_scales(vsc, cl, bt, nb, 2, bs)
        assert _bits_equal(ks, oks) and _bits_equal(vs, ovs)
    else:
        okc, ovc = pa_oracle.scatter_paged_cache(k, v, cl, bt, nb, bs)
    assert np.array_equal(kc.cpu().numpy().view(np.uint8), okc.view(np.uint8))
    assert np.array_equal(vc.cpu().numpy().view(np.uint8), ovc.view(np.uint8))


@pytest.mark.parametrize("dtype", ["f16", "bf16", "f32"])
def test_absmax_scales(dtype):
    from pa_b200 import _lib
    g = gen.Gen(16)
    x = gen.kv_values(g, (33, 2, 128), "lognormal_outlier")
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[dtype]
    tx = torch.from_numpy(x).to(tdt).cuda()
    xr = tx.float().cpu().numpy()
    a = _ops().absmax_scale(tx, _lib.PA_SCALE_CLAMP_THEN_DIVIDE).item()
    b = _ops().absmax_scale(tx, _lib.PA_SCALE_DIVIDE_THEN_CLAMP).item()
    assert np.float32(a) == pa_oracle.quantize_per_tensor(xr, dtype)[1]
    assert np.float32(b) == pa_oracle.bridge_tensor_scale(xr, dtype)
    z = torch.zeros(10, 128, dtype=tdt, device="cuda")
    assert np.float32(_ops().absmax_scale(z).item()) == pa_oracle.quantize_per_tensor(
        np.zeros((10, 128), np.float32), dtype)[1]


@pytest.mark.parametrize("variant", ["fp16", "int8_per_token", "int8_per_tensor"])
def test_bridge_cache_matches_reference_golden(variant):
    from pa_b200.paged_cache import PagedKVCache
    gold = np.load(os.path.join(GOLD, "bridge_cache.npz"))
    k, v = torch.from_numpy(gold["k"]).cuda(), torch.from_numpy(gold["v"]).cuda()
    c = PagedKVCache(1, 2, 128, 40, variant=variant, device="cuda")
    c.prefill(0, k[:-1], v[:-1])
    assert c.decode_append(0, k[-1], v[-1]) == k.shape[0]
    assert np.array_equal(c.k_cache[0].cpu().numpy().view(np.uint8),
                          gold[f"{variant}_k"].view(np.uint8))
    assert np.array_equal(c.v_cache[0].cpu().numpy().view(np.uint8),
                          gold[f"{variant}_v"].view(np.uint8))
    if variant != "fp16":
        assert _bits_equal(c.k_scales[0], gold[f"{variant}_ks"])
        assert _bits_equal(c.v_scales[0], gold[f"{variant}_vs"])


@pytest.mark.parametrize("variant", ["fp16", "int8_per_token", "int8_per_tensor"])
@pytest.mark.parametrize("clen", [17, 31, 128, 500])
def test_bridge_decode_append_then_decode(variant, clen):
    """The bridge flow of tests/test_int8_bridge.py:104-128 at Qwen's 12/2 heads: prefill
    clen-1 tokens, append one, decode with the split-K op, compare with the oracle."""
    from pa_b200 import cuda_ext
    from pa_b200.paged_cache import PagedKVCache
    from pa_testlib import assert_close, scale_for
    g = gen.Gen(17)
    k = gen.kv_values(g, (clen, 2, 128), "normal").astype(np.float16)
    v = gen.kv_values(g, (clen, 2, 128), "normal").astype(np.float16)
    q = g.normal((1, 12, 128)).astype(np.float16)
    c = PagedKVCache(1, 2, 128, clen, variant=variant, device="cuda")
    tk, tv, tq = to_cuda(k, v, q)
    c.prefill(0, tk[:-1], tv[:-1])
    assert c.decode_append(0, tk[-1], tv[-1]) == clen
    out = torch.empty_like(tq)
    ctx = c.context_lens(0)
    if c.is_int8:
        cuda_ext.VARIANTS_INT8["splitk_int8"](out, tq, c.k_cache[0], c.v_cache[0],
                                              c.k_scales[0], c.v_scales[0], c.block_table, ctx,
                                              scale_for(), 16)
        kd, vd = pa_oracle.dequantize_kv(c.k_cache[0].cpu().numpy(), c.v_cache[0].cpu().numpy(),
                                         c.k_scales[0].cpu().numpy(), c.v_scales[0].cpu().numpy())
    else:
        cuda_ext.VARIANTS["splitk"](out, tq, c.k_cache[0], c.v_cache[0], c.block_table, ctx,
                                    scale_for(), 16)
        kd, vd = c.k_cache[0].cpu().numpy(), c.v_cache[0].cpu().numpy()
    ref = pa_oracle.paged_decode_attention(q, kd, vd, c.block_table.cpu().numpy(),
                                           np.array([clen]))
    assert_close(out, ref)


def test_int8_cache_smaller_than_fp16():
    from pa_b200.paged_cache import PagedKVCache
    kw = dict(num_layers=28, num_kv_heads=2, head_dim=128, max_len=2048, device="cuda")
    fp16 = PagedKVCache(variant="fp16", **kw).kv_bytes()
    int8 = PagedKVCache(variant="int8_per_token", **kw).kv_bytes()
    assert int8 / fp16 < 0.6


def _near_half_integers(rng, shape, s):
    """fp16 values whose quotient by s lies on a half-integer (as rounded to fp16) or one or
    two fp16 ulps beside it, over the whole int8 range and a little past it."""
    x = ((rng.integers(-130, 130, size=shape) + 0.5) * float(s)).astype(np.float16)
    steps = rng.integers(-2, 3, size=shape).astype(np.int16)
    return (x.view(np.int16) + steps).view(np.float16)


@pytest.mark.parametrize("scale", [0.37, 0.021, 1.0 / 3.0, 7.77e-3, 0.5, 1.7e-5])
def test_quantizer_near_half_integers_bit_exact(scale):
    """The write kernels quantise by a reciprocal multiply where that provably rounds like the
    division, and divide elsewhere. Values placed on and beside the half-integer boundaries of
    fixed scales, through the token writes and the prefill scatter: bit-exact with the
    oracle's division."""
    s = np.float32(scale)
    rng = np.random.default_rng(int(scale * 1e7) + 1)
    KVH, L = 2, 48
    k = _near_half_integers(rng, (2, L, KVH, 128), s)
    v = _near_half_integers(rng, (2, L, KVH, 128), s)
    ts = torch.tensor(s, device="cuda")
    # Token writes.
    rows_k, rows_v = k.reshape(-1, KVH, 128), v.reshape(-1, KVH, 128)
    slots = np.arange(rows_k.shape[0], dtype=np.int32)
    nb = rows_k.shape[0] // 16
    kc, vc, ks, vs = _caches(nb, KVH)
    tk, tv = to_cuda(rows_k, rows_v)
    _ops().quantize_into_cache(tk, tv, kc, vc, ks, vs, torch.from_numpy(slots).cuda(), 16,
                               k_scale=ts, v_scale=ts)
    okc, ovc, oks, ovs = _oracle_rows(rows_k, rows_v, slots, nb, KVH, 16, "f16", s, s)
    assert _bits_equal(kc, okc) and _bits_equal(vc, ovc)
    # Prefill scatter of the same rows (two sequences of 48 and 37 tokens).
    cl = np.array([L, 37], np.int32)
    bt = np.random.default_rng(3).permutation(8).astype(np.int32).reshape(2, 4)
    kc, vc, ks, vs = _caches(8, KVH)
    tk, tv, tbt, tcl = to_cuda(k, v, bt, cl)
    _ops().prefill_into_cache(tk, tv, kc, vc, tbt, tcl, 16, k_scales=ks, v_scales=vs,
                              k_scale=ts, v_scale=ts)
    kq = pa_oracle.quantize_with_scale(k.astype(np.float32), s)
    vq = pa_oracle.quantize_with_scale(v.astype(np.float32), s)
    okc, ovc = pa_oracle.scatter_paged_cache(kq, vq, cl, bt, 8, 16)
    assert np.array_equal(kc.cpu().numpy().view(np.uint8), okc.view(np.uint8))
    assert np.array_equal(vc.cpu().numpy().view(np.uint8), ovc.view(np.uint8))
    sc = np.full((2, L, KVH), s, np.float32)
    assert _bits_equal(ks, pa_oracle.scatter_scales(sc, cl, bt, 8, KVH, 16))


def test_prefill_many_short_sequences_bit_exact():
    """More sequences than the prefill kernel stages lengths for in shared memory (1024),
    lengths 0-40 (empty sequences write nothing), block size 32: bit-exact with the oracle."""
    S, KVH, bs = 1100, 1, 32
    rng = np.random.default_rng(41)
    cl = rng.integers(0, 41, size=S).astype(np.int32)
    mb = 2
    L = int(cl.max())
    nb = S * mb
    bt = rng.permutation(nb).astype(np.int32).reshape(S, mb)
    k = rng.standard_normal((S, L, KVH, 128)).astype(np.float16)
    v = rng.standard_normal((S, L, KVH, 128)).astype(np.float16)
    kc, vc, ks, vs = _caches(nb, KVH, bs)
    tk, tv, tbt, tcl = to_cuda(k, v, bt, cl)
    _ops().prefill_into_cache(tk, tv, kc, vc, tbt, tcl, bs, k_scales=ks, v_scales=vs)
    kq, ksc = pa_oracle.quantize_per_token(k, "f16")
    vq, vsc = pa_oracle.quantize_per_token(v, "f16")
    okc, ovc = pa_oracle.scatter_paged_cache(kq, vq, cl, bt, nb, bs)
    assert np.array_equal(kc.cpu().numpy().view(np.uint8), okc.view(np.uint8))
    assert np.array_equal(vc.cpu().numpy().view(np.uint8), ovc.view(np.uint8))
    assert _bits_equal(ks, pa_oracle.scatter_scales(ksc, cl, bt, nb, KVH, bs))
    assert _bits_equal(vs, pa_oracle.scatter_scales(vsc, cl, bt, nb, KVH, bs))


@pytest.mark.parametrize("source", ["golden16", "golden32", "goldenbf16"])
@pytest.mark.parametrize("int8", [True, False])
def test_prefill_input_dtypes_bit_exact(source, int8):
    """The prefill scatter with fp16, fp32 and bf16 input rows (the golden rows of the
    reference quantiser), block size 32, into INT8 and FP16 caches: bit-exact with the oracle
    (the FP16 cache gets the rows rounded to fp16)."""
    gold = np.load(os.path.join(GOLD, "quant_rows.npz"))
    if source == "golden16":
        x, dtype, tdt = gold["x16"].astype(np.float32), "f16", torch.float16
    elif source == "golden32":
        x, dtype, tdt = gold["x32"], "f32", torch.float32
    else:
        x = (gold["xbf16_bits"].astype(np.uint32) << 16).view(np.float32)
        dtype, tdt = "bf16", torch.bfloat16
    S, KVH, bs = 2, 2, 32
    L = x.shape[0] // (S * KVH)
    k = np.ascontiguousarray(x[:S * L * KVH].reshape(S, L, KVH, 128))
    v = np.ascontiguousarray(k[:, ::-1])
    cl = np.array([L, L - 5], np.int32)
    mb = (L + bs - 1) // bs
    nb = S * mb + 2
    bt = np.random.default_rng(7).permutation(nb)[:S * mb].astype(np.int32).reshape(S, mb)
    kc, vc, ks, vs = _caches(nb, KVH, bs, int8)
    tk = torch.from_numpy(k).to(tdt).cuda()
    tv = torch.from_numpy(v).to(tdt).cuda()
    tbt, tcl = to_cuda(bt, cl)
    kw = dict(k_scales=ks, v_scales=vs) if int8 else {}
    _ops().prefill_into_cache(tk, tv, kc, vc, tbt, tcl, bs, **kw)
    if int8:
        kq, ksc = pa_oracle.quantize_per_token(k, dtype)
        vq, vsc = pa_oracle.quantize_per_token(v, dtype)
        okc, ovc = pa_oracle.scatter_paged_cache(kq, vq, cl, bt, nb, bs)
        assert _bits_equal(ks, pa_oracle.scatter_scales(ksc, cl, bt, nb, KVH, bs))
        assert _bits_equal(vs, pa_oracle.scatter_scales(vsc, cl, bt, nb, KVH, bs))
    else:
        okc, ovc = pa_oracle.scatter_paged_cache(k.astype(np.float16), v.astype(np.float16), cl,
                                                 bt, nb, bs)
    assert np.array_equal(kc.cpu().numpy().view(np.uint8), okc.view(np.uint8))
    assert np.array_equal(vc.cpu().numpy().view(np.uint8), ovc.view(np.uint8))


@pytest.mark.parametrize("kind", ["i8", "fp8", "f16"])
def test_large_token_write_bit_exact(kind):
    """A large token-granular write (1.32 M rows: 330,000 tokens x 2 kv heads x K and V, a
    grid of 165,000 CTAs) in a shuffled slot order with padding tokens, bit-exact with the
    oracle for INT8 (values and scales), FP8 (e4m3 bytes and scales) and the FP16 copy."""
    N, KVH, bs = 330_000, 2, 16
    g = gen.Gen(41)
    k = gen.kv_values(g, (N, KVH, 128), "lognormal_outlier").astype(np.float16)
    v = gen.kv_values(g, (N, KVH, 128), "normal").astype(np.float16)
    nb = (N + bs - 1) // bs + 5
    slots = gen.Gen(42).permutation(nb * bs)[:N].astype(np.int32)
    slots[::977] = -1  # padding tokens: skipped
    dt = {"i8": torch.int8, "fp8": torch.float8_e4m3fn, "f16": torch.float16}[kind]
    kc = torch.zeros(nb, KVH, 16, bs, 8, dtype=torch.uint8 if kind == "fp8" else dt,
                     device="cuda")
    vc = torch.zeros(nb, KVH, 128, bs, dtype=kc.dtype, device="cuda")
    if kind == "fp8":
        kc, vc = kc.view(dt), vc.view(dt)
    ks = torch.zeros(nb, KVH, bs, dtype=torch.float32, device="cuda")
    vs = torch.zeros_like(ks)
    tk, tv, ts = to_cuda(k, v, slots)
    if kind == "f16":
        _ops().write_into_cache(tk, tv, kc, vc, ts, bs)
        kq, vq = k, v
    else:
        _ops().quantize_into_cache(tk, tv, kc, vc, ks, vs, ts, bs)
        if kind == "i8":
            kq, ksc = pa_oracle.quantize_per_token(k, "f16")
            vq, vsc = pa_oracle.quantize_per_token(v, "f16")
        else:
            kq, ksc = pa_oracle.quantize_per_token_fp8(k)
            vq, vsc = pa_oracle.quantize_per_token_fp8(v)
    _ops().check_status(tk.device)
    m = slots >= 0
    blk, off = slots[m] // bs, slots[m] % bs
    okc = np.zeros((nb, KVH, 16, bs, 8), kq.dtype)
    ovc = np.zeros((nb, KVH, 128, bs), vq.dtype)
    okc[blk, :, :, off, :] = kq[m].reshape(-1, KVH, 16, 8)
    ovc[blk, :, :, off] = vq[m]
    u = np.uint16 if kind == "f16" else np.uint8
    assert np.array_equal(kc.view(torch.uint8).cpu().numpy().view(u), okc.view(u))
    assert np.array_equal(vc.view(torch.uint8).cpu().numpy().view(u), ovc.view(u))
    if kind != "f16":
        oks = np.zeros((nb, KVH, bs), np.float32)
        ovs = np.zeros((nb, KVH, bs), np.float32)
        oks[blk, :, off] = ksc[m]
        ovs[blk, :, off] = vsc[m]
        assert _bits_equal(ks, oks) and _bits_equal(vs, ovs)


def _prefill_slots(rng, S, bs, nb_extra=3, pad_every=0):
    """Slots of a flattened prefill batch: S sequences of random lengths, some continuing at a
    position inside a block (chunked prefill), each through its own shuffled block table, with
    padding tokens (-1) between some sequences. Returns (slots, num_blocks)."""
    lens = rng.integers(1, 700, S)
    starts = np.where(rng.random(S) < 0.4, rng.integers(0, 3 * bs, S), 0)
    nblk = [(st + ln + bs - 1) // bs for st, ln in zip(starts, lens)]
    nb = int(sum(nblk)) + nb_extra
    perm = rng.permutation(nb).astype(np.int64)
    out, used = [], 0
    for st, ln, m in zip(starts, lens, nblk):
        bt = perm[used:used + m]
        used += m
        p = np.arange(st, st + ln)
        out.append((bt[p // bs] * bs + p % bs).astype(np.int32))
        if rng.random() < 0.3:
            out.append(np.full(rng.integers(1, 5), -1, np.int32))
    return np.concatenate(out), nb


def _oracle_slots(k, v, slots, nb, KVH, bs, kind, in_dtype, k_fix=None, v_fix=None):
    """Expected caches (and scales) after the token-granular write of k, v at slots."""
    if kind == "f16":
        kq, vq = k.astype(np.float16), v.astype(np.float16)
        ksc = vsc = None
    elif kind == "fp8":
        kq, ksc = pa_oracle.quantize_per_token_fp8(k)
        vq, vsc = pa_oracle.quantize_per_token_fp8(v)
    elif k_fix is not None:
        kq = pa_oracle.quantize_with_scale(k.astype(np.float32), k_fix)
        vq = pa_oracle.quantize_with_scale(v.astype(np.float32), v_fix)
        ksc = np.full(k.shape[:-1], k_fix, np.float32)
        vsc = np.full(v.shape[:-1], v_fix, np.float32)
    else:
        kq, ksc = pa_oracle.quantize_per_token(k, in_dtype)
        vq, vsc = pa_oracle.quantize_per_token(v, in_dtype)
    m = slots >= 0
    blk, off = slots[m] // bs, slots[m] % bs
    okc = np.zeros((nb, KVH, 16, bs, 8), kq.dtype)
    ovc = np.zeros((nb, KVH, 128, bs), vq.dtype)
    okc[blk, :, :, off, :] = kq[m].reshape(-1, KVH, 16, 8)
    ovc[blk, :, :, off] = vq[m]
    if ksc is None:
        return okc, ovc, None, None
    oks = np.zeros((nb, KVH, bs), np.float32)
    ovs = np.zeros((nb, KVH, bs), np.float32)
    oks[blk, :, off] = ksc[m]
    ovs[blk, :, off] = vsc[m]
    return okc, ovc, oks, ovs


@pytest.mark.parametrize("kind,in_dtype,bs,fixed", [
    ("i8", "f16", 16, False), ("i8", "bf16", 32, False), ("i8", "f32", 16, False),
    ("i8", "f16", 16, True), ("f16", "f16", 16, False), ("f16", "f32", 32, False),
    ("i8", "f16", 8, False), ("fp8", "f16", 16, False), ("fp8", "bf16", 32, False)])
def test_prefill_through_slots_bit_exact(kind, in_dtype, bs, fixed):
    """A prefill batch written through slot_mapping (vLLM-style): tokens of one sequence have
    consecutive slots inside its blocks, so aligned runs of 16 take the grouped page stores
    and the rest (sequence ends, chunked-prefill starts inside a block, block size 8) the
    row path. Values and scales bit-exact with the oracle for int8 (per-token or fixed
    scales), fp8 (e4m3) and fp16 caches, fp16 / bf16 / fp32 input rows."""
    rng = np.random.default_rng(51 + bs)
    slots, nb = _prefill_slots(rng, 60, bs)
    N, KVH = slots.shape[0], 4
    # Large enough for the windowed write (at least 32 of its warps per SM).
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert (N + 15) // 16 * KVH * 2 >= 32 * sms
    g = gen.Gen(52)
    k = gen.kv_values(g, (N, KVH, 128), "lognormal_outlier").astype(np.float32)
    v = gen.kv_values(g, (N, KVH, 128), "normal").astype(np.float32)
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[in_dtype]
    tk = torch.from_numpy(k).to(tdt).cuda()
    tv = torch.from_numpy(v).to(tdt).cuda()
    # The oracle sees the rows as the kernel does: rounded to the input dtype.
    k, v = tk.float().cpu().numpy(), tv.float().cpu().numpy()
    ts = torch.from_numpy(slots).cuda()
    kc, vc, ks, vs = _caches(nb, KVH, bs, int8=(kind != "f16"))
    if kind == "fp8":
        kc, vc = kc.view(torch.float8_e4m3fn), vc.view(torch.float8_e4m3fn)
    kfix = vfix = None
    if kind == "f16":
        _ops().write_into_cache(tk, tv, kc, vc, ts, bs)
    elif fixed:
        kfix, vfix = np.float32(0.093), np.float32(0.021)
        _ops().quantize_into_cache(tk, tv, kc, vc, ks, vs, ts, bs,
                                   k_scale=torch.tensor(kfix, device="cuda"),
                                   v_scale=torch.tensor(vfix, device="cuda"))
    else:
        _ops().quantize_into_cache(tk, tv, kc, vc, ks, vs, ts, bs)
    _ops().check_status(tk.device)
    okc, ovc, oks, ovs = _oracle_slots(k, v, slots, nb, KVH, bs, kind, in_dtype, kfix, vfix)
    u = np.uint16 if kind == "f16" else np.uint8
    kb, vb = (kc.view(torch.uint8), vc.view(torch.uint8)) if kind == "fp8" else (kc, vc)
    assert np.array_equal(kb.cpu().numpy().view(u), okc.view(u))
    assert np.array_equal(vb.cpu().numpy().view(u), ovc.view(u))
    if oks is not None:
        assert _bits_equal(ks, oks) and _bits_equal(vs, ovs)
