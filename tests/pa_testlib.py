"""Shared helpers for the parity tests: seeded inputs (oracle/gen.py), the numpy oracle, and
torch tensors on the GPU built from the same host arrays."""

import collections
import math

import numpy as np

import gen
import pa_oracle

HEAD_DIM = 128
BLOCK_SIZE = 16
# North-star tolerance for the attention output (fp32 accumulate, fp16 output).
ATOL = 2e-3
RTOL = 1e-2


def make_lens(clen, num_seqs):
    """Per-sequence context lengths varied inside a batch, as the reference tests do
    (tests/test_paged_decode_attn.py:25-28)."""
    return [max(1, clen - 5 * b) for b in range(num_seqs)]


_CASES = collections.OrderedDict()  # recent fp16_case results (the variant names share cases)
_CASES_MAX = 24


def fp16_case(seed, num_seqs, num_heads, num_kv_heads, lens, block_size=BLOCK_SIZE,
              dist="normal", extra_blocks=1, max_blocks=None):
    """gen.decode_case plus its fp16 paged cache. Recent cases are kept and handed out as
    fresh copies, so callers may modify what they get."""
    key = (seed, num_seqs, num_heads, num_kv_heads, tuple(int(n) for n in lens), block_size,
           dist, extra_blocks, max_blocks)
    c = _CASES.get(key)
    if c is None:
        need = sum((int(n) + block_size - 1) // block_size for n in lens)
        c = gen.decode_case(seed, num_seqs, num_heads, num_kv_heads, lens,
                            block_size=block_size, num_blocks=need + extra_blocks, dist=dist,
                            max_blocks=max_blocks)
        c["k_cache"], c["v_cache"] = pa_oracle.scatter_paged_cache(
            c["k"], c["v"], c["context_lens"], c["block_table"], c["num_blocks"], block_size)
        _CASES[key] = c
        if len(_CASES) > _CASES_MAX:
            _CASES.popitem(last=False)
    else:
        _CASES.move_to_end(key)
    return {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in c.items()}


def int8_case(c, mode, block_size=BLOCK_SIZE):
    """Quantise the contiguous K/V of a case with the oracle and scatter it (the reference
    builder build_paged_kv_cache_int8, tests/paged_decode_attn.py:124-199)."""
    k, v, lens, bt, nb = c["k"], c["v"], c["context_lens"], c["block_table"], c["num_blocks"]
    KVH = k.shape[2]
    if mode == "per_token":
        kq, ks = pa_oracle.quantize_per_token(k, "f16")
        vq, vs = pa_oracle.quantize_per_token(v, "f16")
    else:
        # per-tensor over the valid tokens only would differ from the reference builder,
        # which quantises the whole [S, L, H, D] tensor; do the same.
        kq, s1 = pa_oracle.quantize_per_tensor(k, "f16")
        vq, s2 = pa_oracle.quantize_per_tensor(v, "f16")
        ks = np.full(k.shape[:-1], s1, dtype=np.float32)
        vs = np.full(v.shape[:-1], s2, dtype=np.float32)
    kc, vc = pa_oracle.scatter_paged_cache(kq, vq, lens, bt, nb, block_size)
    kss = pa_oracle.scatter_scales(ks, lens, bt, nb, KVH, block_size)
    vss = pa_oracle.scatter_scales(vs, lens, bt, nb, KVH, block_size)
    return dict(k_cache=kc, v_cache=vc, k_scales=kss, v_scales=vss)


def _rows(rng, n, kvh, d, dist, outlier_ch):
    """K or V rows [n, kvh, d]: N(0,1), or for "lognormal_outlier" each (token, kv-head) row
    scaled by LogNormal(0, 0.5) and one fixed channel per kv-head x20 (oracle/gen.py's
    stress distribution)."""
    x = rng.standard_normal((n, kvh, d), dtype=np.float32)
    if dist == "lognormal_outlier":
        x *= np.exp(0.5 * rng.standard_normal((n, kvh, 1), dtype=np.float32))
        x[:, np.arange(kvh), outlier_ch] *= 20.0
    elif dist != "normal":
        raise ValueError(dist)
    return x.astype(np.float16)


def ragged_case(seed, num_heads, num_kv_heads, lens, block_size=BLOCK_SIZE, dist="normal"):
    """A large ragged batch drawn token by token: fp16 q/K/V from numpy's seeded generator,
    only for the valid tokens of each sequence, scattered straight into the paged cache (no
    [num_seqs, max_len] padding, which for long-tailed lengths is most of the memory). Also
    returns the fp16 rows per sequence for the INT8 variant (ragged_int8)."""
    rng = np.random.default_rng(seed)
    lens = np.asarray(lens, dtype=np.int32)
    S, H, KVH, D = len(lens), num_heads, num_kv_heads, HEAD_DIM
    nb = sum((int(n) + block_size - 1) // block_size for n in lens) + 1
    bt = gen.block_table_for(gen.Gen(seed), lens, nb, block_size)
    q = rng.standard_normal((S, H, D), dtype=np.float32).astype(np.float16)
    kc = np.zeros((nb, KVH, D // 8, block_size, 8), np.float16)
    vc = np.zeros((nb, KVH, D, block_size), np.float16)
    rows = []
    ch_k, ch_v = rng.integers(0, D, KVH), rng.integers(0, D, KVH)
    for b, n in enumerate(lens):
        k = _rows(rng, int(n), KVH, D, dist, ch_k)
        v = _rows(rng, int(n), KVH, D, dist, ch_v)
        t = np.arange(int(n))
        blk, off = bt[b, t // block_size], t % block_size
        kc[blk, :, :, off, :] = k.reshape(int(n), KVH, D // 8, 8)
        vc[blk, :, :, off] = v
        rows.append((k, v))
    return dict(q=q, k_cache=kc, v_cache=vc, block_table=bt, context_lens=lens, num_blocks=nb,
                rows=rows)


def ragged_int8(c, block_size=BLOCK_SIZE):
    """Per-token INT8 cache of a ragged_case, quantised row by row with the oracle."""
    nb, bt = c["num_blocks"], c["block_table"]
    KVH, D = c["k_cache"].shape[1], HEAD_DIM
    kc = np.zeros((nb, KVH, D // 8, block_size, 8), np.int8)
    vc = np.zeros((nb, KVH, D, block_size), np.int8)
    ks = np.zeros((nb, KVH, block_size), np.float32)
    vs = np.zeros((nb, KVH, block_size), np.float32)
    for b, (k, v) in enumerate(c["rows"]):
        n = k.shape[0]
        kq, ksc = pa_oracle.quantize_per_token(k, "f16")
        vq, vsc = pa_oracle.quantize_per_token(v, "f16")
        t = np.arange(n)
        blk, off = bt[b, t // block_size], t % block_size
        kc[blk, :, :, off, :] = kq.reshape(n, KVH, D // 8, 8)
        vc[blk, :, :, off] = vq
        ks[blk, :, off] = ksc
        vs[blk, :, off] = vsc
    return dict(k_cache=kc, v_cache=vc, k_scales=ks, v_scales=vs)


def oracle_out(q, k_cache, v_cache, bt, lens, scale=None):
    return pa_oracle.paged_decode_attention(q, k_cache, v_cache, bt, lens, scale=scale)


def to_cuda(*arrays):
    import torch
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrays]


def assert_close(out, ref, atol=ATOL, rtol=RTOL):
    import torch
    out = out.float().cpu() if hasattr(out, "cpu") else torch.from_numpy(out)
    ref = torch.from_numpy(np.asarray(ref, dtype=np.float32))
    torch.testing.assert_close(out, ref, atol=atol, rtol=rtol)


def scale_for(head_dim=HEAD_DIM):
    return 1.0 / math.sqrt(head_dim)
