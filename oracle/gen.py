"""Deterministic synthetic inputs for parity tests and fixtures -- TEST INFRASTRUCTURE ONLY.

A counter-based splitmix64 stream with Irwin-Hall normals (sum of 12 uniforms minus 6) uses
only integer arithmetic and exact float64 sums, so the same seed gives the same fp16 tensors
on any machine and numpy version. (The lognormal magnitudes use np.exp; fixtures store a
hash of their inputs so any drift is reported instead of silently changing the oracle.)

Shapes and value distributions follow BASELINE.json's configs: N(0,1) q/K/V, or the INT8
stress distribution "row = N(0,1) x LogNormal(0, 0.5) per (token, kv-head), with outlier
channels x20" (one seeded channel per kv-head, since 1% of 128 channels is 1.28).
"""

import hashlib

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _mix(z):
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


class Gen:
    """Counter-based generator: every draw consumes a fresh range of counters."""

    def __init__(self, seed):
        with np.errstate(over="ignore"):
            self.key = _mix(np.uint64(seed) * _GOLDEN + np.uint64(0x1234567))
        self.ctr = 0

    def _bits(self, n):
        with np.errstate(over="ignore"):
            idx = np.arange(self.ctr, self.ctr + n, dtype=np.uint64)
            self.ctr += n
            return _mix(self.key + idx * _GOLDEN)

    def uniform(self, shape):
        n = int(np.prod(shape)) if shape else 1
        u = (self._bits(n) >> np.uint64(40)).astype(np.float64) / float(1 << 24)
        return u.reshape(shape)

    def normal(self, shape):
        n = int(np.prod(shape)) if shape else 1
        u = self.uniform((n, 12))
        return (u.sum(axis=1) - 6.0).reshape(shape)

    def randint(self, lo, hi, shape):
        return (lo + np.floor(self.uniform(shape) * (hi - lo))).astype(np.int64)

    def permutation(self, n):
        return np.argsort(self.uniform((n,)), kind="stable")


def kv_values(g, shape, dist):
    """K or V values [..., kv_heads, D] as float32 (callers round to their dtype)."""
    x = g.normal(shape)
    if dist == "normal":
        return x.astype(np.float32)
    if dist == "lognormal_outlier":
        mag = np.exp(0.5 * g.normal(shape[:-1]))[..., None]
        x = x * mag
        kvh, d = shape[-2], shape[-1]
        ch = g.randint(0, d, (kvh,))
        for h in range(kvh):
            x[..., h, ch[h]] *= 20.0
        return x.astype(np.float32)
    raise ValueError(dist)


def block_table_for(g, context_lens, num_blocks, block_size=16, max_blocks=None):
    """Distinct physical blocks per sequence from a seeded permutation of the pool; unused
    entries are 0, as in the reference builder (paged_decode_attn.py:82)."""
    nblk = [(int(c) + block_size - 1) // block_size for c in context_lens]
    mb = max(max(nblk), 1) if max_blocks is None else max_blocks
    assert sum(nblk) <= num_blocks, "block pool too small"
    perm = g.permutation(num_blocks)
    bt = np.zeros((len(context_lens), mb), dtype=np.int32)
    nxt = 0
    for b, n in enumerate(nblk):
        bt[b, :n] = perm[nxt:nxt + n]
        nxt += n
    return bt


def decode_case(seed, num_seqs, num_heads, num_kv_heads, context_lens, head_dim=128,
                block_size=16, num_blocks=None, dist="normal", max_blocks=None):
    """q fp16 [S, H, D]; contiguous k, v fp16 [S, Lmax, KVH, D]; int32 lens and table."""
    g = Gen(seed)
    lens = np.asarray(context_lens, dtype=np.int32)
    Lmax = max(int(lens.max()), 1)
    q = g.normal((num_seqs, num_heads, head_dim)).astype(np.float16)
    k = kv_values(g, (num_seqs, Lmax, num_kv_heads, head_dim), dist).astype(np.float16)
    v = kv_values(g, (num_seqs, Lmax, num_kv_heads, head_dim), dist).astype(np.float16)
    need = sum((int(c) + block_size - 1) // block_size for c in lens)
    nb = num_blocks if num_blocks is not None else need + 1
    bt = block_table_for(g, lens, nb, block_size, max_blocks)
    return dict(q=q, k=k, v=v, context_lens=lens, block_table=bt, num_blocks=nb)


def sha256_arrays(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()
