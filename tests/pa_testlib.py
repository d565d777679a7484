"""Shared helpers for the parity tests: seeded inputs (oracle/gen.py), the numpy oracle, and
torch tensors on the GPU built from the same host arrays."""

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


def fp16_case(seed, num_seqs, num_heads, num_kv_heads, lens, block_size=BLOCK_SIZE,
              dist="normal", extra_blocks=1, max_blocks=None):
    need = sum((c + block_size - 1) // block_size for c in lens)
    c = gen.decode_case(seed, num_seqs, num_heads, num_kv_heads, lens, block_size=block_size,
                        num_blocks=need + extra_blocks, dist=dist, max_blocks=max_blocks)
    kc, vc = pa_oracle.scatter_paged_cache(c["k"], c["v"], c["context_lens"], c["block_table"],
                                           c["num_blocks"], block_size)
    c["k_cache"], c["v_cache"] = kc, vc
    return c


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
