"""GPU: the bridge's decode loop on this library's cache and ops.

The reference bridge (benchmarks/int8_bridge/qwen_paged_attn.py:39-74) routes a model's
attention through a PagedKVCache: on the prompt it calls cache.prefill(layer, k, v); on each
generated token it calls cache.decode_append(layer, k, v) and then the split-K op
(VARIANTS["splitk"] or VARIANTS_INT8["splitk_int8"]) with cache.context_lens(layer) and the
cache's shared block table. This test drives that same call sequence on pa_b200.PagedKVCache
(its drop-in) for several layers, one prompt and several decode tokens, with random post-RoPE
q/k/v in place of a model, and compares every decode output with the oracle on the rows
written so far (INT8 through the oracle's quantiser and dequantize_kv).
"""

import math

import numpy as np
import pytest
import torch

import pa_oracle
from pa_testlib import ATOL, RTOL

pytestmark = pytest.mark.gpu

KVH, H, D, BS = 2, 12, 128, 16  # Qwen2.5-1.5B geometry: 12 q heads, 2 kv heads


def _oracle_out(oc, q):
    """Oracle decode of q [H, D] over the oracle cache's rows so far (the restated bridge
    cache, pinned bit-exact to the reference's PagedKVCache by the golden fixtures)."""
    kc, vc = oc.k_cache, oc.v_cache
    if oc.is_int8:
        kc, vc = pa_oracle.dequantize_kv(kc, vc, oc.k_scales, oc.v_scales)
    bt = np.arange(oc.num_blocks, dtype=np.int32)[None]
    return pa_oracle.paged_decode_attention(q[None], kc, vc, bt,
                                            np.array([oc.length], np.int32),
                                            scale=1.0 / math.sqrt(D))[0]


@pytest.mark.parametrize("variant", ["fp16", "int8_per_token", "int8_per_tensor"])
def test_bridge_decode_loop(variant):
    from pa_b200 import cuda_ext
    from pa_b200.paged_cache import PagedKVCache
    layers, prompt, steps = 3, 45, 24
    cache = PagedKVCache(num_layers=layers, num_kv_heads=KVH, head_dim=D,
                         max_len=prompt + steps, block_size=BS, variant=variant)
    rng = np.random.default_rng(11)
    oracles = [pa_oracle.BridgeCacheOracle(KVH, D, prompt + steps, BS, variant=variant)
               for _ in range(layers)]
    scale = 1.0 / math.sqrt(D)
    for layer in range(layers):
        k = rng.standard_normal((prompt, KVH, D), dtype=np.float32).astype(np.float16)
        v = rng.standard_normal((prompt, KVH, D), dtype=np.float32).astype(np.float16)
        cache.prefill(layer, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
        oracles[layer].prefill(k, v)
    for t in range(steps):
        for layer in range(layers):
            k1 = rng.standard_normal((KVH, D), dtype=np.float32).astype(np.float16)
            v1 = rng.standard_normal((KVH, D), dtype=np.float32).astype(np.float16)
            q = rng.standard_normal((1, H, D), dtype=np.float32).astype(np.float16)
            n = cache.decode_append(layer, torch.from_numpy(k1).cuda(),
                                    torch.from_numpy(v1).cuda())
            assert n == prompt + t + 1 == oracles[layer].decode_append(k1, v1)
            qd = torch.from_numpy(q).cuda()
            out = torch.empty_like(qd)
            ctx = cache.context_lens(layer)
            if cache.is_int8:
                cuda_ext.VARIANTS_INT8["splitk_int8"](
                    out, qd, cache.k_cache[layer], cache.v_cache[layer], cache.k_scales[layer],
                    cache.v_scales[layer], cache.block_table, ctx, scale, cache.block_size)
            else:
                cuda_ext.VARIANTS["splitk"](out, qd, cache.k_cache[layer], cache.v_cache[layer],
                                            cache.block_table, ctx, scale, cache.block_size)
            ref = _oracle_out(oracles[layer], q[0])
            torch.testing.assert_close(out[0].float().cpu(), torch.from_numpy(ref), atol=ATOL,
                                       rtol=RTOL)
