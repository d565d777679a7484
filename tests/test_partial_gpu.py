"""GPU: per-range partials + LSE merge (the cross-GPU split-K path) emulated on one GPU.

Each emulated rank owns a block-aligned token range of every sequence; its block table row
lists only its blocks and its context length is the range length (0 allowed). Merging the
ranks' partials must equal the one-pass decode over the whole context."""

import numpy as np
import pytest
import torch

import pa_oracle
from pa_testlib import assert_close, fp16_case, int8_case, scale_for, to_cuda

pytestmark = pytest.mark.gpu


def _rank_views(bt, lens, parts, bs=16):
    """Per rank: (block_table, context_lens) covering a block-aligned share of each seq."""
    S = len(lens)
    views = []
    for p in range(parts):
        tbl = np.zeros_like(bt)
        cl = np.zeros(S, np.int32)
        for b in range(S):
            nblk = (int(lens[b]) + bs - 1) // bs
            lo = (nblk * p) // parts
            hi = (nblk * (p + 1)) // parts
            tbl[b, :hi - lo] = bt[b, lo:hi]
            t_lo, t_hi = lo * bs, min(hi * bs, int(lens[b]))
            cl[b] = max(0, t_hi - t_lo)
        views.append((tbl, cl))
    return views


@pytest.mark.parametrize("parts", [1, 2, 3, 8])
@pytest.mark.parametrize("kind", ["fp16", "int8"])
@pytest.mark.parametrize("num_heads,num_kv_heads", [(64, 8), (8, 2), (32, 1)])
def test_partials_merge_to_full_decode(parts, kind, num_heads, num_kv_heads):
    from pa_b200 import ops
    lens = [3000, 40, 1, 777]
    c = fp16_case(21, 4, num_heads, num_kv_heads, lens)
    q = to_cuda(c["q"])[0]
    if kind == "fp16":
        kc, vc = to_cuda(c["k_cache"], c["v_cache"])
        ks = vs = None
        kd, vd = c["k_cache"], c["v_cache"]
    else:
        qc = int8_case(c, "per_token")
        kc, vc, ks, vs = to_cuda(qc["k_cache"], qc["v_cache"], qc["k_scales"], qc["v_scales"])
        kd, vd = pa_oracle.dequantize_kv(qc["k_cache"], qc["v_cache"], qc["k_scales"],
                                         qc["v_scales"])
    ps = []
    for tbl, cl in _rank_views(c["block_table"], c["context_lens"], parts):
        tb, tc = to_cuda(tbl, cl)
        ps.append(ops.decode_partial(q, kc, vc, tb, tc, scale_for(), 16, k_scales=ks,
                                     v_scales=vs))
    stacked = torch.stack(ps).contiguous()
    out = torch.empty_like(q)
    ops.merge_partials(out, stacked, num_heads, num_kv_heads)
    ref = pa_oracle.paged_decode_attention(c["q"], kd, vd, c["block_table"], c["context_lens"])
    assert_close(out, ref)
