"""GPU: the decode step (ops.decode_step / pa_decode_step): append each sequence's new token to
the cache and decode, in one call.

The fused form (the decode kernel writes each new token just before reading its page) must
give bit-identical caches and outputs to the two-kernel form (write kernel, then decode), and
both must equal the reference's sequence: the token written like quantize_per_token /
decode_append (bit-exact cache bytes and scales, checked against the separate write op, which
is pinned to the oracle) and the decode of the oracle over the updated cache. Covered: INT8
per-token and per-tensor, FP16 and FP8 caches; fp16, bf16 and fp32 rows; single-pass and
split-K; block sizes 16 and 32; ragged batches whose new tokens open a new block, share a block
with older tokens, or sit mid-page; groups of more than 16 q heads per kv head (written by the
separate kernel); a bad block id (flagged, nothing written); and a CUDA-graph-captured loop of
steps with the lengths advanced on the device.
"""

import math

import numpy as np
import pytest
import torch

import pa_oracle
from pa_testlib import ATOL, RTOL

pytestmark = pytest.mark.gpu

D = 128
SCALE = 1.0 / math.sqrt(D)


def _setup(kind, lens, H, KVH, bs=16, seed=0, per_tensor=False):
    """A cache holding lens[b] - 1 old tokens per sequence (written by prefill), the rows of
    the new token, q, and block tables with room for the new token."""
    from pa_b200 import ops
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    lens = np.asarray(lens, np.int64)
    B = len(lens)
    NB = int(sum((int(c) + bs - 1) // bs for c in lens)) + 7
    perm = torch.randperm(NB, generator=gen, device="cuda").to(torch.int32)
    maxb = int((lens.max() + bs - 1) // bs) + 1
    bt = torch.full((B, maxb), 0, dtype=torch.int32, device="cuda")
    nxt = 0
    for b in range(B):
        n = int((lens[b] + bs - 1) // bs)
        bt[b, :n] = perm[nxt:nxt + n]
        nxt += n
    dt = {"f16": torch.float16, "i8": torch.int8, "f8": torch.float8_e4m3fn}[kind]
    kc = torch.zeros(NB, KVH, D // 8, bs, 8, dtype=dt, device="cuda")
    vc = torch.zeros(NB, KVH, D, bs, dtype=dt, device="cuda")
    ks = vs = None
    if kind != "f16":
        ks = torch.zeros(NB, KVH, bs, dtype=torch.float32, device="cuda")
        vs = torch.zeros_like(ks)
    L = int(lens.max())
    rows_k = (torch.randn(B, L, KVH, D, generator=gen, device="cuda") *
              torch.exp(0.5 * torch.randn(B, L, KVH, 1, generator=gen, device="cuda"))).half()
    rows_v = (torch.randn(B, L, KVH, D, generator=gen, device="cuda") *
              torch.exp(0.5 * torch.randn(B, L, KVH, 1, generator=gen, device="cuda"))).half()
    rows_k[..., 3] *= 20.0
    rows_v[..., 77] *= 20.0
    old = torch.from_numpy((lens - 1).astype(np.int32)).cuda()
    kf = vf = None
    if per_tensor:
        kf = ops.absmax_scale(rows_k).reshape(1).contiguous()
        vf = ops.absmax_scale(rows_v).reshape(1).contiguous()
    if kind == "f8":
        t = torch.arange(L, device="cuda")
        blk = bt.long().gather(1, (t // bs).clamp(max=maxb - 1).expand(B, L))
        slots = torch.where(t[None, :] < old[:, None].long(), blk * bs + t % bs,
                            torch.full_like(blk, -1)).to(torch.int32).reshape(-1)
        ops.quantize_into_cache(rows_k.reshape(-1, KVH, D), rows_v.reshape(-1, KVH, D), kc, vc,
                                ks, vs, slots, bs)
    else:
        ops.prefill_into_cache(rows_k, rows_v, kc, vc, bt, old, bs, k_scales=ks, v_scales=vs,
                               k_scale=kf, v_scale=vf)
    new_k = (torch.randn(B, KVH, D, generator=gen, device="cuda") * 2).half()
    new_v = (torch.randn(B, KVH, D, generator=gen, device="cuda") * 2).half()
    new_k[:, :, 3] *= 20.0
    q = torch.randn(B, H, D, generator=gen, device="cuda").half()
    cl = torch.from_numpy(lens.astype(np.int32)).cuda()
    torch.cuda.synchronize()
    return dict(q=q, bt=bt, cl=cl, kc=kc, vc=vc, ks=ks, vs=vs, new_k=new_k, new_v=new_v,
                kf=kf, vf=vf, bs=bs)


def _clone(c):
    return {k: (v.clone() if torch.is_tensor(v) else v) for k, v in c.items()}


def _step(c, new_k, new_v, fused, splitk=False):
    from pa_b200 import ops
    out = torch.full_like(c["q"], float("nan"))
    ops.decode_step(out, c["q"], new_k, new_v, c["kc"], c["vc"], c["bt"], c["cl"], SCALE,
                    c["bs"], k_scales=c["ks"], v_scales=c["vs"], k_scale=c["kf"],
                    v_scale=c["vf"], splitk=splitk, fused=fused)
    torch.cuda.synchronize()
    ops.check_status()
    return out


def _separate(c, new_k, new_v, splitk=False):
    """The reference sequence with this library's separate ops: write the new tokens
    (quantize_into_cache / write_into_cache at their slots), then decode."""
    from pa_b200 import ops
    bs = c["bs"]
    pos = c["cl"].long() - 1
    slots = (c["bt"].long().gather(1, (pos // bs).view(-1, 1)).view(-1) * bs + pos % bs)
    slots = slots.to(torch.int32)
    if c["kc"].dtype == torch.float16:
        ops.write_into_cache(new_k, new_v, c["kc"], c["vc"], slots, bs)
    else:
        ops.quantize_into_cache(new_k, new_v, c["kc"], c["vc"], c["ks"], c["vs"], slots, bs,
                                k_scale=c["kf"], v_scale=c["vf"])
    out = torch.full_like(c["q"], float("nan"))
    ops.decode(out, c["q"], c["kc"], c["vc"], c["bt"], c["cl"], SCALE, bs, k_scales=c["ks"],
               v_scales=c["vs"], splitk=splitk)
    torch.cuda.synchronize()
    ops.check_status()
    return out


def _oracle(c):
    f8 = c["kc"].dtype == torch.float8_e4m3fn
    kc = (c["kc"].view(torch.uint8) if f8 else c["kc"]).cpu().numpy()
    vc = (c["vc"].view(torch.uint8) if f8 else c["vc"]).cpu().numpy()
    if c["ks"] is not None:
        deq = pa_oracle.dequantize_fp8 if f8 else pa_oracle.dequantize_kv
        kc, vc = deq(kc, vc, c["ks"].cpu().numpy(), c["vs"].cpu().numpy())
    return pa_oracle.paged_decode_attention(c["q"].cpu().numpy(), kc, vc, c["bt"].cpu().numpy(),
                                            c["cl"].cpu().numpy(), scale=SCALE)


def _same_cache(a, b):
    for key in ("kc", "vc", "ks", "vs"):
        if a[key] is None:
            continue
        x, y = a[key], b[key]
        if x.dtype == torch.float8_e4m3fn:
            x, y = x.view(torch.uint8), y.view(torch.uint8)
        if x.dtype == torch.float32:
            x, y = x.view(torch.int32), y.view(torch.int32)
        assert torch.equal(x, y), key


LENS = [1, 16, 17, 33, 300, 1000, 4097, 2, 512, 513]


@pytest.mark.parametrize("kind,per_tensor", [("i8", False), ("i8", True), ("f16", False),
                                             ("f8", False)])
@pytest.mark.parametrize("splitk", [False, True])
@pytest.mark.parametrize("H,KVH", [(12, 2), (32, 8), (28, 4)])
def test_step_fused_equals_separate_and_oracle(kind, per_tensor, splitk, H, KVH):
    c0 = _setup(kind, LENS, H, KVH, seed=H + KVH, per_tensor=per_tensor)
    cf, cu, cs = _clone(c0), _clone(c0), _clone(c0)
    out_f = _step(cf, c0["new_k"], c0["new_v"], fused=True, splitk=splitk)
    out_u = _step(cu, c0["new_k"], c0["new_v"], fused=False, splitk=splitk)
    out_s = _separate(cs, c0["new_k"], c0["new_v"], splitk=splitk)
    _same_cache(cf, cs)
    _same_cache(cu, cs)
    assert torch.equal(out_f, out_u)
    assert torch.equal(out_f, out_s)
    torch.testing.assert_close(out_f.float().cpu(), torch.from_numpy(_oracle(cf)), atol=ATOL,
                               rtol=RTOL)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_step_row_dtypes(dtype):
    c0 = _setup("i8", [40, 7, 1000], 12, 2, seed=5)
    nk, nv = c0["new_k"].to(dtype), c0["new_v"].to(dtype)
    cf, cs = _clone(c0), _clone(c0)
    out_f = _step(cf, nk, nv, fused=True)
    out_s = _separate(cs, nk, nv)
    _same_cache(cf, cs)
    assert torch.equal(out_f, out_s)


def test_step_block_size_32_and_large_groups():
    """block_size 32; 40 q heads per kv head (three head tiles: the separate write kernel)."""
    for H, KVH in ((12, 2), (80, 2)):
        c0 = _setup("i8", [31, 32, 33, 700], H, KVH, bs=32, seed=H)
        cf, cs = _clone(c0), _clone(c0)
        out_f = _step(cf, c0["new_k"], c0["new_v"], fused=True)
        out_s = _separate(cs, c0["new_k"], c0["new_v"])
        _same_cache(cf, cs)
        assert torch.equal(out_f, out_s)
        torch.testing.assert_close(out_f.float().cpu(), torch.from_numpy(_oracle(cf)),
                                   atol=ATOL, rtol=RTOL)


def test_step_bad_block_id_is_flagged_and_not_written():
    from pa_b200 import _lib, ops
    c0 = _setup("i8", [100, 50], 12, 2, seed=9)
    c = _clone(c0)
    nb = c["kc"].shape[0]
    c["bt"][1, (50 - 1) // 16] = nb + 3  # the new token's block is out of range
    before = c["kc"].clone()
    out = torch.empty_like(c["q"])
    ops.decode_step(out, c["q"], c["new_k"], c["new_v"], c["kc"], c["vc"], c["bt"], c["cl"],
                    SCALE, 16, k_scales=c["ks"], v_scales=c["vs"])
    torch.cuda.synchronize()
    assert ops.read_status() & _lib.PA_ERR_BLOCK_ID
    # Sequence 0's token was written, nothing else changed outside its slot.
    changed = (c["kc"] != before).nonzero()
    blk0 = int(c["bt"][0, (100 - 1) // 16])
    assert changed.numel() > 0 and bool((changed[:, 0] == blk0).all())


def test_step_loop_captured_in_a_cuda_graph():
    """Eight steps captured once (lengths advanced on the device between steps, new rows
    refreshed in place) replay to the same caches and outputs as eight eager steps."""
    from pa_b200 import ops
    steps = 8
    lens0 = [70, 16, 1000, 33]
    c0 = _setup("i8", [n + steps for n in lens0], 28, 4, seed=13)
    c0["cl"] -= steps  # start 8 tokens short of the table's room
    gen = torch.Generator(device="cuda")
    gen.manual_seed(3)
    rows = [((torch.randn(4, 4, D, generator=gen, device="cuda")).half(),
             (torch.randn(4, 4, D, generator=gen, device="cuda")).half()) for _ in range(steps)]

    eager = _clone(c0)
    outs = []
    for t in range(steps):
        eager["cl"] += 1
        outs.append(_step(eager, rows[t][0], rows[t][1], fused=True))

    g_in = _clone(c0)
    nk, nv = torch.empty_like(rows[0][0]), torch.empty_like(rows[0][1])
    out = torch.empty_like(c0["q"])
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # one call creates the stream's workspace before capture
        warm = _clone(c0)
        warm["cl"] += 1
        ops.decode_step(out, warm["q"], rows[0][0], rows[0][1], warm["kc"], warm["vc"],
                        warm["bt"], warm["cl"], SCALE, 16, k_scales=warm["ks"],
                        v_scales=warm["vs"], validate=False)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        g_in["cl"].add_(1)
        ops.decode_step(out, g_in["q"], nk, nv, g_in["kc"], g_in["vc"], g_in["bt"], g_in["cl"],
                        SCALE, 16, k_scales=g_in["ks"], v_scales=g_in["vs"], validate=False)
    for t in range(steps):
        nk.copy_(rows[t][0])
        nv.copy_(rows[t][1])
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, outs[t]), t
    _same_cache(g_in, eager)
    assert ops.read_status() == 0


def test_paged_cache_append_and_decode_matches_the_bridge_sequence():
    """PagedKVCache.append_and_decode == decode_append followed by the split-K op."""
    from pa_b200 import cuda_ext
    from pa_b200.paged_cache import PagedKVCache
    for variant in ("fp16", "int8_per_token", "int8_per_tensor"):
        torch.manual_seed(0)
        a = PagedKVCache(2, 2, D, 200, variant=variant)
        b = PagedKVCache(2, 2, D, 200, variant=variant)
        k = torch.randn(60, 2, D, dtype=torch.float16, device="cuda")
        v = torch.randn(60, 2, D, dtype=torch.float16, device="cuda")
        for cache in (a, b):
            cache.prefill(1, k, v)
        for _ in range(5):
            k1 = torch.randn(2, D, dtype=torch.float16, device="cuda")
            v1 = torch.randn(2, D, dtype=torch.float16, device="cuda")
            q = torch.randn(1, 12, D, dtype=torch.float16, device="cuda")
            fused = a.append_and_decode(1, k1, v1, q, SCALE)
            b.decode_append(1, k1, v1)
            ref = torch.empty_like(q)
            if b.is_int8:
                cuda_ext.VARIANTS_INT8["splitk_int8"](ref, q, b.k_cache[1], b.v_cache[1],
                                                      b.k_scales[1], b.v_scales[1],
                                                      b.block_table, b.context_lens(1), SCALE,
                                                      16)
            else:
                cuda_ext.VARIANTS["splitk"](ref, q, b.k_cache[1], b.v_cache[1], b.block_table,
                                            b.context_lens(1), SCALE, 16)
            torch.cuda.synchronize()
            assert torch.equal(fused, ref), variant
        assert torch.equal(a.k_cache, b.k_cache) and torch.equal(a.v_cache, b.v_cache)


def test_decode_plan_matches_decode_and_rejects_other_shapes():
    """ops.DecodePlan: checks once, then run() equals decode() for the plan's tensors and for
    other tensors of the same shapes; different shapes raise."""
    from pa_b200 import ops
    for kind in ("f16", "i8"):
        c = _setup(kind, LENS, 12, 2, seed=21)
        out = torch.empty_like(c["q"])
        plan = ops.DecodePlan(out, c["q"], c["kc"], c["vc"], c["bt"], c["cl"], SCALE, 16,
                              k_scales=c["ks"], v_scales=c["vs"])
        plan.run(host_context_lens=c["cl"].cpu())
        ref = torch.empty_like(out)
        ops.decode(ref, c["q"], c["kc"], c["vc"], c["bt"], c["cl"], SCALE, 16,
                   k_scales=c["ks"], v_scales=c["vs"])
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        q2 = torch.randn_like(c["q"])
        out2 = torch.empty_like(out)
        plan.run(out=out2, q=q2)
        ops.decode(ref, q2, c["kc"], c["vc"], c["bt"], c["cl"], SCALE, 16, k_scales=c["ks"],
                   v_scales=c["vs"])
        torch.cuda.synchronize()
        assert torch.equal(out2, ref)
        with pytest.raises(RuntimeError, match="plan"):
            plan.run(q=q2[:1].contiguous())
        with pytest.raises(RuntimeError, match="context_lens must be >= 1"):
            plan.run(host_context_lens=torch.zeros_like(c["cl"].cpu()))



def test_decode_plans_on_two_streams_overlap_safely():
    """Two DecodePlans driven from two streams, as a double-buffered serving loop does: each
    stream gets its own workspace, so decodes in flight on both streams at once give the same
    bits as the same decodes run one after another on one stream. Each round also uploads the
    inputs from pinned memory and reads the output back on its stream."""
    from pa_b200 import ops
    for kind in ("f16", "i8"):
        c = _setup(kind, LENS, 12, 2, seed=23)
        qs = [torch.randn_like(c["q"]) for _ in range(4)]
        refs = []
        for q in qs:
            r = torch.empty_like(q)
            ops.decode(r, q, c["kc"], c["vc"], c["bt"], c["cl"], SCALE, 16,
                       k_scales=c["ks"], v_scales=c["vs"])
            refs.append(r.cpu())
        streams = [torch.cuda.Stream(), torch.cuda.Stream()]
        dq = [torch.empty_like(c["q"]) for _ in range(2)]
        dout = [torch.empty_like(c["q"]) for _ in range(2)]
        hq = [torch.empty(c["q"].shape, dtype=c["q"].dtype, pin_memory=True) for _ in range(4)]
        hout = [torch.empty(c["q"].shape, dtype=c["q"].dtype, pin_memory=True)
                for _ in range(4)]
        for h, q in zip(hq, qs):
            h.copy_(q.cpu())
        plans = [ops.DecodePlan(dout[i], dq[i], c["kc"], c["vc"], c["bt"], c["cl"], SCALE, 16,
                                k_scales=c["ks"], v_scales=c["vs"]) for i in range(2)]
        host_cl = c["cl"].cpu()
        torch.cuda.synchronize()
        events = [None, None]
        for k in range(4):
            i = k & 1
            if events[i] is not None:
                events[i].synchronize()
            with torch.cuda.stream(streams[i]):
                dq[i].copy_(hq[k], non_blocking=True)
                plans[i].run(host_context_lens=host_cl)
                hout[k].copy_(dout[i], non_blocking=True)
                events[i] = torch.cuda.Event()
                events[i].record()
        torch.cuda.synchronize()
        for k in range(4):
            assert torch.equal(hout[k], refs[k]), (kind, k)
        assert ops.read_status(c["q"].device) == 0
