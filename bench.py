"""Benchmark of the B200 paged-attention decode path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl ours|reference]

Metric: achieved HBM GB/s of a paged-decode step -- algorithmic bytes of KV
(plus per-token scales for INT8/FP8) read per step / step time -- with seqs/s and % of peak.

Headline workload: BASELINE config 2 (FP16, batch 64, context 4096, 32 q / 8 kv heads,
head_dim 128, block 16, shuffled block tables over 16384 blocks). At N GPUs every rank runs
its own config-2 batch (sequence sharding, no communication): weak scaling.

The same run also measures, one after another in this process, and reports under "configs":
  cfg3           INT8 per-token decode + one-token quantize-write per sequence (B64, ctx 8192,
                 12/2 heads, lognormal rows with one x20 outlier channel per kv head)
  cfg3_f16       config 3's shapes with an FP16 cache (the FP16 comparison of config 3)
  cfg3_pt        config 3 with per-tensor INT8 scales (the per-tensor comparison)
  cfg4           long-context split-K INT8 (B8, ctx U[65536,131072], 64/8), kv heads sharded
                 across the ranks (strong scaling)
  cfg4_ctxsplit  config 4 with every sequence's context split across the ranks: per-rank
                 partials, NCCL all-gather, LSE merge (strong scaling)
  cfg5           ragged INT8 serving batch + one-token write (B256, 28/4, ctx lognormal median
                 2048 sigma 1 clipped to [16, 32768]), sequences LPT-sharded (strong scaling)
  cfg6           config 3 with an FP8 (e4m3) cache
and, at one GPU, the cache-write kernels alone ("write_kernels": 512 B read + 264 B written per
(token, kv head)). Every config carries a parity check of its timed output against an fp32
restatement of the reference decode in torch on the device (2e-3 abs + 1e-2 rel), its
roofline and, at one GPU, a CPU baseline. Configs 3/3_f16/3_pt/6 and the write kernels run at
one GPU only. --config NAME measures only that workload (as the headline); --config writes
only the cache-write kernels.

Inputs are synthetic (seeded), larger than L2 (126 MB); timing is CUDA events on the launching
stream around one replay of a CUDA graph of K steps, max over ranks.
--impl reference times the reference algorithm's CPU implementation (the oracle port) on a
bounded sample of the same workload, on this host's cores.
"""

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "cuda-pa-int8_b200"))

HEAD_DIM = 128
BLOCK = 16
METRIC = "paged-decode achieved HBM GB/s (% of B200 peak) and seqs/sec at 1/2/4/8 GPUs"
NOMINAL_GBS = 8000.0
ATOL, RTOL = 2e-3, 1e-2  # north-star tolerance of the attention output

SPECS = {
    "cfg2": dict(B=64, H=32, KVH=8, kv="f16", ctx="fixed", L=4096, NB=16384, step=0,
                 dist="normal", shard="weak",
                 desc="cfg2 FP16 decode B64 ctx4096 32/8 heads"),
    "cfg3": dict(B=64, H=12, KVH=2, kv="i8", ctx="fixed", L=8192, step=1,
                 dist="lognormal_outlier", shard="weak",
                 desc="cfg3 INT8 per-token decode + 1-token quantize-write B64 ctx8192 12/2"),
    "cfg3_f16": dict(B=64, H=12, KVH=2, kv="f16", ctx="fixed", L=8192, step=1,
                     dist="lognormal_outlier", shard="weak",
                     desc="cfg3 shapes, FP16 cache + 1-token fp16 write B64 ctx8192 12/2"),
    "cfg3_pt": dict(B=64, H=12, KVH=2, kv="i8", per_tensor=True, ctx="fixed", L=8192, step=1,
                    dist="lognormal_outlier", shard="weak",
                    desc="cfg3 per-tensor-scale INT8 decode + 1-token write B64 ctx8192 12/2"),
    "cfg4": dict(B=8, H=64, KVH=8, kv="i8", ctx="uniform", L=(65536, 131072), step=0,
                 splitk=True, dist="lognormal_outlier", shard="kvhead",
                 desc="cfg4 INT8 split-K decode B8 ctx U[65536,131072] 64/8 (kv-head sharded)"),
    "cfg4_ctxsplit": dict(B=8, H=64, KVH=8, kv="i8", ctx="uniform", L=(65536, 131072), step=0,
                          dist="lognormal_outlier", shard="context",
                          desc="cfg4 INT8 B8 ctx U[65536,131072] 64/8, context split across "
                               "ranks: partials + NCCL all-gather + LSE merge"),
    "cfg5": dict(B=256, H=28, KVH=4, kv="i8", ctx="lognormal", L=2048, step=1,
                 dist="lognormal_outlier", shard="seq",
                 desc="cfg5 ragged INT8 serving B256 28/4 + 1-token write (sequence sharded)"),
    "cfg6": dict(B=64, H=12, KVH=2, kv="f8", ctx="fixed", L=8192, step=1,
                 dist="lognormal_outlier", shard="weak",
                 desc="cfg6 FP8-e4m3 per-token decode + 1-token quantize-write B64 ctx8192 "
                      "12/2"),
}
SECONDARY_1GPU = ["cfg3", "cfg3_f16", "cfg3_pt", "cfg4", "cfg4_ctxsplit", "cfg5", "cfg6"]
SECONDARY_MULTI = ["cfg4", "cfg4_ctxsplit", "cfg5"]


def scaling_of(name):
    """Configs 4 and 5 split one fixed workload across the ranks (by kv head, context or
    sequence): strong scaling. The others give every rank its own batch: weak scaling."""
    return "weak" if SPECS[name]["shard"] == "weak" else "strong"


def config_name(c):
    c = str(c)
    return c if c.startswith("cfg") else "cfg" + c


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--config", default=None,
                   help="measure only this workload (2..6, a name from SPECS, or 'writes' "
                        "for the cache-write kernels alone)")
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--splitk", action="store_true", help="use the split-K pair")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--soak-ms", type=float, default=1500.0,
                   help="untimed load before the timed region so the clock sampler sees it")
    a = p.parse_args()
    if a.config is not None and a.config != "writes":
        a.config = config_name(a.config)
        if a.config not in SPECS:
            p.error(f"unknown config {a.config}")
    return a


def measured_peak():
    path = os.path.join(HERE, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------------------------------
# Workloads
# ---------------------------------------------------------------------------------------
class Workload:
    """Device-resident paged cache + one step's inputs for one rank."""


def _kv_rows(torch, shape, dist, gen, device):
    """K or V rows [..., kv_heads, head_dim] fp16: N(0,1), or for "lognormal_outlier" each
    (token, kv head) row scaled by LogNormal(0, 0.5) and one seeded channel per kv head x20
    (1% of 128 channels, fixed to one channel per kv head)."""
    x = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
    if dist == "lognormal_outlier":
        mag = torch.exp(0.5 * torch.randn(shape[:-1], generator=gen, device=device))
        x = x * mag.unsqueeze(-1)
        kvh = shape[-2]
        ch = torch.randint(0, shape[-1], (kvh,), generator=gen, device=device)
        x[..., torch.arange(kvh, device=device), ch] *= 20.0
    return x.to(torch.float16)


def _global_lens(spec):
    """Context lengths of the whole batch before the step's new token (seeded)."""
    import numpy as np
    rng = np.random.default_rng(99)
    B = spec["B"]
    if spec["ctx"] == "fixed":
        return np.full(B, spec["L"] - spec["step"], dtype=np.int64)
    if spec["ctx"] == "uniform":
        lo, hi = spec["L"]
        return rng.integers(lo, hi + 1, size=B).astype(np.int64)
    lens = np.clip(np.exp(rng.normal(math.log(spec["L"]), 1.0, size=B)), 16, 32768)
    return lens.astype(np.int64) - spec["step"]


def _seq_rows(torch, spec, b, device):
    """Full K and V rows [L_b, KVH, D] of sequence b of a context-split workload, generated
    from a per-sequence seed so that every rank (and the parity check) sees the same rows."""
    lens = _global_lens(spec)
    g = torch.Generator(device=device)
    g.manual_seed(7000 + b)
    L = int(lens[b])
    k = _kv_rows(torch, (L, spec["KVH"], HEAD_DIM), spec["dist"], g, device)
    v = _kv_rows(torch, (L, spec["KVH"], HEAD_DIM), spec["dist"], g, device)
    return k, v


def _block_table(torch, gen, lens, step, NB, device):
    """Every sequence's blocks from one seeded permutation of the pool (fragmented)."""
    B = len(lens)
    maxb = max(1, int((max(lens) + step + BLOCK - 1) // BLOCK))
    perm = torch.randperm(NB, generator=gen, device=device).to(torch.int32)
    bt = torch.zeros(B, maxb, dtype=torch.int32, device=device)
    nxt = 0
    for b in range(B):
        nb_b = int((lens[b] + step + BLOCK - 1) // BLOCK)
        bt[b, :nb_b] = perm[nxt:nxt + nb_b]
        nxt += nb_b
    return bt


def build_workload(torch, name, rank, world, device):
    import numpy as np
    from pa_b200 import ops, shard
    spec = SPECS[name]
    gen = torch.Generator(device=device)
    gen.manual_seed(1234 + (rank if spec["shard"] == "weak" else 0))
    w = Workload()
    w.name, w.spec = name, spec
    B, H, KVH = spec["B"], spec["H"], spec["KVH"]
    w.kv = spec["kv"]
    w.per_tensor = bool(spec.get("per_tensor"))
    w.splitk = bool(spec.get("splitk"))
    w.step_tokens = spec["step"]
    lens = _global_lens(spec)
    w.seqs_total = B
    parts = None
    if spec["shard"] == "kvhead":
        KVH //= world
        H //= world
    elif spec["shard"] == "seq":
        parts = shard.lpt_partition(lens.tolist(), world)
        lens = lens[parts[rank]]
        B = len(lens)
    elif spec["shard"] == "context":
        w.global_lens = lens
        w.ranges = [shard.token_ranges(int(c), world)[rank] for c in lens]
        lens = np.array([hi - lo for lo, hi in w.ranges], dtype=np.int64)
    NB = spec.get("NB") or int(sum((int(c) + w.step_tokens + BLOCK - 1) // BLOCK
                                   for c in lens)) + 64
    w.B, w.H, w.KVH, w.NB = B, H, KVH, NB
    w.lens_host = (lens + w.step_tokens).astype(np.int32)  # context after the step's write
    bt = _block_table(torch, gen, lens, w.step_tokens, NB, device)
    w.block_table = bt
    w.context_lens = torch.from_numpy(w.lens_host).to(device)
    # q: the same on every rank for the sharded configs (each rank takes its heads).
    qgen = torch.Generator(device=device)
    qgen.manual_seed(4321 + (rank if spec["shard"] == "weak" else 0))
    q = torch.randn(spec["B"], spec["H"], HEAD_DIM, generator=qgen, device=device)
    if spec["shard"] == "kvhead":
        q = q[:, rank * H:(rank + 1) * H]
    elif spec["shard"] == "seq":
        q = q[torch.as_tensor(parts[rank], device=device)]
    w.q = q.to(torch.float16).contiguous()
    w.out = torch.empty_like(w.q)
    fp8 = w.kv == "f8"
    dt = torch.float8_e4m3fn if fp8 else (torch.int8 if w.kv == "i8" else torch.float16)
    w.k_cache = torch.zeros(NB, KVH, HEAD_DIM // 8, BLOCK, 8, dtype=dt, device=device)
    w.v_cache = torch.zeros(NB, KVH, HEAD_DIM, BLOCK, dtype=dt, device=device)
    scaled = w.kv != "f16"
    w.k_scales = (torch.zeros(NB, KVH, BLOCK, dtype=torch.float32, device=device)
                  if scaled else None)
    w.v_scales = torch.zeros_like(w.k_scales) if scaled else None
    w.k_fix = w.v_fix = None

    def fill(k, v, bt_rows, lens_rows):
        """Write contiguous rows [S, L, KVH, D] of some sequences through the library's own
        cache-write kernels."""
        if fp8:
            S, L = k.shape[0], k.shape[1]
            t = torch.arange(L, device=device)
            lens_c = torch.as_tensor(np.asarray(lens_rows), device=device).long()
            blk = bt_rows.long().gather(1, (t // BLOCK).expand(S, L))
            slots = torch.where(t[None, :] < lens_c[:, None], blk * BLOCK + t % BLOCK,
                                torch.full_like(blk, -1)).to(torch.int32).reshape(-1)
            ops.quantize_into_cache(k.reshape(-1, KVH, HEAD_DIM), v.reshape(-1, KVH, HEAD_DIM),
                                    w.k_cache, w.v_cache, w.k_scales, w.v_scales, slots, BLOCK)
        else:
            ops.prefill_into_cache(k, v, w.k_cache, w.v_cache, bt_rows.contiguous(),
                                   torch.as_tensor(np.asarray(lens_rows), dtype=torch.int32,
                                                   device=device),
                                   BLOCK, k_scales=w.k_scales, v_scales=w.v_scales,
                                   k_scale=w.k_fix, v_scale=w.v_fix)

    if spec["shard"] == "context":
        # Each rank writes its token range of every sequence's (shared, seeded) rows.
        for b in range(B):
            lo, hi = w.ranges[b]
            if hi <= lo:
                continue
            k, v = _seq_rows(torch, spec, b, device)
            fill(k[lo:hi].unsqueeze(0).contiguous(), v[lo:hi].unsqueeze(0).contiguous(),
                 bt[b:b + 1], [hi - lo])
            del k, v
    elif w.kv == "f16" and spec["dist"] == "normal":
        w.k_cache.copy_(torch.randn(w.k_cache.shape, generator=gen, device=device))
        w.v_cache.copy_(torch.randn(w.v_cache.shape, generator=gen, device=device))
    else:
        chunk = max(1, (256 << 20) // (int(lens.max()) * KVH * HEAD_DIM * 2))
        state = gen.get_state()
        if w.per_tensor:
            # One scale per tensor over the whole batch (quantize_per_tensor,
            # tests/paged_decode_attn.py:115-121): a first pass over the same seeded rows.
            kmax = torch.zeros((), device=device)
            vmax = torch.zeros((), device=device)
            for b0 in range(0, B, chunk):
                b1 = min(B, b0 + chunk)
                L = int(lens[b0:b1].max())
                k = _kv_rows(torch, (b1 - b0, L, KVH, HEAD_DIM), spec["dist"], gen, device)
                v = _kv_rows(torch, (b1 - b0, L, KVH, HEAD_DIM), spec["dist"], gen, device)
                kmax = torch.maximum(kmax, ops.absmax_scale(k))
                vmax = torch.maximum(vmax, ops.absmax_scale(v))
            w.k_fix, w.v_fix = kmax.reshape(1).contiguous(), vmax.reshape(1).contiguous()
            gen.set_state(state)
        for b0 in range(0, B, chunk):
            b1 = min(B, b0 + chunk)
            L = int(lens[b0:b1].max())
            k = _kv_rows(torch, (b1 - b0, L, KVH, HEAD_DIM), spec["dist"], gen, device)
            v = _kv_rows(torch, (b1 - b0, L, KVH, HEAD_DIM), spec["dist"], gen, device)
            fill(k, v, bt[b0:b1], lens[b0:b1])
            del k, v
    if w.step_tokens:
        # The token written each step, at position lens[b] (context_lens[b] - 1).
        w.new_k = _kv_rows(torch, (B, KVH, HEAD_DIM), spec["dist"], gen, device)
        w.new_v = _kv_rows(torch, (B, KVH, HEAD_DIM), spec["dist"], gen, device)
    per_tok = KVH * (2 * HEAD_DIM * (2 if w.kv == "f16" else 1) + (0 if w.kv == "f16" else 8))
    w.ctx_total = int(w.lens_host.sum())
    w.decode_bytes = w.ctx_total * per_tok
    w.write_bytes = ((B * KVH * (2 * HEAD_DIM * 2 + 2 * HEAD_DIM + 8)) if w.step_tokens
                     else 0)
    w.step_bytes = w.decode_bytes
    w.cache_bytes = (w.k_cache.numel() * w.k_cache.element_size() * 2 +
                     (2 * w.k_scales.numel() * 4 if scaled else 0))
    if spec["shard"] == "context":
        w.splitter = shard.SplitContextDecode()
    torch.cuda.synchronize()
    return w


def make_step(w, splitk=False, validate=False, decode_only=False):
    """One step of the workload: [one-token cache write per sequence +] decode. Returns the
    step function and this library's kernel launches per step."""
    from pa_b200 import ops
    scale = 1.0 / math.sqrt(HEAD_DIM)
    use_split = splitk or w.splitk

    if w.spec["shard"] == "context":
        def decode():
            w.splitter.step(w.out, w.q, w.k_cache, w.v_cache, w.block_table, w.context_lens,
                            scale, BLOCK, k_scales=w.k_scales, v_scales=w.v_scales)
        dec_launches = 2  # partial decode + merge (the all-gather is NCCL's)
    else:
        def decode():
            ops.decode(w.out, w.q, w.k_cache, w.v_cache, w.block_table, w.context_lens, scale,
                       BLOCK, k_scales=w.k_scales, v_scales=w.v_scales, splitk=use_split,
                       validate=validate)
        dec_launches = 2 if use_split else 1

    if w.step_tokens and not decode_only:
        # The decode step API: every sequence's new token is written into the cache, then the
        # decode runs. With its default the write is a launch of its own for these batch sizes
        # (more than 64 sequence x kv-head rows), else the decode kernel writes the tokens.
        def step():
            ops.decode_step(w.out, w.q, w.new_k, w.new_v, w.k_cache, w.v_cache, w.block_table,
                            w.context_lens, scale, BLOCK, k_scales=w.k_scales,
                            v_scales=w.v_scales, k_scale=w.k_fix, v_scale=w.v_fix,
                            splitk=use_split, validate=validate)
        fused = w.q.shape[0] * w.k_cache.shape[1] <= 64
        return step, dec_launches + (0 if fused else 1)
    return decode, dec_launches


# ---------------------------------------------------------------------------------------
# Timing
# ---------------------------------------------------------------------------------------
def _max_over_ranks(torch, dist, device, vals):
    if not dist:
        return vals
    t = torch.tensor(vals, device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t]


def _sum_over_ranks(torch, dist, device, vals):
    if not dist:
        return vals
    t = torch.tensor(vals, device=device, dtype=torch.float64)
    dist.all_reduce(t)
    return [float(x) for x in t]


def capture(torch, fn, steps, warmup, stream):
    """Warm `fn` up eagerly on `stream`, then capture `steps` calls into one CUDA graph."""
    with torch.cuda.stream(stream):
        for _ in range(max(3, warmup)):
            fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for _ in range(steps):
            fn()
    torch.cuda.synchronize()
    return g


def replay_ms(torch, g, steps, dist):
    """Device time of one replay of `g` (K steps) per step, between CUDA events on the
    current stream (the one replay() launches on), after a barrier."""
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def eager_ms(torch, fn, steps, warmup, dist):
    """Device time per call of `steps` eager calls of `fn` (host launches included), on the
    current stream."""
    for _ in range(max(3, warmup)):
        fn()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


# ---------------------------------------------------------------------------------------
# Parity: the timed output against an fp32 restatement of the reference decode
# (tests/paged_decode_attn.py:4-49, INT8 through dequantize_kv :202-216), in torch on the
# device, for a few sequences of the workload.
# ---------------------------------------------------------------------------------------
def _dense_seq(torch, k_cache, v_cache, k_scales, v_scales, bt_row, ctx):
    """fp32 K, V [ctx, KVH, D] of one sequence gathered from a paged cache (dequantised)."""
    nblk = (ctx + BLOCK - 1) // BLOCK
    blocks = bt_row[:nblk].long()
    KVH = k_cache.shape[1]
    kc, vc = k_cache, v_cache
    f8 = kc.dtype == getattr(torch, "float8_e4m3fn", None)
    if f8:  # gather as bytes, then convert
        kc, vc = kc.view(torch.uint8), vc.view(torch.uint8)
    k = kc[blocks]
    v = vc[blocks]
    if f8:
        k, v = k.view(torch.float8_e4m3fn), v.view(torch.float8_e4m3fn)
    k = k.float().permute(0, 3, 1, 2, 4).reshape(nblk * BLOCK, KVH, HEAD_DIM)[:ctx]
    v = v.float().permute(0, 3, 1, 2).reshape(nblk * BLOCK, KVH, HEAD_DIM)[:ctx]
    if k_scales is not None:
        ks = k_scales[blocks].permute(0, 2, 1).reshape(nblk * BLOCK, KVH)[:ctx]
        vs = v_scales[blocks].permute(0, 2, 1).reshape(nblk * BLOCK, KVH)[:ctx]
        k = k * ks.unsqueeze(-1)
        v = v * vs.unsqueeze(-1)
    return k, v


def _ref_decode(torch, q_row, k, v):
    """softmax(scale q.k) v for one sequence: q_row [H, D], k/v [ctx, KVH, D] -> [H, D]."""
    H = q_row.shape[0]
    KVH = k.shape[1]
    qh = q_row.float().view(KVH, H // KVH, HEAD_DIM)
    s = torch.einsum("kgd,tkd->kgt", qh, k) / math.sqrt(HEAD_DIM)
    p = torch.softmax(s, dim=-1)
    return torch.einsum("kgt,tkd->kgd", p, v).reshape(H, HEAD_DIM)


def _compare(torch, out_row, ref):
    d = (out_row.float() - ref).abs()
    excess = float((d - (ATOL + RTOL * ref.abs())).max())
    return float(d.max()), excess


def parity(torch, w, dist, device):
    """Compare the workload's last output with the fp32 torch reference on up to three
    sequences of this rank (the first, the longest, one seeded pick); max over ranks."""
    import numpy as np
    B = w.B
    picks = sorted({0, int(np.argmax(w.lens_host)), int(np.random.default_rng(5).integers(B))})
    max_abs, excess = 0.0, -1.0
    for b in picks:
        if w.spec["shard"] == "context":
            # The reference needs the whole context: rebuild this sequence's cache in full
            # from its seeded rows with the same write kernel.
            from pa_b200 import ops
            k_rows, v_rows = _seq_rows(torch, w.spec, b, device)
            L = k_rows.shape[0]
            nblk = (L + BLOCK - 1) // BLOCK
            KVH = w.KVH
            kc = torch.zeros(nblk, KVH, HEAD_DIM // 8, BLOCK, 8, dtype=torch.int8, device=device)
            vc = torch.zeros(nblk, KVH, HEAD_DIM, BLOCK, dtype=torch.int8, device=device)
            ks = torch.zeros(nblk, KVH, BLOCK, dtype=torch.float32, device=device)
            vs = torch.zeros_like(ks)
            bt1 = torch.arange(nblk, dtype=torch.int32, device=device).view(1, -1)
            ops.prefill_into_cache(k_rows.unsqueeze(0).contiguous(),
                                   v_rows.unsqueeze(0).contiguous(), kc, vc, bt1,
                                   torch.tensor([L], dtype=torch.int32, device=device), BLOCK,
                                   k_scales=ks, v_scales=vs)
            k, v = _dense_seq(torch, kc, vc, ks, vs, bt1[0], L)
            del k_rows, v_rows, kc, vc
        else:
            k, v = _dense_seq(torch, w.k_cache, w.v_cache, w.k_scales, w.v_scales,
                              w.block_table[b], int(w.lens_host[b]))
        ref = _ref_decode(torch, w.q[b], k, v)
        m, e = _compare(torch, w.out[b], ref)
        max_abs, excess = max(max_abs, m), max(excess, e)
        del k, v
    max_abs, excess = _max_over_ranks(torch, dist, device, [max_abs, excess])
    return {"ok": excess <= 0.0, "max_abs": max_abs, "max_excess_over_tol": excess,
            "seqs_checked_per_rank": len(picks), "tolerance": "2e-3 abs + 1e-2 rel",
            "reference": "fp32 torch restatement of the reference decode on the device"}


# ---------------------------------------------------------------------------------------
# Clock sampling
# ---------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = []
        for line in out.splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), smax=float(parts[2]),
                                 power=float(parts[3]) if parts[3] not in ("[N/A]", "") else 0.0,
                                 hw=parts[5], hwt=parts[6], swt=parts[7], pcap=parts[8]))
            except ValueError:
                continue
        if not rows:
            return None
        load = [r for r in rows if r["power"] > 250.0] or rows
        reasons = set()
        for r in load:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                              ("swt", "sw_thermal_slowdown"), ("pcap", "sw_power_cap")):
                if r[key].lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in load),
                "sm_max_mhz": max(r["smax"] for r in rows),
                "reasons": sorted(reasons), "samples": len(rows), "samples_under_load": len(load)}


# ---------------------------------------------------------------------------------------
# CPU baseline: the oracle port of the reference decode on a bounded sample
# ---------------------------------------------------------------------------------------
_CPU_SAMPLES = {  # name -> (kv kind, q heads, kv heads, context of the one sampled sequence)
    "cfg2": ("f16", 32, 8, 4096), "cfg3": ("i8", 12, 2, 8192), "cfg3_f16": ("f16", 12, 2, 8192),
    "cfg3_pt": ("i8", 12, 2, 8192), "cfg4": ("i8", 64, 8, 8192),
    "cfg4_ctxsplit": ("i8", 64, 8, 8192), "cfg5": ("i8", 28, 4, 3376),
    "cfg6": ("f8", 12, 2, 8192),
}


def _cpu_sample(name):
    """One bounded CPU step of the workload: the decode of one sequence (at most 8192
    tokens) of the configuration's shape, through the oracle port of the reference algorithm
    (tests/paged_decode_attn.py:4-49; INT8 via dequantize_kv first, :202-216; FP8 through the
    same dequantisation of e4m3 values)."""
    import numpy as np
    sys.path.insert(0, os.path.join(HERE, "oracle"))
    import pa_oracle
    kind, H, KVH, ctx = _CPU_SAMPLES[name]
    nblk = (ctx + BLOCK - 1) // BLOCK
    rng = np.random.default_rng(7)
    bt = rng.permutation(nblk).reshape(1, nblk).astype(np.int32)
    lens = np.full(1, ctx, np.int32)
    q = rng.standard_normal((1, H, HEAD_DIM), dtype=np.float32).astype(np.float16)
    if kind != "f16":
        if kind == "i8":
            kc = rng.integers(-127, 128, (nblk, KVH, 16, BLOCK, 8), dtype=np.int8)
            vc = rng.integers(-127, 128, (nblk, KVH, HEAD_DIM, BLOCK), dtype=np.int8)
            deq = pa_oracle.dequantize_kv
        else:
            kc = rng.integers(0, 0x7f, (nblk, KVH, 16, BLOCK, 8), dtype=np.uint8)
            vc = rng.integers(0, 0x7f, (nblk, KVH, HEAD_DIM, BLOCK), dtype=np.uint8)
            deq = pa_oracle.dequantize_fp8
        ks = rng.random((nblk, KVH, BLOCK), dtype=np.float32) * 0.05
        vs = rng.random((nblk, KVH, BLOCK), dtype=np.float32) * 0.05

        def step():
            kd, vd = deq(kc, vc, ks, vs)
            pa_oracle.paged_decode_attention(q, kd, vd, bt, lens, acc=np.float32)
    else:
        kc = rng.standard_normal((nblk, KVH, 16, BLOCK, 8), dtype=np.float32).astype(np.float16)
        vc = rng.standard_normal((nblk, KVH, HEAD_DIM, BLOCK), dtype=np.float32).astype(np.float16)

        def step():
            pa_oracle.paged_decode_attention(q, kc, vc, bt, lens, acc=np.float32)
    per_tok = KVH * (2 * HEAD_DIM * (2 if kind == "f16" else 1) + (0 if kind == "f16" else 8))
    desc = (f"1 sequence of ctx {ctx} ({H}/{KVH} heads, {kind} cache"
            f"{', dequantised first' if kind != 'f16' else ''}) per step, numpy oracle decode "
            "(BLAS matmuls)")
    return step, ctx * per_tok, desc


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def cpu_baseline(name, steps=None, warmup=1, budget_s=10.0):
    """Time the CPU reference path: `warmup` untimed steps, then `steps` timed steps (or as
    many as fit in budget_s when steps is None). Returns the cpu_baseline record."""
    step, nbytes, desc = _cpu_sample(name)
    for _ in range(max(1, warmup)):
        step()
    done = 0
    t0 = time.perf_counter()
    while True:
        step()
        done += 1
        el = time.perf_counter() - t0
        if (steps is not None and done >= steps) or (steps is None and el >= budget_s):
            break
    blas_threads = None
    try:
        import threadpoolctl
        info = threadpoolctl.threadpool_info()
        blas_threads = max((i.get("num_threads") or 0) for i in info) if info else None
    except Exception:
        pass
    try:
        import torch
        torch_threads = torch.get_num_threads()
    except Exception:
        torch_threads = None
    return {"value": done * nbytes / el / 1e9, "unit": "GB/s",
            "cores": blas_threads or os.cpu_count() or 1, "kind": "port",
            "host_cpus": os.cpu_count(), "torch_threads": torch_threads,
            "blas_threads": blas_threads, "cpu_model": _cpu_model(),
            "sample": f"{desc}; {done} steps in {el:.1f} s"}


def profile_traffic(name):
    """DRAM bytes (read + write) per launch of the workload's dominant kernel from the
    committed ncu summaries (profiles/traffic.json), or None when there is none."""
    path = os.path.join(HERE, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(name)
    except Exception:
        return None


def config_desc(name, w, splitk):
    spec = SPECS[name]
    d = {"workload": spec["desc"], "head_dim": HEAD_DIM, "block_size": BLOCK,
         "op": ("split-K pair" if (splitk or spec.get("splitk")) else
                "partials + all-gather + merge" if spec["shard"] == "context" else "single-pass"),
         "l2": "inputs larger than L2 (126 MB): KV cache %.0f MB per GPU" % (w.cache_bytes / 1e6)
         if w is not None else "n/a"}
    if w is not None:
        d.update({"global_batch": None, "per_gpu_batch": w.B, "num_heads": w.H,
                  "num_kv_heads": w.KVH,
                  "kv_dtype": {"f16": "fp16", "i8": "int8", "f8": "fp8_e4m3"}[w.kv] +
                  (" per-tensor" if w.per_tensor else ""),
                  "ctx_tokens_per_gpu": w.ctx_total})
    return d


# ---------------------------------------------------------------------------------------
# One configuration
# ---------------------------------------------------------------------------------------
def run_config(torch, name, args, rank, world, device, dist, peak, soak_ms=0.0):
    """Build, time (step and decode alone), check parity; returns (record, workload)."""
    w = build_workload(torch, name, rank, world, device)
    step, launches = make_step(w, args.splitk)
    dec, _ = make_step(w, args.splitk, decode_only=True)
    cap = torch.cuda.Stream(device)
    cap.wait_stream(torch.cuda.current_stream(device))
    res = {}
    if w.spec["shard"] == "context":
        # NCCL all-gather inside: timed as eager calls (host launches included); the kernels
        # alone (partial decode + merge of the local partials, no collective) as a graph.
        from pa_b200 import ops
        scale = 1.0 / math.sqrt(HEAD_DIM)

        def kernels_only():
            part = ops.decode_partial(w.q, w.k_cache, w.v_cache, w.block_table,
                                      w.context_lens, scale, BLOCK, k_scales=w.k_scales,
                                      v_scales=w.v_scales)
            ops.merge_partials(w.out, part.unsqueeze(0), w.H, w.KVH)

        with torch.cuda.stream(cap):
            ms = eager_ms(torch, step, args.steps, args.warmup, dist)
        g_dec = capture(torch, kernels_only, args.steps, args.warmup, cap)
        dec_ms = replay_ms(torch, g_dec, args.steps, dist)
        del g_dec
        with torch.cuda.stream(cap):
            step()  # leave the full (gathered and merged) output for the parity check
        torch.cuda.synchronize()
        res["timing"] = ("eager calls between CUDA events (NCCL all-gather inside); "
                         "kernel_ms = partial decode + merge of the local partials, graph")
    else:
        g_step = capture(torch, step, args.steps, args.warmup, cap)
        g_dec = capture(torch, dec, args.steps, args.warmup, cap)
        # One untimed replay of each graph: a graph's first launch also uploads it to the
        # device, which would otherwise land inside the timed replay.
        g_step.replay()
        g_dec.replay()
        torch.cuda.synchronize()
        if soak_ms > 0:
            t_end = time.perf_counter() + soak_ms / 1e3
            while time.perf_counter() < t_end:
                g_step.replay()
                torch.cuda.synchronize()
        ms = replay_ms(torch, g_step, args.steps, dist)
        dec_ms = replay_ms(torch, g_dec, args.steps, dist)
        g_step.replay()  # the step last, so the output includes the step's new token
        torch.cuda.synchronize()
        del g_step, g_dec
        res["timing"] = "CUDA graph of the K steps, replayed once between CUDA events"
    ms, dec_ms = _max_over_ranks(torch, dist, device, [ms, dec_ms])
    tot_bytes, seqs, dec_bytes = _sum_over_ranks(
        torch, dist, device, [float(w.step_bytes), float(w.B), float(w.decode_bytes)])
    if w.spec["shard"] in ("kvhead", "context"):
        seqs = float(w.seqs_total)  # every rank works on every sequence
    from pa_b200 import ops
    status = ops.read_status(device)
    st = torch.tensor([status], device=device, dtype=torch.int64)
    if dist:
        dist.all_reduce(st, op=dist.ReduceOp.MAX)
    kernel_gbs = float(w.decode_bytes) / (dec_ms * 1e-3) / 1e9  # this rank, slowest rank's time
    res.update({
        "workload": w.spec["desc"], "n_gpus": world, "scaling": scaling_of(name),
        "kv_dtype": config_desc(name, w, args.splitk)["kv_dtype"],
        "ms_per_step": ms, "kernel_ms": dec_ms,
        "value": tot_bytes / (ms * 1e-3) / 1e9, "unit": "GB/s",
        "kernel_gbs_aggregate": dec_bytes / (dec_ms * 1e-3) / 1e9,
        "seqs_per_s": seqs / (ms * 1e-3),
        "gpu_launches": launches * args.steps,
        "roofline": {"bound": "hbm", "achieved": kernel_gbs, "peak": peak, "unit": "GB/s",
                     "frac": kernel_gbs / peak,
                     "traffic": profile_traffic(name) if world == 1 else None,
                     "algorithmic_bytes_per_launch": w.decode_bytes},
        "device_status": int(st.item()),
        "parity": parity(torch, w, dist, device),
        "global_batch": int(seqs),
    })
    return res, w


def write_kernels(torch, device, peak, steps):
    """The cache-write kernels alone at config 3's bulk size (64 x 8192 tokens, 2 kv heads):
    the token-granular quantize-write through slot_mapping (at this size the windowed kernel,
    whose aligned runs of 16 slots, here every sequence's blocks, take the grouped page
    stores) and the block-granular prefill scatter. Algorithmic bytes per (token, kv head):
    2 x 128 x 2 B read, 2 x 128 B + 2 x 4 B written."""
    from pa_b200 import ops
    S, L, KVH = 64, 8192, 2
    N = S * L
    gen = torch.Generator(device=device)
    gen.manual_seed(77)
    k = _kv_rows(torch, (S, L, KVH, HEAD_DIM), "lognormal_outlier", gen, device)
    v = _kv_rows(torch, (S, L, KVH, HEAD_DIM), "lognormal_outlier", gen, device)
    NB = N // BLOCK
    kc = torch.zeros(NB, KVH, HEAD_DIM // 8, BLOCK, 8, dtype=torch.int8, device=device)
    vc = torch.zeros(NB, KVH, HEAD_DIM, BLOCK, dtype=torch.int8, device=device)
    ks = torch.zeros(NB, KVH, BLOCK, dtype=torch.float32, device=device)
    vs = torch.zeros_like(ks)
    perm = torch.randperm(NB, generator=gen, device=device).to(torch.int32)
    bt = perm.view(S, L // BLOCK).contiguous()
    cl = torch.full((S,), L, dtype=torch.int32, device=device)
    t = torch.arange(L, device=device)
    slots = (bt.long().gather(1, (t // BLOCK).expand(S, L)) * BLOCK + t % BLOCK)
    slots = slots.to(torch.int32).reshape(-1).contiguous()
    k2, v2 = k.view(N, KVH, HEAD_DIM), v.view(N, KVH, HEAD_DIM)
    nbytes = N * KVH * (2 * HEAD_DIM * 2 + 2 * HEAD_DIM + 8)
    cap = torch.cuda.Stream(device)
    cap.wait_stream(torch.cuda.current_stream(device))
    reps = max(3, min(steps, 20))
    out = {}
    for label, fn, kern in (
            ("quantize_into_cache", lambda: ops.quantize_into_cache(
                k2, v2, kc, vc, ks, vs, slots, BLOCK), "write_slots_kernel"),
            ("prefill_into_cache", lambda: ops.prefill_into_cache(
                k, v, kc, vc, bt, cl, BLOCK, k_scales=ks, v_scales=vs), "prefill_kernel")):
        g = capture(torch, fn, reps, 3, cap)
        g.replay()  # untimed: the first launch also uploads the graph
        torch.cuda.synchronize()
        ms = replay_ms(torch, g, reps, None)
        del g
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[label] = {"kernel": kern, "ms_per_launch": ms, "token_rows": N * KVH,
                      "algorithmic_bytes_per_launch": nbytes,
                      "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak,
                                   "unit": "GB/s", "frac": gbs / peak,
                                   "traffic": profile_traffic(kern)}}
    from pa_b200 import ops as _ops
    status = _ops.read_status(device)
    for r in out.values():
        r["device_status"] = status
    del k, v, kc, vc, ks, vs
    torch.cuda.empty_cache()
    return out


def e2e_measure(torch, w, args, dist, device, total_bytes, total_seqs):
    """End to end through the public API: pinned host q (+ table + lengths) -> device, the
    decode call (with its argument validation), result read back to pinned host memory.

    Without decode-step writes the headline is a serving loop over two independent batches of
    this workload that alternate on two CUDA streams (double buffering): a step uploads its
    batch's inputs, decodes and reads the output back on its batch's stream, so one batch's
    copies run while the other batch decodes. Before a batch's buffers are reused, two steps
    later, the host waits for that batch's previous output. Every step's copies are inside
    the timed region. The same steps on one stream, each waiting for its own output, are
    reported as "serial" (the headline where the step writes the cache, whose steps cannot
    overlap)."""
    from pa_b200 import cuda_ext, ops
    # A batch's inputs (q, block table, lengths) sit in one pinned staging buffer and are
    # uploaded with one copy into views of one device buffer.
    parts = (w.q, w.block_table, w.context_lens)
    offs, n = [], 0
    for t in parts:
        offs.append(n)
        n += (t.numel() * t.element_size() + 15) // 16 * 16
    scale = 1.0 / math.sqrt(HEAD_DIM)
    split = args.splitk or w.splitk

    def view(buf, i):
        t = parts[i]
        nb = t.numel() * t.element_size()
        return buf[offs[i]:offs[i] + nb].view(t.dtype).view(t.shape)

    class Batch:
        """One batch's pinned and device buffers, its stream and its DecodePlan."""

        def __init__(self):
            self.hstage = torch.zeros(n, dtype=torch.uint8, pin_memory=True)
            self.dstage = torch.empty(n, dtype=torch.uint8, device=device)
            self.hq, self.hbt, self.hcl = (view(self.hstage, i) for i in range(3))
            self.dq, self.dbt, self.dcl = (view(self.dstage, i) for i in range(3))
            for h, t in zip((self.hq, self.hbt, self.hcl), parts):
                h.copy_(t.cpu())
            self.hout = torch.empty(w.out.shape, dtype=w.out.dtype, pin_memory=True)
            self.dout = torch.empty_like(w.out)
            self.stream = torch.cuda.Stream(device)
            self.done = torch.cuda.Event()
            self.pending = False
            # A serving loop's decode: the arguments are checked once (ops.DecodePlan), each
            # step only uploads its inputs, checks the lengths on the pinned host copy they
            # came from (the reference's context_lens >= 1 check, without a device sync) and
            # launches.
            self.plan = None if w.step_tokens else ops.DecodePlan(
                self.dout, self.dq, w.k_cache, w.v_cache, self.dbt, self.dcl, scale, BLOCK,
                k_scales=w.k_scales, v_scales=w.v_scales, splitk=split)

        def issue(self, reference_names=False):
            """Upload, decode and read back on the current stream; nothing waits."""
            self.dstage.copy_(self.hstage, non_blocking=True)
            if reference_names:
                # The reference's op names (cuda_ext): their context_lens check reads the
                # device tensor back, one synchronisation per call.
                if w.kv == "i8":
                    cuda_ext.VARIANTS_INT8["splitk_int8" if split else "warp_int8"](
                        self.dout, self.dq, w.k_cache, w.v_cache, w.k_scales, w.v_scales,
                        self.dbt, self.dcl, scale, BLOCK)
                else:
                    cuda_ext.VARIANTS["splitk" if split else "warp"](
                        self.dout, self.dq, w.k_cache, w.v_cache, self.dbt, self.dcl, scale,
                        BLOCK)
            elif w.step_tokens:
                ops.decode_step(self.dout, self.dq, w.new_k, w.new_v, w.k_cache, w.v_cache,
                                self.dbt, self.dcl, scale, BLOCK, k_scales=w.k_scales,
                                v_scales=w.v_scales, k_scale=w.k_fix, v_scale=w.v_fix,
                                splitk=split, host_context_lens=self.hcl)
            else:
                self.plan.run(host_context_lens=self.hcl)
            self.hout.copy_(self.dout, non_blocking=True)

    batches = [Batch(), Batch()]

    def serial_step(reference_names=False):
        b = batches[0]
        with torch.cuda.stream(b.stream):
            b.issue(reference_names)
        b.stream.synchronize()

    step_no = [0]

    def pipelined_step():
        b = batches[step_no[0] & 1]
        step_no[0] += 1
        if b.pending:
            b.done.synchronize()  # this batch's previous output is in b.hout
        with torch.cuda.stream(b.stream):
            b.issue()
            b.done.record()
        b.pending = True

    def drain():
        for b in batches:
            if b.pending:
                b.done.synchronize()
                b.pending = False

    def timed(fn):
        for _ in range(3):
            fn()
        drain()
        if dist:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            fn()
        drain()
        return _max_over_ranks(torch, dist, device, [(time.perf_counter() - t0) / args.steps])[0]

    b0 = batches[0]
    h2d = b0.hstage.numel()
    d2h = b0.hout.numel() * b0.hout.element_size()
    serial_s = timed(serial_step)
    serial = {"value": total_bytes / serial_s / 1e9, "unit": "GB/s",
              "ms_per_step": serial_s * 1e3,
              "path": ("pa_b200.ops.decode_step" if w.step_tokens else
                       "pa_b200.ops.DecodePlan.run") +
                      " on one stream, each step waiting for its output"}
    if w.step_tokens:
        e2e_s = serial_s
        path = serial["path"]
    else:
        e2e_s = timed(pipelined_step)
        path = ("pa_b200.ops.DecodePlan.run, two batches alternating on two streams (one "
                "batch's copies overlap the other's decode)")
    rec = {"value": total_bytes / e2e_s / 1e9, "unit": "GB/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
           "seqs_per_s": total_seqs / e2e_s, "ms_per_step": e2e_s * 1e3,
           "path": path + "; inputs uploaded from one pinned staging buffer per batch, "
                          "lengths checked on its host copy, output read back to pinned "
                          "memory"}
    if not w.step_tokens:
        rec["serial"] = serial
        # Both batches decode the same inputs: their outputs read back on the host must be
        # identical to each other and to the device-timed run's output.
        ref_out = w.out.cpu()
        rec["outputs_match"] = all(torch.equal(b.hout, ref_out) for b in batches)
    if not w.step_tokens and w.kv != "f8":
        ref_s = timed(lambda: serial_step(reference_names=True))
        rec["reference_names"] = {"value": total_bytes / ref_s / 1e9, "unit": "GB/s",
                                  "ms_per_step": ref_s * 1e3,
                                  "path": "pa_b200.cuda_ext on one stream (reference op "
                                          "names: one context_lens device read-back per "
                                          "call)"}
    return rec


def main():
    args = parse()
    import numpy as np  # noqa: F401

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    head = args.config or "cfg2"

    if args.impl == "reference":
        if rank != 0:
            return 0
        base = cpu_baseline(head, steps=args.steps, warmup=args.warmup)
        line = {"metric": METRIC, "value": base["value"], "unit": "GB/s", "impl": "reference",
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "higher_is_better": True, "scaling": scaling_of(head),
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": config_desc(head, None, args.splitk),
                "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    import torch
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=device)
    peak, peak_kind = measured_peak()

    if args.config == "writes":
        # The cache-write kernels alone (one GPU), as recorded under configs.write_kernels.
        rec = write_kernels(torch, device, peak, args.steps)
        if rank == 0:
            print(json.dumps({"metric": "cache-write achieved HBM GB/s", "unit": "GB/s",
                              "n_gpus": 1, "steps": args.steps, "write_kernels": rec}),
                  flush=True)
        if dist:
            dist.destroy_process_group()
        return 0

    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    rec, w = run_config(torch, head, args, rank, world, device, dist, peak,
                        soak_ms=args.soak_ms)
    cfg_head = config_desc(head, w, args.splitk)
    cfg_head["global_batch"] = rec["global_batch"]
    e2e = None
    if not args.no_e2e and w.spec["shard"] != "context":
        e2e = e2e_measure(torch, w, args, dist, device,
                          rec["value"] * rec["ms_per_step"] * 1e6, rec["global_batch"])
    del w
    torch.cuda.empty_cache()

    configs = {}
    if args.config is None:
        for name in (SECONDARY_1GPU if world == 1 else SECONDARY_MULTI):
            r, wc = run_config(torch, name, args, rank, world, device, dist, peak)
            if rank == 0 and world == 1 and not args.no_cpu_baseline:
                r["cpu_baseline"] = cpu_baseline(name, budget_s=4.0)
            configs[name] = r
            del wc
            torch.cuda.empty_cache()
        if world == 1:
            configs["write_kernels"] = write_kernels(torch, device, peak, args.steps)
    clocks = sampler.stop() if sampler else None

    kernel = "decode (%s)" % ("split-K pair" if (args.splitk or SPECS[head].get("splitk"))
                              else "partials + merge" if SPECS[head]["shard"] == "context"
                              else "single pass")
    line = {
        "metric": METRIC, "value": rec["value"], "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": rec["ms_per_step"],
        "higher_is_better": True, "scaling": rec["scaling"], "vs_baseline": None,
        "dtype": {"f16": "f16", "i8": "int8", "f8": "fp8_e4m3"}[SPECS[head]["kv"]],
        "data": "synthetic",
        "config": cfg_head,
        "seqs_per_s": rec["seqs_per_s"],
        "pct_of_nominal_8000": 100.0 * rec["roofline"]["achieved"] / NOMINAL_GBS,
        "pct_of_measured_peak": 100.0 * rec["roofline"]["achieved"] / peak,
        "gpu_launches": rec["gpu_launches"],
        "timing": rec["timing"],
        "roofline": dict(rec["roofline"], peak_kind=peak_kind, kernel=kernel,
                         kernel_ms=rec["kernel_ms"]),
        "parity": rec["parity"],
        "device_status": rec["device_status"],
        "clocks": clocks,
    }
    if e2e:
        line["e2e"] = e2e
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline(head)
    if configs:
        line["configs"] = configs
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
