"""Benchmark of the B200 paged-attention decode path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2|3|4|5] [--impl ours|reference]

Metric: achieved HBM GB/s of a paged-decode step -- algorithmic bytes of KV
(plus per-token scales for INT8) read per step / step time -- with seqs/s and % of peak.
Default workload: BASELINE config 2 (FP16, batch 64, context 4096, 32 q / 8 kv heads,
head_dim 128, block 16, shuffled block tables over 16384 blocks). At N GPUs every rank runs
its own config-2 batch (sequence sharding, no communication): weak scaling.
Other configs: 3 INT8 per-token decode + one-token
quantize-write per sequence (B64, ctx 8192, 12/2); 4 long-context split-K INT8 sharded by
kv-head (B8, ctx U[65536,131072], 64/8); 5 ragged INT8 serving batch + one-token write per
sequence, sequences LPT-sharded across ranks (B256, 28/4, ctx lognormal median 2048 sigma 1).
Configs 4 and 5 divide one fixed workload among the ranks (strong scaling).
Inputs are synthetic (seeded), far larger than L2 (126 MB) for configs 2-5 except where
noted in the JSON; timing is CUDA events on the launching stream, max over ranks.
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


def scaling_of(cfg):
    """Configs 4 and 5 split one fixed workload across the ranks (by kv head, by sequence):
    strong scaling. The others give every rank its own batch: weak scaling."""
    return "strong" if cfg in (4, 5) else "weak"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--config", type=int, default=2, choices=[2, 3, 4, 5, 6])
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--splitk", action="store_true", help="use the split-K pair")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--soak-ms", type=float, default=1500.0,
                   help="untimed load before the timed region so the clock sampler sees it")
    return p.parse_args()


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
    x = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
    if dist == "lognormal_outlier":
        mag = torch.exp(0.5 * torch.randn(shape[:-1], generator=gen, device=device))
        x = x * mag.unsqueeze(-1)
        kvh = shape[-2]
        ch = torch.randint(0, shape[-1], (kvh,), generator=gen, device=device)
        x[..., torch.arange(kvh, device=device), ch] *= 20.0
    return x.to(torch.float16)


def build_workload(torch, cfg, rank, world, device):
    import numpy as np
    from pa_b200 import ops
    gen = torch.Generator(device=device)
    gen.manual_seed(1234 + rank)
    w = Workload()
    w.cfg = cfg
    rng = np.random.default_rng(99)
    if cfg == 2:
        B, H, KVH, int8 = 64, 32, 8, False
        lens = np.full(B, 4096, dtype=np.int64)
        NB = 16384
    elif cfg in (3, 6):
        B, H, KVH, int8 = 64, 12, 2, True
        lens = np.full(B, 8192 - 1, dtype=np.int64)  # +1 token written each step
        NB = B * 8192 // BLOCK + 64
    elif cfg == 4:
        B, H, KVH, int8 = 8, 64, 8, True
        lens = rng.integers(65536, 131073, size=B)
        assert KVH % world == 0, "config 4 shards 8 kv heads"
        KVH //= world
        H //= world
        NB = int(sum((int(c) + BLOCK - 1) // BLOCK for c in lens)) + 8
    else:
        B, H, KVH, int8 = 256, 28, 4, True
        all_lens = np.clip(np.exp(rng.normal(math.log(2048), 1.0, size=B)), 16, 32768)
        all_lens = all_lens.astype(np.int64) - 1  # +1 token written each step
        from pa_b200 import shard
        parts = shard.lpt_partition(all_lens.tolist(), world)
        lens = all_lens[parts[rank]]
        B = len(lens)
        NB = int(sum((int(c) + 1 + BLOCK - 1) // BLOCK for c in lens)) * 2 + 64
    w.B, w.H, w.KVH, w.int8, w.NB = B, H, KVH, int8, NB
    w.fp8 = cfg == 6  # config 3's shapes with the FP8 (e4m3) cache instead of INT8
    w.step_tokens = 1 if cfg in (3, 5, 6) else 0
    w.lens_host = lens.astype(np.int32)
    maxb = int((lens.max() + w.step_tokens + BLOCK - 1) // BLOCK)
    # Fragmented pool: every sequence's blocks come from one seeded permutation of the pool.
    perm = torch.randperm(NB, generator=gen, device=device).to(torch.int32)
    bt = torch.zeros(B, maxb, dtype=torch.int32, device=device)
    nxt = 0
    for b in range(B):
        nb_b = int((lens[b] + w.step_tokens + BLOCK - 1) // BLOCK)
        bt[b, :nb_b] = perm[nxt:nxt + nb_b]
        nxt += nb_b
    w.block_table = bt
    w.context_lens = torch.from_numpy(w.lens_host + w.step_tokens).to(device)
    w.q = torch.randn(B, H, HEAD_DIM, generator=gen, device=device).to(torch.float16)
    w.out = torch.empty_like(w.q)
    dt = torch.float8_e4m3fn if w.fp8 else (torch.int8 if int8 else torch.float16)
    w.k_cache = torch.empty(NB, KVH, HEAD_DIM // 8, BLOCK, 8, dtype=dt, device=device)
    w.v_cache = torch.empty(NB, KVH, HEAD_DIM, BLOCK, dtype=dt, device=device)
    if not int8:
        w.k_cache.copy_(torch.randn(w.k_cache.shape, generator=gen, device=device))
        w.v_cache.copy_(torch.randn(w.v_cache.shape, generator=gen, device=device))
        w.k_scales = w.v_scales = None
    else:
        w.k_scales = torch.zeros(NB, KVH, BLOCK, dtype=torch.float32, device=device)
        w.v_scales = torch.zeros(NB, KVH, BLOCK, dtype=torch.float32, device=device)
        # Fill through the bulk quantize-scatter kernel, a chunk of sequences at a time.
        chunk = max(1, (256 << 20) // (int(lens.max()) * KVH * HEAD_DIM * 2))
        for b0 in range(0, B, chunk):
            b1 = min(B, b0 + chunk)
            L = int(lens[b0:b1].max())
            k = _kv_rows(torch, (b1 - b0, L, KVH, HEAD_DIM), "lognormal_outlier", gen, device)
            v = _kv_rows(torch, (b1 - b0, L, KVH, HEAD_DIM), "lognormal_outlier", gen, device)
            if w.fp8:
                # Token rows through the FP8 write kernel (slot -1 past each context).
                t = torch.arange(L, device=device)
                lens_c = torch.from_numpy(w.lens_host[b0:b1].astype(np.int64)).to(device)
                blk = bt[b0:b1].long().gather(1, (t // BLOCK).expand(b1 - b0, L))
                slots = torch.where(t[None, :] < lens_c[:, None], blk * BLOCK + t % BLOCK,
                                    torch.full_like(blk, -1)).to(torch.int32).reshape(-1)
                ops.quantize_into_cache(k.reshape(-1, KVH, HEAD_DIM), v.reshape(-1, KVH, HEAD_DIM),
                                        w.k_cache, w.v_cache, w.k_scales, w.v_scales, slots,
                                        BLOCK)
            else:
                ops.prefill_into_cache(k, v, w.k_cache, w.v_cache, bt[b0:b1].contiguous(),
                                       torch.from_numpy(w.lens_host[b0:b1]).to(device), BLOCK,
                                       k_scales=w.k_scales, v_scales=w.v_scales)
            del k, v
    if w.step_tokens:
        # The token written each step: slot of position lens[b] in sequence b.
        pos = torch.from_numpy(w.lens_host.astype(np.int64)).to(device)
        blk = bt.gather(1, (pos // BLOCK).view(-1, 1)).view(-1).long()
        w.slots = (blk * BLOCK + pos % BLOCK).to(torch.int32)
        w.new_k = _kv_rows(torch, (B, KVH, HEAD_DIM), "lognormal_outlier", gen, device)
        w.new_v = _kv_rows(torch, (B, KVH, HEAD_DIM), "lognormal_outlier", gen, device)
    per_tok = KVH * (2 * HEAD_DIM * (1 if int8 else 2) + (8 if int8 else 0))
    w.ctx_total = int((w.lens_host + w.step_tokens).sum())
    w.decode_bytes = w.ctx_total * per_tok
    w.write_bytes = (B * KVH * (2 * HEAD_DIM * 2 + 2 * HEAD_DIM + 8)) if w.step_tokens else 0
    w.step_bytes = w.decode_bytes
    w.cache_bytes = (w.k_cache.numel() * w.k_cache.element_size() * 2 +
                     (2 * w.k_scales.numel() * 4 if int8 else 0))
    return w


def make_step(torch, w, splitk, validate=False, decode_only=False):
    """One step of the workload: [one-token quantize-write per sequence +] decode."""
    from pa_b200 import ops
    scale = 1.0 / math.sqrt(HEAD_DIM)
    use_split = splitk or w.cfg == 4

    def decode():
        ops.decode(w.out, w.q, w.k_cache, w.v_cache, w.block_table, w.context_lens, scale,
                   BLOCK, k_scales=w.k_scales, v_scales=w.v_scales, splitk=use_split,
                   validate=validate)

    dec_launches = 2 if use_split else 1
    if w.step_tokens and not decode_only:
        def step():
            ops.quantize_into_cache(w.new_k, w.new_v, w.k_cache, w.v_cache, w.k_scales,
                                    w.v_scales, w.slots, BLOCK)
            decode()
        return step, 1 + dec_launches
    return decode, dec_launches


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
        self.t0 = self.t1 = None

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
def _cpu_sample(cfg):
    """One bounded CPU step of the workload: the decode of one sequence (at most 8192
    tokens) of the configuration's shape, through the oracle port of the reference algorithm
    (tests/paged_decode_attn.py:4-49; INT8 via dequantize_kv first, :202-216)."""
    import numpy as np
    sys.path.insert(0, os.path.join(HERE, "oracle"))
    import pa_oracle
    H, KVH, ctx, int8 = {2: (32, 8, 4096, False), 3: (12, 2, 8192, True),
                         4: (64, 8, 8192, True), 5: (28, 4, 3376, True)}[cfg]
    nblk = (ctx + BLOCK - 1) // BLOCK
    rng = np.random.default_rng(7)
    bt = rng.permutation(nblk).reshape(1, nblk).astype(np.int32)
    lens = np.full(1, ctx, np.int32)
    q = rng.standard_normal((1, H, HEAD_DIM), dtype=np.float32).astype(np.float16)
    if int8:
        kc = rng.integers(-127, 128, (nblk, KVH, 16, BLOCK, 8), dtype=np.int8)
        vc = rng.integers(-127, 128, (nblk, KVH, HEAD_DIM, BLOCK), dtype=np.int8)
        ks = rng.random((nblk, KVH, BLOCK), dtype=np.float32) * 0.05
        vs = rng.random((nblk, KVH, BLOCK), dtype=np.float32) * 0.05

        def step():
            kd, vd = pa_oracle.dequantize_kv(kc, vc, ks, vs)
            pa_oracle.paged_decode_attention(q, kd, vd, bt, lens, acc=np.float32)
    else:
        kc = rng.standard_normal((nblk, KVH, 16, BLOCK, 8), dtype=np.float32).astype(np.float16)
        vc = rng.standard_normal((nblk, KVH, HEAD_DIM, BLOCK), dtype=np.float32).astype(np.float16)

        def step():
            pa_oracle.paged_decode_attention(q, kc, vc, bt, lens, acc=np.float32)
    per_tok = KVH * (2 * HEAD_DIM * (1 if int8 else 2) + (8 if int8 else 0))
    desc = (f"1 sequence of ctx {ctx} ({H}/{KVH} heads{', int8 dequant' if int8 else ''}) per "
            "step, numpy oracle decode (BLAS matmuls on all host threads)")
    return step, ctx * per_tok, desc


def cpu_baseline(cfg, steps=None, warmup=1, budget_s=10.0):
    """Time the CPU reference path: `warmup` untimed steps, then `steps` timed steps (or as
    many as fit in budget_s when steps is None). Returns the cpu_baseline record."""
    step, nbytes, desc = _cpu_sample(cfg)
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
    return {"value": done * nbytes / el / 1e9, "unit": "GB/s", "cores": os.cpu_count() or 1,
            "kind": "port", "sample": f"{desc}; {done} steps in {el:.1f} s"}


def profile_traffic(cfg):
    """DRAM bytes (read + write) per decode launch from the committed ncu summary of this
    workload (profiles/), or None when there is none."""
    path = os.path.join(HERE, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(f"cfg{cfg}")
    except Exception:
        return None


def config_desc(cfg, w, splitk):
    names = {2: "cfg2 FP16 decode B64 ctx4096 32/8 heads",
             3: "cfg3 INT8 per-token decode + 1-token quantize-write B64 ctx8192 12/2",
             4: "cfg4 INT8 split-K decode B8 ctx U[65536,131072] 64/8 (kv-head sharded)",
             5: "cfg5 ragged INT8 serving B256 28/4 + 1-token write (sequence sharded)",
             6: "cfg6 FP8-e4m3 per-token decode + 1-token quantize-write B64 ctx8192 12/2"}
    d = {"workload": names[cfg], "head_dim": HEAD_DIM, "block_size": BLOCK,
         "op": ("splitk pair" if (splitk or cfg == 4) else "single-pass"),
         "l2": "inputs larger than L2 (126 MB): KV cache %.0f MB per GPU" % (w.cache_bytes / 1e6)
         if w is not None else "n/a"}
    if w is not None:
        d.update({"global_batch": None, "per_gpu_batch": w.B, "num_heads": w.H,
                  "num_kv_heads": w.KVH,
                  "kv_dtype": "fp8_e4m3" if w.fp8 else ("int8" if w.int8 else "fp16"),
                  "ctx_tokens_per_gpu": w.ctx_total})
    return d


def main():
    args = parse()
    import numpy as np  # noqa: F401

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return 0
        base = cpu_baseline(args.config, steps=args.steps, warmup=args.warmup)
        line = {"metric": METRIC, "value": base["value"], "unit": "GB/s", "impl": "reference",
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "higher_is_better": True, "scaling": scaling_of(args.config),
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": config_desc(args.config, None, args.splitk),
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

    w = build_workload(torch, args.config, rank, world, device)
    step, launches = make_step(torch, w, args.splitk)
    decode_only, decode_launches = make_step(torch, w, args.splitk, decode_only=True)

    # Warm up eagerly on the capture stream (its workspace is created here), then capture
    # the K timed steps into one CUDA graph so that host launch overhead is not measured.
    cap = torch.cuda.Stream(device)
    cap.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(cap):
        for _ in range(max(3, args.warmup)):
            step()
            decode_only()
    torch.cuda.synchronize()
    g_step = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_step, stream=cap):
        for _ in range(args.steps):
            step()
    g_dec = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_dec, stream=cap):
        for _ in range(args.steps):
            decode_only()
    torch.cuda.synchronize()

    # Untimed soak so the clock sampler sees the kernel under load, then the timed steps.
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    t_end = time.perf_counter() + args.soak_ms / 1e3
    while time.perf_counter() < t_end:
        g_step.replay()
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    g_step.replay()
    end.record()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    ms = start.elapsed_time(end) / args.steps
    # The dominant kernel alone (decode), same device clock, for the roofline figure.
    d0 = torch.cuda.Event(enable_timing=True)
    d1 = torch.cuda.Event(enable_timing=True)
    d0.record()
    g_dec.replay()
    d1.record()
    torch.cuda.synchronize()
    dec_ms = d0.elapsed_time(d1) / args.steps
    if dist:
        t = torch.tensor([ms, dec_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, dec_ms = float(t[0]), float(t[1])
        tot = torch.tensor([float(w.step_bytes), float(w.B)], device=device, dtype=torch.float64)
        dist.all_reduce(tot)
        total_bytes, total_seqs = float(tot[0]), float(tot[1])
    else:
        total_bytes, total_seqs = float(w.step_bytes), float(w.B)
    if args.config == 4:
        total_seqs = float(w.B)  # every rank decodes all sequences, for its share of kv heads
    del g_step, g_dec
    from pa_b200 import ops
    status = ops.read_status(device)

    # End to end through the public API: pinned host q (+ table + lengths) -> device, the
    # decode call (with its argument validation), result read back to pinned host memory.
    e2e = None
    if not args.no_e2e:
        from pa_b200 import cuda_ext
        hq = w.q.cpu().pin_memory()
        hbt = w.block_table.cpu().pin_memory()
        hcl = w.context_lens.cpu().pin_memory()
        hout = torch.empty(w.out.shape, dtype=w.out.dtype, pin_memory=True)
        dq, dbt, dcl, dout = (torch.empty_like(w.q), torch.empty_like(w.block_table),
                              torch.empty_like(w.context_lens), torch.empty_like(w.out))
        scale = 1.0 / math.sqrt(HEAD_DIM)

        def e2e_step():
            dq.copy_(hq, non_blocking=True)
            dbt.copy_(hbt, non_blocking=True)
            dcl.copy_(hcl, non_blocking=True)
            if w.step_tokens:
                ops.quantize_into_cache(w.new_k, w.new_v, w.k_cache, w.v_cache, w.k_scales,
                                        w.v_scales, w.slots, BLOCK)
            if w.fp8:
                # No reference op takes an FP8 cache: the library's own decode op.
                ops.decode(dout, dq, w.k_cache, w.v_cache, dbt, dcl, scale, BLOCK,
                           k_scales=w.k_scales, v_scales=w.v_scales, splitk=args.splitk)
            elif w.int8:
                name = "splitk_int8" if (args.splitk or args.config == 4) else "warp_int8"
                cuda_ext.VARIANTS_INT8[name](dout, dq, w.k_cache, w.v_cache, w.k_scales,
                                             w.v_scales, dbt, dcl, scale, BLOCK)
            else:
                name = "splitk" if args.splitk else "warp"
                cuda_ext.VARIANTS[name](dout, dq, w.k_cache, w.v_cache, dbt, dcl, scale, BLOCK)
            hout.copy_(dout, non_blocking=True)
            torch.cuda.current_stream().synchronize()

        for _ in range(3):
            e2e_step()
        if dist:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_step()
        e2e_s = (time.perf_counter() - t0) / args.steps
        if dist:
            t = torch.tensor([e2e_s], device=device, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_s = float(t.item())
        h2d = (hq.numel() * hq.element_size() + hbt.numel() * 4 + hcl.numel() * 4)
        d2h = hout.numel() * hout.element_size()
        e2e = {"value": total_bytes / e2e_s / 1e9, "unit": "GB/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "seqs_per_s": total_seqs / e2e_s, "ms_per_step": e2e_s * 1e3,
               "path": ("pa_b200.ops.decode" if w.fp8 else "pa_b200.cuda_ext") +
                       " (validate=True: one context_lens host check/step)"}

    peak, peak_kind = measured_peak()
    value = total_bytes / (ms * 1e-3) / 1e9
    per_gpu = float(w.step_bytes) / (ms * 1e-3) / 1e9
    kernel_gbs = float(w.decode_bytes) / (dec_ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": scaling_of(args.config),
        "vs_baseline": None, "dtype": "fp8_e4m3" if w.fp8 else ("int8" if w.int8 else "f16"),
        "data": "synthetic",
        "config": config_desc(args.config, w, args.splitk),
        "seqs_per_s": total_seqs / (ms * 1e-3),
        "pct_of_nominal_8000": 100.0 * per_gpu / NOMINAL_GBS,
        "pct_of_measured_peak": 100.0 * per_gpu / peak,
        "gpu_launches": launches * args.steps,
        "timing": "CUDA graph of the K steps, replayed once between CUDA events",
        "roofline": {"bound": "hbm", "achieved": kernel_gbs, "peak": peak, "unit": "GB/s",
                     "frac": kernel_gbs / peak, "peak_kind": peak_kind,
                     "kernel": "decode (%s)" % ("split-K pair" if (args.splitk or args.config == 4)
                                                else "single pass"),
                     "kernel_ms": dec_ms,
                     "traffic": profile_traffic(args.config),
                     "algorithmic_bytes_per_launch": w.decode_bytes},
        "device_status": status,
        "clocks": clocks,
    }
    line["config"]["global_batch"] = int(total_seqs)
    if e2e:
        line["e2e"] = e2e
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline(args.config)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
