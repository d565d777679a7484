"""GPU parity at the BASELINE configurations' full sizes.

Every decode configuration the benchmark times is run here at its own size through the
reference's op names (cuda_ext.VARIANTS / VARIANTS_INT8) and compared, sequence by sequence,
with the oracle (oracle/pa_oracle.py: paged_decode_attention, INT8 through dequantize_kv) at
the north-star tolerance, 2e-3 absolute + 1e-2 relative:
  * config 2: FP16, 64 sequences x 4096 tokens, 32/8 heads, 16384 shuffled blocks;
  * config 3: INT8 per-token, 64 x 8192 tokens, 12/2 heads, lognormal rows with one x20
    outlier channel per kv head; the same cache with per-tensor scales; the FP16 cache of the
    same rows; an FP8 (e4m3) cache of the same rows;
  * config 4: INT8 split-K, 64/8 heads, two sequences of 131072 tokens and one of 65537;
  * config 5: INT8, the whole 256-sequence ragged batch (lognormal lengths, median 2048,
    sigma 1, clipped to [16, 32768]), 28/4 heads.
Caches are written by the library's own write kernels (bit-exact with the oracle's quantiser,
tests/test_quant_gpu.py); the oracle reads each sequence's pages, copied to the host.
"""

import math

import numpy as np
import pytest
import torch

import pa_oracle
from pa_testlib import ATOL, RTOL

pytestmark = pytest.mark.gpu

D = 128
BS = 16
SCALE = 1.0 / math.sqrt(D)


def _rows(shape, dist, gen):
    x = torch.randn(shape, generator=gen, device="cuda", dtype=torch.float32)
    if dist == "lognormal_outlier":
        x = x * torch.exp(0.5 * torch.randn(shape[:-1], generator=gen, device="cuda")).unsqueeze(-1)
        kvh = shape[-2]
        ch = torch.randint(0, D, (kvh,), generator=gen, device="cuda")
        x[..., torch.arange(kvh, device="cuda"), ch] *= 20.0
    return x.half()


def _build(lens, H, KVH, kinds, dist, seed, extra_blocks=64):
    """Seeded rows -> paged caches of each kind in `kinds` ('f16', 'i8', 'i8pt', 'f8') over one
    shuffled block pool; returns q, block_table, context_lens and the caches."""
    from pa_b200 import ops
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    lens = np.asarray(lens, dtype=np.int64)
    B = len(lens)
    NB = int(sum((int(c) + BS - 1) // BS for c in lens)) + extra_blocks
    perm = torch.randperm(NB, generator=gen, device="cuda").to(torch.int32)
    maxb = int((lens.max() + BS - 1) // BS)
    bt = torch.zeros(B, maxb, dtype=torch.int32, device="cuda")
    nxt = 0
    for b in range(B):
        n = int((lens[b] + BS - 1) // BS)
        bt[b, :n] = perm[nxt:nxt + n]
        nxt += n
    cl = torch.from_numpy(lens.astype(np.int32)).cuda()
    q = torch.randn(B, H, D, generator=gen, device="cuda").half()
    caches = {}
    for kind in kinds:
        dt = {"f16": torch.float16, "i8": torch.int8, "i8pt": torch.int8,
              "f8": torch.float8_e4m3fn}[kind]
        kc = torch.zeros(NB, KVH, D // 8, BS, 8, dtype=dt, device="cuda")
        vc = torch.zeros(NB, KVH, D, BS, dtype=dt, device="cuda")
        ks = vs = None
        if kind != "f16":
            ks = torch.zeros(NB, KVH, BS, dtype=torch.float32, device="cuda")
            vs = torch.zeros_like(ks)
        caches[kind] = [kc, vc, ks, vs, None, None]
    # Rows are generated in chunks of sequences; every cache kind gets the same rows.
    chunk = max(1, (256 << 20) // (int(lens.max()) * KVH * D * 2))
    state = gen.get_state()
    if "i8pt" in kinds:
        kmax = torch.zeros((), device="cuda")
        vmax = torch.zeros((), device="cuda")
        for b0 in range(0, B, chunk):
            b1 = min(B, b0 + chunk)
            L = int(lens[b0:b1].max())
            k = _rows((b1 - b0, L, KVH, D), dist, gen)
            v = _rows((b1 - b0, L, KVH, D), dist, gen)
            # Per-tensor scale over the valid tokens of the batch.
            t = torch.arange(L, device="cuda")
            valid = (t[None, :] < cl[b0:b1, None].long())[..., None, None]
            kmax = torch.maximum(kmax, ops.absmax_scale((k * valid).contiguous()))
            vmax = torch.maximum(vmax, ops.absmax_scale((v * valid).contiguous()))
        caches["i8pt"][4] = kmax.reshape(1).contiguous()
        caches["i8pt"][5] = vmax.reshape(1).contiguous()
        gen.set_state(state)
    for b0 in range(0, B, chunk):
        b1 = min(B, b0 + chunk)
        L = int(lens[b0:b1].max())
        k = _rows((b1 - b0, L, KVH, D), dist, gen)
        v = _rows((b1 - b0, L, KVH, D), dist, gen)
        for kind, (kc, vc, ks, vs, kf, vf) in caches.items():
            if kind == "f8":
                t = torch.arange(L, device="cuda")
                blk = bt[b0:b1].long().gather(1, (t // BS).expand(b1 - b0, L))
                slots = torch.where(t[None, :] < cl[b0:b1, None].long(), blk * BS + t % BS,
                                    torch.full_like(blk, -1)).to(torch.int32).reshape(-1)
                ops.quantize_into_cache(k.reshape(-1, KVH, D), v.reshape(-1, KVH, D), kc, vc,
                                        ks, vs, slots, BS)
            else:
                ops.prefill_into_cache(k, v, kc, vc, bt[b0:b1].contiguous(), cl[b0:b1], BS,
                                       k_scales=ks, v_scales=vs, k_scale=kf, v_scale=vf)
        del k, v
    ops.check_status()
    return q, bt, cl, caches


def _oracle_seq(q_row, kc, vc, ks, vs, bt_row, ctx, acc):
    """Oracle decode of one sequence from its pages (copied to the host)."""
    nblk = (ctx + BS - 1) // BS
    idx = bt_row[:nblk].long()
    f8 = kc.dtype == torch.float8_e4m3fn
    kp = (kc.view(torch.uint8) if f8 else kc)[idx].cpu().numpy()
    vp = (vc.view(torch.uint8) if f8 else vc)[idx].cpu().numpy()
    if ks is not None:
        ksp, vsp = ks[idx].cpu().numpy(), vs[idx].cpu().numpy()
        deq = pa_oracle.dequantize_fp8 if f8 else pa_oracle.dequantize_kv
        kp, vp = deq(kp, vp, ksp, vsp)
    bt1 = np.arange(nblk, dtype=np.int32)[None]
    return pa_oracle.paged_decode_attention(q_row[None], kp, vp, bt1,
                                            np.array([ctx], np.int32), scale=SCALE, acc=acc)[0]


def _check(out, q, bt, cl, kc, vc, ks, vs, seqs=None, acc=np.float64):
    qh = q.cpu().numpy()
    lens = cl.cpu().numpy()
    outh = out.float().cpu()
    for b in (range(len(lens)) if seqs is None else seqs):
        ref = _oracle_seq(qh[b], kc, vc, ks, vs, bt[b], int(lens[b]), acc)
        torch.testing.assert_close(outh[b], torch.from_numpy(ref), atol=ATOL, rtol=RTOL,
                                   msg=lambda m: f"sequence {b} (ctx {lens[b]}): {m}")


def _run(name, q, bt, cl, kc, vc, ks=None, vs=None):
    from pa_b200 import cuda_ext, ops
    out = torch.full_like(q, float("nan"))
    if ks is None:
        cuda_ext.VARIANTS[name](out, q, kc, vc, bt, cl, SCALE, BS)
    elif kc.dtype == torch.int8:
        cuda_ext.VARIANTS_INT8[name](out, q, kc, vc, ks, vs, bt, cl, SCALE, BS)
    else:
        ops.decode(out, q, kc, vc, bt, cl, SCALE, BS, k_scales=ks, v_scales=vs,
                   splitk=(name == "splitk"))
    torch.cuda.synchronize()
    ops.check_status()
    return out


def test_config2_fp16_full_size():
    q, bt, cl, caches = _build([4096] * 64, 32, 8, ["f16"], "normal", seed=202,
                               extra_blocks=16384 - 64 * 256)
    kc, vc, _, _, _, _ = caches["f16"]
    assert kc.shape[0] == 16384
    for name in ("warp", "splitk"):
        out = _run(name, q, bt, cl, kc, vc)
        _check(out, q, bt, cl, kc, vc, None, None)


@pytest.fixture(scope="module")
def config3():
    q, bt, cl, caches = _build([8192] * 64, 12, 2, ["i8", "i8pt", "f16", "f8"],
                               "lognormal_outlier", seed=303)
    yield q, bt, cl, caches
    del caches
    torch.cuda.empty_cache()


@pytest.mark.parametrize("name", ["warp_int8", "splitk_int8"])
def test_config3_int8_per_token_full_size(config3, name):
    q, bt, cl, caches = config3
    kc, vc, ks, vs, _, _ = caches["i8"]
    _check(_run(name, q, bt, cl, kc, vc, ks, vs), q, bt, cl, kc, vc, ks, vs)


def test_config3_int8_per_tensor_full_size(config3):
    q, bt, cl, caches = config3
    kc, vc, ks, vs, kf, vf = caches["i8pt"]
    # Every written scale slot holds the one per-tensor scale.
    nblk = int(cl[0].item()) // BS
    assert bool((ks[bt[0, :nblk].long()] == kf).all())
    _check(_run("warp_int8", q, bt, cl, kc, vc, ks, vs), q, bt, cl, kc, vc, ks, vs)


def test_config3_fp16_and_fp8_same_rows_full_size(config3):
    q, bt, cl, caches = config3
    kc, vc, _, _, _, _ = caches["f16"]
    _check(_run("warp", q, bt, cl, kc, vc), q, bt, cl, kc, vc, None, None)
    kc, vc, ks, vs, _, _ = caches["f8"]
    _check(_run("warp", q, bt, cl, kc, vc, ks, vs), q, bt, cl, kc, vc, ks, vs)


@pytest.mark.parametrize("name", ["splitk_int8", "warp_int8"])
def test_config4_long_context_int8(name):
    q, bt, cl, caches = _build([131072, 65537, 131072], 64, 8, ["i8"], "lognormal_outlier",
                               seed=404)
    kc, vc, ks, vs, _, _ = caches["i8"]
    out = _run(name, q, bt, cl, kc, vc, ks, vs)
    _check(out, q, bt, cl, kc, vc, ks, vs, acc=np.float32)


def test_config5_ragged_batch_int8_full_size():
    rng = np.random.default_rng(99)
    lens = np.clip(np.exp(rng.normal(math.log(2048), 1.0, size=256)), 16, 32768).astype(np.int64)
    q, bt, cl, caches = _build(lens, 28, 4, ["i8"], "lognormal_outlier", seed=505)
    kc, vc, ks, vs, _, _ = caches["i8"]
    _check(_run("warp_int8", q, bt, cl, kc, vc, ks, vs), q, bt, cl, kc, vc, ks, vs)
