"""GPU: the FP8 (e4m3, per-token fp32 scale) KV cache. The cache write is compared bit for bit
with the oracle's quantiser; the decode ops (single pass and split-K) against the oracle on the
dequantised cache, including a page whose slots past the context hold NaN encodings."""

import numpy as np
import pytest
import torch

import pa_oracle
from pa_testlib import BLOCK_SIZE, assert_close, fp16_case, oracle_out, scale_for, to_cuda

pytestmark = pytest.mark.gpu


def _ops():
    from pa_b200 import ops
    return ops


def _fp8_case(c, pad_byte=0):
    """Oracle-quantised e4m3 cache of a case (slots past each context hold pad_byte)."""
    k, v, lens, bt, nb = c["k"], c["v"], c["context_lens"], c["block_table"], c["num_blocks"]
    KVH = k.shape[2]
    kq, ks = pa_oracle.quantize_per_token_fp8(k)
    vq, vs = pa_oracle.quantize_per_token_fp8(v)
    kc, vc = pa_oracle.scatter_paged_cache(kq, vq, lens, bt, nb, BLOCK_SIZE)
    if pad_byte:
        used = np.zeros((nb, BLOCK_SIZE), dtype=bool)
        for b, n in enumerate(lens):
            t = np.arange(int(n))
            used[bt[b, t // BLOCK_SIZE], t % BLOCK_SIZE] = True
        kc = np.where(used[:, None, None, :, None], kc, np.uint8(pad_byte)).astype(np.uint8)
        vc = np.where(used[:, None, None, :], vc, np.uint8(pad_byte)).astype(np.uint8)
    kss = pa_oracle.scatter_scales(ks, lens, bt, nb, KVH, BLOCK_SIZE)
    vss = pa_oracle.scatter_scales(vs, lens, bt, nb, KVH, BLOCK_SIZE)
    return kc, vc, kss, vss


def _to_fp8(a):
    return torch.from_numpy(np.ascontiguousarray(a)).view(torch.float8_e4m3fn).cuda()


@pytest.mark.parametrize("splitk", [False, True])
@pytest.mark.parametrize("lens,heads", [([1, 17, 500], (8, 2)), ([1500, 33], (32, 8)),
                                        ([700, 4096], (12, 2)), ([300, 64], (32, 2))])
def test_fp8_decode_matches_dequant_oracle(splitk, lens, heads):
    H, KVH = heads
    c = fp16_case(81, len(lens), H, KVH, lens)
    kc, vc, ks, vs = _fp8_case(c)
    q, bt, cl, kss, vss = to_cuda(c["q"], c["block_table"], c["context_lens"], ks, vs)
    out = torch.empty_like(q)
    _ops().decode(out, q, _to_fp8(kc), _to_fp8(vc), bt, cl, scale_for(), BLOCK_SIZE,
                  k_scales=kss, v_scales=vss, splitk=splitk)
    kd, vd = pa_oracle.dequantize_fp8(kc, vc, ks, vs)
    assert_close(out, oracle_out(c["q"], kd, vd, c["block_table"], c["context_lens"]))
    _ops().check_status(q.device)


def test_fp8_decode_ignores_nan_bytes_past_the_context():
    c = fp16_case(82, 2, 8, 2, [23, 41])  # both contexts end inside a page
    kc, vc, ks, vs = _fp8_case(c, pad_byte=0x7F)  # 0x7F is an e4m3 NaN
    q, bt, cl, kss, vss = to_cuda(c["q"], c["block_table"], c["context_lens"], ks, vs)
    out = torch.empty_like(q)
    _ops().decode(out, q, _to_fp8(kc), _to_fp8(vc), bt, cl, scale_for(), BLOCK_SIZE,
                  k_scales=kss, v_scales=vss)
    assert torch.isfinite(out).all()
    kd, vd = pa_oracle.dequantize_fp8(kc, vc, ks, vs)
    assert_close(out, oracle_out(c["q"], kd, vd, c["block_table"], c["context_lens"]))


@pytest.mark.parametrize("splitk", [False, True])
def test_fp8_cache_with_bf16_q(splitk):
    """bf16 q and out over an FP8 cache (pa_decode_bf16q with PA_DTYPE_FP8E4M3)."""
    c = fp16_case(84, 3, 12, 2, [1, 600, 37])
    kc, vc, ks, vs = _fp8_case(c)
    qb = torch.from_numpy(np.ascontiguousarray(c["q"])).to(torch.bfloat16)
    q = qb.cuda()
    bt, cl, kss, vss = to_cuda(c["block_table"], c["context_lens"], ks, vs)
    out = torch.empty_like(q)
    _ops().decode_bf16(out, q, _to_fp8(kc), _to_fp8(vc), bt, cl, scale_for(), BLOCK_SIZE,
                       k_scales=kss, v_scales=vss, splitk=splitk)
    assert out.dtype == torch.bfloat16
    kd, vd = pa_oracle.dequantize_fp8(kc, vc, ks, vs)
    assert_close(out, oracle_out(qb.float().numpy(), kd, vd, c["block_table"],
                                 c["context_lens"]))
    _ops().check_status(q.device)


@pytest.mark.parametrize("in_dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_fp8_cache_write_is_bit_exact(in_dtype):
    rng = np.random.default_rng(5)
    N, KVH, D, NB = 37, 4, 128, 12
    k = (rng.standard_normal((N, KVH, D)) * 3).astype(np.float32)
    v = (rng.standard_normal((N, KVH, D)) * 0.5).astype(np.float32)
    k[3] = 0.0             # zero rows: scale 0, zeros
    v[5, 1, :7] = 1e4      # a large value, the row max maps to 448
    kt = torch.from_numpy(k).to(in_dtype)
    vt = torch.from_numpy(v).to(in_dtype)
    kin = kt.float().numpy()
    vin = vt.float().numpy()
    slots = rng.permutation(NB * BLOCK_SIZE)[:N].astype(np.int32)
    slots[7] = -1          # a padding token: skipped
    kc = torch.zeros((NB, KVH, D // 8, BLOCK_SIZE, 8), dtype=torch.uint8).view(
        torch.float8_e4m3fn).cuda()
    vc = torch.zeros((NB, KVH, D, BLOCK_SIZE), dtype=torch.uint8).view(torch.float8_e4m3fn).cuda()
    ksc = torch.zeros((NB, KVH, BLOCK_SIZE), dtype=torch.float32, device="cuda")
    vsc = torch.zeros_like(ksc)
    _ops().quantize_into_cache(kt.cuda(), vt.cuda(), kc, vc, ksc, vsc,
                               torch.from_numpy(slots).cuda(), BLOCK_SIZE)
    torch.cuda.synchronize()
    kq, ks = pa_oracle.quantize_per_token_fp8(kin)
    vq, vs = pa_oracle.quantize_per_token_fp8(vin)
    kcache = kc.view(torch.uint8).cpu().numpy()
    vcache = vc.view(torch.uint8).cpu().numpy()
    kscale = ksc.cpu().numpy()
    vscale = vsc.cpu().numpy()
    for n in range(N):
        if slots[n] < 0:
            continue
        blk, off = divmod(int(slots[n]), BLOCK_SIZE)
        assert np.array_equal(kcache[blk, :, :, off, :].reshape(KVH, D), kq[n])
        assert np.array_equal(vcache[blk, :, :, off], vq[n])
        assert np.array_equal(kscale[blk, :, off], ks[n])
        assert np.array_equal(vscale[blk, :, off], vs[n])


def test_reference_named_int8_ops_reject_an_fp8_cache():
    """The drop-in names keep the reference's dtype contract: its INT8 ops take int8 caches
    only, so an e4m3 cache is rejected there (it is decoded through ops.decode)."""
    from pa_b200 import cuda_ext
    c = fp16_case(83, 1, 8, 2, [40])
    kc, vc, ks, vs = _fp8_case(c)
    q, bt, cl, kss, vss = to_cuda(c["q"], c["block_table"], c["context_lens"], ks, vs)
    with pytest.raises(RuntimeError, match="k_cache must be int8"):
        cuda_ext.VARIANTS_INT8["warp_int8"](torch.empty_like(q), q, _to_fp8(kc), _to_fp8(vc),
                                            kss, vss, bt, cl, scale_for(), BLOCK_SIZE)
    with pytest.raises(RuntimeError, match="k_cache must be fp16"):
        cuda_ext.VARIANTS["warp"](torch.empty_like(q), q, _to_fp8(kc), _to_fp8(vc), bt, cl,
                                  scale_for(), BLOCK_SIZE)
