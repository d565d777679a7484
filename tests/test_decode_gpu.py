"""GPU parity: decode kernels vs the numpy oracle on identical seeded inputs.

Mirrors the reference's test matrix (tests/test_paged_decode_attn.py): every variant name,
CONTEXT_LENS x GQA x NUM_SEQS, long contexts across split boundaries, INT8 per-token and
per-tensor against the dequantised-cache oracle, finite outputs, ctx=0 rejection, and the
precision metrics; tolerance tightened to the north-star 2e-3 abs / 1e-2 rel.
"""


import numpy as np
import pytest
import torch

import pa_oracle
from pa_testlib import (BLOCK_SIZE, assert_close, fp16_case, int8_case, make_lens, oracle_out,
                        ragged_case, ragged_int8, scale_for, to_cuda)

pytestmark = pytest.mark.gpu

CONTEXT_LENS = [1, 15, 16, 17, 31, 128, 500]
GQA = [(8, 8), (8, 2), (8, 1), (16, 4)]
NUM_SEQS = [1, 3]
LONG_CONTEXT_LENS = [512, 513, 1024, 2000, 4096]
VARIANTS = ["naive", "vec", "online", "warp", "splitk"]
VARIANTS_INT8 = ["warp_int8", "splitk_int8"]


def _ext():
    from pa_b200 import cuda_ext
    return cuda_ext


def _run_fp16(variant, c, scale=None, block_size=BLOCK_SIZE):
    q, kc, vc, bt, cl = to_cuda(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                c["context_lens"])
    out = torch.empty_like(q)
    _ext().VARIANTS[variant](out, q, kc, vc, bt, cl, scale or scale_for(), block_size)
    return out


def _run_int8(variant, c, qc, block_size=BLOCK_SIZE):
    q, bt, cl = to_cuda(c["q"], c["block_table"], c["context_lens"])
    kc, vc, ks, vs = to_cuda(qc["k_cache"], qc["v_cache"], qc["k_scales"], qc["v_scales"])
    out = torch.empty_like(q)
    _ext().VARIANTS_INT8[variant](out, q, kc, vc, ks, vs, bt, cl, scale_for(), block_size)
    return out


def _int8_oracle(c, qc):
    kd, vd = pa_oracle.dequantize_kv(qc["k_cache"], qc["v_cache"], qc["k_scales"],
                                     qc["v_scales"])
    return oracle_out(c["q"], kd, vd, c["block_table"], c["context_lens"])


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("clen", CONTEXT_LENS)
@pytest.mark.parametrize("num_heads,num_kv_heads", GQA)
@pytest.mark.parametrize("num_seqs", NUM_SEQS)
def test_fp16_matches_oracle(variant, clen, num_heads, num_kv_heads, num_seqs):
    c = fp16_case(0, num_seqs, num_heads, num_kv_heads, make_lens(clen, num_seqs))
    out = _run_fp16(variant, c)
    ref = oracle_out(c["q"], c["k_cache"], c["v_cache"], c["block_table"], c["context_lens"])
    assert_close(out, ref)


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("clen", LONG_CONTEXT_LENS)
@pytest.mark.parametrize("num_heads,num_kv_heads", [(8, 8), (8, 2)])
def test_fp16_long_contexts(variant, clen, num_heads, num_kv_heads):
    c = fp16_case(1, 2, num_heads, num_kv_heads, make_lens(clen, 2))
    out = _run_fp16(variant, c)
    ref = oracle_out(c["q"], c["k_cache"], c["v_cache"], c["block_table"], c["context_lens"])
    assert_close(out, ref)


@pytest.mark.parametrize("variant", VARIANTS_INT8)
@pytest.mark.parametrize("mode", ["per_token", "per_tensor"])
@pytest.mark.parametrize("clen", CONTEXT_LENS)
@pytest.mark.parametrize("num_heads,num_kv_heads", GQA)
@pytest.mark.parametrize("num_seqs", NUM_SEQS)
def test_int8_matches_dequant_oracle(variant, mode, clen, num_heads, num_kv_heads, num_seqs):
    c = fp16_case(0, num_seqs, num_heads, num_kv_heads, make_lens(clen, num_seqs))
    qc = int8_case(c, mode)
    assert_close(_run_int8(variant, c, qc), _int8_oracle(c, qc))


@pytest.mark.parametrize("variant", VARIANTS_INT8)
@pytest.mark.parametrize("mode", ["per_token", "per_tensor"])
@pytest.mark.parametrize("clen", LONG_CONTEXT_LENS)
@pytest.mark.parametrize("num_heads,num_kv_heads", [(8, 8), (8, 2)])
def test_int8_long_contexts(variant, mode, clen, num_heads, num_kv_heads):
    c = fp16_case(1, 2, num_heads, num_kv_heads, make_lens(clen, 2), dist="lognormal_outlier")
    qc = int8_case(c, mode)
    assert_close(_run_int8(variant, c, qc), _int8_oracle(c, qc))


# GQA shapes of the BASELINE configs and the head-tile paths: G = 4, 6, 7, 8 (one 8-row
# tile), 12 and 16 (one 16-row tile), 20 and 32 (two 16-row tiles).
@pytest.mark.parametrize("num_heads,num_kv_heads", [(32, 8), (12, 2), (28, 4), (64, 8),
                                                    (12, 1), (16, 1), (40, 2), (32, 1)])
@pytest.mark.parametrize("kind", ["fp16", "int8"])
@pytest.mark.parametrize("splitk", [False, True])
def test_gqa_shapes(num_heads, num_kv_heads, kind, splitk):
    lens = [700, 33, 1, 1500]
    c = ragged_case(2, num_heads, num_kv_heads, lens, dist="lognormal_outlier")
    if kind == "fp16":
        out = _run_fp16("splitk" if splitk else "warp", c)
        ref = oracle_out(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                         c["context_lens"])
    else:
        qc = ragged_int8(c)
        out = _run_int8("splitk_int8" if splitk else "warp_int8", c, qc)
        ref = _int8_oracle(c, qc)
    assert_close(out, ref)


@pytest.mark.parametrize("block_size", [32, 64, 128])
@pytest.mark.parametrize("kind", ["fp16", "int8"])
def test_block_sizes(block_size, kind):
    lens = [1, 17, 100, 300, 1029]
    c = fp16_case(3, 5, 8, 2, lens, block_size=block_size)
    if kind == "fp16":
        for v in ("warp", "splitk"):
            out = _run_fp16(v, c, block_size=block_size)
            assert_close(out, oracle_out(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                         c["context_lens"]))
    else:
        qc = int8_case(c, "per_token", block_size=block_size)
        for v in VARIANTS_INT8:
            assert_close(_run_int8(v, c, qc, block_size=block_size), _int8_oracle(c, qc))


@pytest.mark.parametrize("kind", ["fp16", "int8"])
def test_ragged_batch_many_sequences(kind):
    """A serving-like ragged batch: page ranges of warps cut through many sequences, so the
    cross-warp combine path is exercised heavily."""
    g = np.random.default_rng(5)
    lens = np.clip(np.exp(g.normal(np.log(300), 1.0, size=150)), 1, 5000).astype(int).tolist()
    c = ragged_case(4, 28, 4, lens)
    if kind == "fp16":
        out = _run_fp16("warp", c)
        ref = oracle_out(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                         c["context_lens"])
    else:
        qc = ragged_int8(c)
        out = _run_int8("warp_int8", c, qc)
        ref = _int8_oracle(c, qc)
    assert_close(out, ref)


def test_batch_larger_than_one_launch():
    lens = [(i * 7) % 40 + 1 for i in range(1100)]
    c = fp16_case(6, len(lens), 8, 2, lens)
    for v in ("warp", "splitk"):
        out = _run_fp16(v, c)
        assert_close(out, oracle_out(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                     c["context_lens"]))


def test_single_pass_and_splitk_agree():
    c = fp16_case(7, 3, 16, 4, [3000, 2049, 17])
    a = _run_fp16("warp", c).float()
    b = _run_fp16("splitk", c).float()
    torch.testing.assert_close(a, b, atol=2e-3, rtol=1e-2)


def test_repeated_calls_are_stable():
    """The arrival counters reset themselves: many back-to-back calls give the same result."""
    c = fp16_case(8, 2, 8, 1, [6000, 3000])
    q, kc, vc, bt, cl = to_cuda(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                c["context_lens"])
    outs = []
    for _ in range(5):
        out = torch.empty_like(q)
        _ext().VARIANTS["warp"](out, q, kc, vc, bt, cl, scale_for(), BLOCK_SIZE)
        outs.append(out)
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


def test_custom_scale():
    c = fp16_case(9, 2, 8, 2, [200, 90])
    out = _run_fp16("warp", c, scale=0.05)
    assert_close(out, oracle_out(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                 c["context_lens"], scale=0.05))


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("clen", [1, 17, 4096])
def test_outputs_finite(variant, clen):
    c = fp16_case(0, 2, 8, 2, make_lens(clen, 2))
    assert torch.isfinite(_run_fp16(variant, c)).all()


@pytest.mark.parametrize("variant", VARIANTS_INT8)
@pytest.mark.parametrize("clen", [1, 17, 4096])
def test_int8_outputs_finite(variant, clen):
    c = fp16_case(0, 2, 8, 2, make_lens(clen, 2))
    assert torch.isfinite(_run_int8(variant, c, int8_case(c, "per_token"))).all()


@pytest.mark.parametrize("variant", VARIANTS)
def test_empty_context_rejected(variant):
    c = fp16_case(0, 2, 8, 2, [8, 1])
    q, kc, vc, bt = to_cuda(c["q"], c["k_cache"], c["v_cache"], c["block_table"])
    lens = torch.tensor([8, 0], dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    with pytest.raises(RuntimeError):
        _ext().VARIANTS[variant](out, q, kc, vc, bt, lens, scale_for(), BLOCK_SIZE)


@pytest.mark.parametrize("variant", VARIANTS_INT8)
def test_int8_empty_context_rejected(variant):
    c = fp16_case(0, 2, 8, 2, [8, 1])
    qc = int8_case(c, "per_token")
    q, bt = to_cuda(c["q"], c["block_table"])
    kc, vc, ks, vs = to_cuda(qc["k_cache"], qc["v_cache"], qc["k_scales"], qc["v_scales"])
    lens = torch.tensor([8, 0], dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    with pytest.raises(RuntimeError):
        _ext().VARIANTS_INT8[variant](out, q, kc, vc, ks, vs, bt, lens, scale_for(), BLOCK_SIZE)


def test_wrong_dtypes_rejected():
    c = fp16_case(0, 1, 8, 2, [20])
    q, kc, vc, bt, cl = to_cuda(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                c["context_lens"])
    out = torch.empty_like(q)
    f = _ext().VARIANTS["warp"]
    with pytest.raises(RuntimeError, match="q must be fp16"):
        f(out, q.float(), kc, vc, bt, cl, 0.1, 16)
    with pytest.raises(RuntimeError, match="block_table must be int32"):
        f(out, q, kc, vc, bt.long(), cl, 0.1, 16)
    with pytest.raises(RuntimeError, match="context_lens must be int32"):
        f(out, q, kc, vc, bt, cl.long(), 0.1, 16)
    with pytest.raises(RuntimeError, match="block_size"):
        f(out, q, kc, vc, bt, cl, 0.1, 8)
    with pytest.raises(RuntimeError, match="k_cache must be int8"):
        _ext().VARIANTS_INT8["warp_int8"](out, q, kc, vc, kc.float(), vc.float(), bt, cl, 0.1,
                                          16)


def test_unread_table_entries_are_ignored():
    """Entries past a sequence's last block are never read (garbage there is harmless)."""
    from pa_b200 import ops
    c = fp16_case(10, 2, 8, 2, [40, 17], max_blocks=6)
    bt = c["block_table"].copy()
    bt[0, 3:] = -7
    bt[1, 2:] = 1 << 30
    c["block_table"] = bt
    ops.read_status()
    out = _run_fp16("warp", c)
    assert ops.read_status() == 0
    assert_close(out, oracle_out(c["q"], c["k_cache"], c["v_cache"], bt, c["context_lens"]))


def test_bad_block_id_is_flagged_not_faulted():
    """A block id outside the cache inside the context is clamped on the device and
    reported through the status word; no out-of-bounds access happens."""
    from pa_b200 import ops
    c = fp16_case(11, 2, 8, 2, [40, 17])
    c["block_table"] = c["block_table"].copy()
    c["block_table"][0, 1] = c["num_blocks"] + 5
    ops.read_status()
    out = _run_fp16("warp", c)
    torch.cuda.synchronize()
    assert ops.read_status() & 64  # PA_ERR_BLOCK_ID
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("variant", VARIANTS_INT8)
@pytest.mark.parametrize("clen", [128, 500])
@pytest.mark.parametrize("num_heads,num_kv_heads", [(8, 8), (8, 2)])
def test_int8_precision_metric(variant, clen, num_heads, num_kv_heads):
    """Per-token INT8 error vs FP16 is small and no worse than per-tensor
    (tests/test_paged_decode_attn.py:256-306)."""
    c = fp16_case(0, 2, num_heads, num_kv_heads, make_lens(clen, 2))
    fp16 = _run_fp16("warp", c).float()

    def rel(mode):
        out = _run_int8(variant, c, int8_case(c, mode)).float()
        return ((out - fp16).abs() / fp16.abs().clamp_min(1e-3)).mean().item()

    pt, ptn = rel("per_token"), rel("per_tensor")
    assert pt < 0.2
    assert pt <= ptn + 1e-3


@pytest.mark.parametrize("variant", VARIANTS_INT8)
def test_int8_precision_outlier_distribution(variant):
    """Per-token stays close to FP16 under outlier K channels and beats per-tensor
    (tests/test_paged_decode_attn.py:419-464; channels [3, 50, 97] x20)."""
    c = fp16_case(0, 2, 8, 2, make_lens(500, 2))
    k = c["k"].astype(np.float32)
    k[:, :, :, [3, 50, 97]] *= 20.0
    c["k"] = k.astype(np.float16)
    c["k_cache"], c["v_cache"] = pa_oracle.scatter_paged_cache(
        c["k"], c["v"], c["context_lens"], c["block_table"], c["num_blocks"])
    fp16 = _run_fp16("warp", c).float().flatten()

    def cos(mode):
        out = _run_int8(variant, c, int8_case(c, mode)).float().flatten()
        return (out @ fp16 / (out.norm() * fp16.norm() + 1e-12)).item()

    pt, ptn = cos("per_token"), cos("per_tensor")
    assert pt > 0.99
    assert pt >= ptn - 1e-4


def test_golden_cfg1_on_gpu():
    """BASELINE config 1 through the GPU against the reference's own outputs."""
    import os
    gold = np.load(os.path.join(os.path.dirname(__file__), "golden", "decode_cfg1.npz"))
    import gen
    lens = gen.Gen(1).randint(64, 513, (4,))
    c = gen.decode_case(seed=101, num_seqs=4, num_heads=12, num_kv_heads=2, context_lens=lens,
                        num_blocks=256)
    c["k_cache"], c["v_cache"] = pa_oracle.scatter_paged_cache(
        c["k"], c["v"], c["context_lens"], c["block_table"], c["num_blocks"])
    for v in VARIANTS:
        assert_close(_run_fp16(v, c), gold["out_f16"])
    for mode in ("per_token", "per_tensor"):
        qc = int8_case(c, mode)
        for v in VARIANTS_INT8:
            assert_close(_run_int8(v, c, qc), gold[f"out_{mode}"])
