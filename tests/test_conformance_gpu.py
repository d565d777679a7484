"""GPU: inputs the reference's launchers accept and this build refuses, refused cleanly.

The reference's FP16 launchers accept any block_size that is a multiple of 8 and divides their
tile (kernels/paged_attention_v3_warp.cu:149, paged_attention_v4_splitk.cu:203) and any
head_dim, and they do not check contiguity. This build's decode kernels take 16-token subpages
and head_dim 128, and read tensors as contiguous; anything else is refused before any launch,
with a RuntimeError naming the limit (Python names) or PA_ERR_INVALID_ARG / PA_ERR_UNSUPPORTED
(C ABI). No reference test or bench uses the refused forms. These are the only differences in
what is accepted; everything else the reference accepts is run by its own tests, unchanged,
against these names.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _fp16_inputs(bs=16, D=128, NB=8, B=2, H=8, KVH=2):
    q = torch.randn(B, H, D, dtype=torch.float16, device="cuda")
    kc = torch.randn(NB, KVH, D // 8, bs, 8, dtype=torch.float16, device="cuda")
    vc = torch.randn(NB, KVH, D, bs, dtype=torch.float16, device="cuda")
    bt = torch.arange(B * (NB // B), dtype=torch.int32, device="cuda").view(B, -1)
    cl = torch.full((B,), bs, dtype=torch.int32, device="cuda")
    return q, kc, vc, bt, cl


@pytest.mark.parametrize("name", ["naive", "vec", "online", "warp", "splitk"])
def test_fp16_block_size_8_is_refused(name):
    from pa_b200 import cuda_ext
    q, kc, vc, bt, cl = _fp16_inputs(bs=8)
    out = torch.empty_like(q)
    with pytest.raises(RuntimeError, match="block_size"):
        cuda_ext.VARIANTS[name](out, q, kc, vc, bt, cl, 0.088, 8)


def test_head_dim_other_than_128_is_refused():
    from pa_b200 import cuda_ext
    q, kc, vc, bt, cl = _fp16_inputs(D=64)
    out = torch.empty_like(q)
    with pytest.raises(RuntimeError, match="head_dim"):
        cuda_ext.VARIANTS["warp"](out, q, kc, vc, bt, cl, 0.125, 16)


def test_non_contiguous_tensors_are_refused():
    from pa_b200 import cuda_ext
    q, kc, vc, bt, cl = _fp16_inputs()
    qt = torch.randn(q.shape[1], q.shape[0], q.shape[2], dtype=torch.float16,
                     device="cuda").transpose(0, 1)
    out = torch.empty_like(q)
    with pytest.raises(RuntimeError, match="contiguous"):
        cuda_ext.VARIANTS["warp"](out, qt, kc, vc, bt, cl, 0.088, 16)


def test_c_abi_codes_for_the_refused_forms():
    from pa_b200 import _lib
    L = _lib.lib()
    p = 1 << 20
    rc = L.pa_decode_f16(p, p, p, p, p, p, 1, 8, 2, 128, 4, 8, 2, 0.1, p, 1 << 30, None)
    assert rc == _lib.PA_ERR_INVALID_ARG and b"block_size" in L.pa_last_error()
    rc = L.pa_decode_f16(p, p, p, p, p, p, 1, 8, 2, 64, 4, 16, 2, 0.1, p, 1 << 30, None)
    assert rc == _lib.PA_ERR_UNSUPPORTED and b"head_dim" in L.pa_last_error()
