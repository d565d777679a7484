"""GPU: the allocation-free FP16 decode entry point, pa_decode_f16_noalloc, through the C ABI.

Some callers cannot allocate device memory at the moment they run attention: plugins whose
host framework owns all device memory, and serving loops that must stay out of any
allocator. They call this entry point, which
keeps its scratch in a static device array instead of a caller-provided workspace. Its
output must match the regular entry point's (pa_decode_f16 with a workspace) on the same
inputs, on two calls in a row: the second call reuses the array the first one left behind.
This file is collected last so that a run stopping at the first failure has run the others.
"""

import pytest
import torch

import pa_oracle
from pa_testlib import ATOL, RTOL, fp16_case, scale_for, to_cuda

pytestmark = pytest.mark.gpu


def _lib():
    from pa_b200 import _lib
    return _lib, _lib.lib()


def test_noalloc_matches_workspace_entry_point_twice():
    L, lib = _lib()
    c = fp16_case(31, 5, 32, 8, [4096, 700, 33, 1, 2500])
    q, kc, vc, bt, cl = to_cuda(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                c["context_lens"])
    B, H, D = q.shape
    NB, KVH = kc.shape[0], kc.shape[1]
    mb = bt.shape[1]
    sc = scale_for()
    stream = torch.cuda.current_stream().cuda_stream
    need = lib.pa_decode_workspace_bytes(B, H, KVH, D, mb, 16, L.PA_DTYPE_F16, 0)
    assert need > 0
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    ref = torch.empty_like(q)
    rc = lib.pa_decode_f16(ref.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                           bt.data_ptr(), cl.data_ptr(), B, H, KVH, D, NB, 16, mb, sc,
                           ws.data_ptr(), need, stream)
    assert rc == 0, lib.pa_last_error()
    oracle = pa_oracle.paged_decode_attention(c["q"], c["k_cache"], c["v_cache"],
                                              c["block_table"], c["context_lens"])
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        rc = lib.pa_decode_f16_noalloc(out.data_ptr(), q.data_ptr(), kc.data_ptr(),
                                       vc.data_ptr(), bt.data_ptr(), cl.data_ptr(), B, H, KVH,
                                       D, NB, 16, mb, sc, stream)
        assert rc == 0, lib.pa_last_error()
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), ref.float(), atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(out.float().cpu(), torch.from_numpy(oracle), atol=ATOL,
                                   rtol=RTOL)


def test_noalloc_rejects_shapes_beyond_its_scratch():
    """16 q heads per kv head need larger partial slots than the static scratch holds: the
    call is refused on the host with PA_ERR_WORKSPACE and nothing is launched."""
    L, lib = _lib()
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.pa_decode_f16_noalloc(1 << 20, 1 << 20, 1 << 20, 1 << 20, 1 << 20, 1 << 20, 4,
                                   32, 2, 128, 64, 16, 8, 0.1, stream)
    assert rc == L.PA_ERR_WORKSPACE
    assert b"static scratch" in lib.pa_last_error()
