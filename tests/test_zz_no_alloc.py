"""GPU: the allocation-free FP16 decode entry point, pa_decode_f16_noalloc, through the C ABI.

Some callers cannot allocate device memory at the moment they run attention: plugins whose
host framework owns all device memory, and serving loops that must stay out of any
allocator. They call this entry point, which keeps its scratch in a static device array
instead of a caller-provided workspace. Its output must match the regular entry point's
(pa_decode_f16 with a workspace) on the same inputs, on two calls in a row: the second call
reuses the array the first one left behind. A second shape (other block size, kv heads and
group size) follows the first on the same array, and errors the kernel finds on the device
are read back through pa_decode_f16_noalloc_read_status.
This file is collected last so that a run stopping at the first failure has run the others.
"""

import ctypes

import pytest
import torch

import pa_oracle
from pa_testlib import ATOL, RTOL, fp16_case, scale_for, to_cuda

pytestmark = pytest.mark.gpu

# (seed, num_seqs, num_heads, num_kv_heads, context_lens, block_size)
SHAPES = [
    (31, 5, 32, 8, [4096, 700, 33, 1, 2500], 16),
    (32, 3, 21, 3, [1500, 64, 3001], 32),
]


def _lib():
    from pa_b200 import _lib
    return _lib, _lib.lib()


def _read_status(lib, stream):
    st = ctypes.c_int(-1)
    assert lib.pa_decode_f16_noalloc_read_status(ctypes.byref(st), stream) == 0, \
        lib.pa_last_error()
    return st.value


def _noalloc(lib, out, q, kc, vc, bt, cl, bs, stream):
    B, H, D = q.shape
    return lib.pa_decode_f16_noalloc(out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                     bt.data_ptr(), cl.data_ptr(), B, H, kc.shape[1], D,
                                     kc.shape[0], bs, bt.shape[1], scale_for(), stream)


def _check_shape(shape):
    L, lib = _lib()
    seed, B, H, KVH, lens, bs = shape
    c = fp16_case(seed, B, H, KVH, lens, block_size=bs)
    q, kc, vc, bt, cl = to_cuda(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                c["context_lens"])
    D = q.shape[2]
    NB = kc.shape[0]
    mb = bt.shape[1]
    stream = torch.cuda.current_stream().cuda_stream
    need = lib.pa_decode_workspace_bytes(B, H, KVH, D, mb, bs, L.PA_DTYPE_F16, 0)
    assert need > 0
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    ref = torch.empty_like(q)
    rc = lib.pa_decode_f16(ref.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                           bt.data_ptr(), cl.data_ptr(), B, H, KVH, D, NB, bs, mb, scale_for(),
                           ws.data_ptr(), need, stream)
    assert rc == 0, lib.pa_last_error()
    oracle = pa_oracle.paged_decode_attention(c["q"], c["k_cache"], c["v_cache"],
                                              c["block_table"], c["context_lens"])
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        rc = _noalloc(lib, out, q, kc, vc, bt, cl, bs, stream)
        assert rc == 0, lib.pa_last_error()
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), ref.float(), atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(out.float().cpu(), torch.from_numpy(oracle), atol=ATOL,
                                   rtol=RTOL)
    assert _read_status(lib, stream) == 0


def test_noalloc_matches_workspace_entry_point_twice():
    _check_shape(SHAPES[0])


def test_noalloc_second_shape_after_the_first():
    """Block size 32, 3 kv heads of 7 q heads each, on the array the previous shape used."""
    _check_shape(SHAPES[1])
    _check_shape(SHAPES[0])


def test_noalloc_reports_device_errors():
    """A block_table entry outside the cache is flagged on the device (the read is clamped,
    nothing faults) and comes back through the status reader, which then clears it; the next
    good call on the same array is correct and reports nothing."""
    L, lib = _lib()
    seed, B, H, KVH, lens, bs = SHAPES[0]
    c = fp16_case(seed, B, H, KVH, lens, block_size=bs)
    q, kc, vc, bt, cl = to_cuda(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                c["context_lens"])
    stream = torch.cuda.current_stream().cuda_stream
    _read_status(lib, stream)  # start from a clear word
    bad = bt.clone()
    bad[1, 3] = kc.shape[0] + 5
    out = torch.empty_like(q)
    assert _noalloc(lib, out, q, kc, vc, bad, cl, bs, stream) == 0
    st = _read_status(lib, stream)
    assert st & L.PA_ERR_BLOCK_ID, st
    assert _read_status(lib, stream) == 0
    assert _noalloc(lib, out, q, kc, vc, bt, cl, bs, stream) == 0
    torch.cuda.synchronize()
    oracle = pa_oracle.paged_decode_attention(c["q"], c["k_cache"], c["v_cache"],
                                              c["block_table"], c["context_lens"])
    torch.testing.assert_close(out.float().cpu(), torch.from_numpy(oracle), atol=ATOL, rtol=RTOL)
    assert _read_status(lib, stream) == 0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    """16 q heads per kv head need larger partial slots than the static scratch holds: the
    call is refused on the host with PA_ERR_WORKSPACE and nothing is launched."""
    L, lib = _lib()
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.pa_decode_f16_noalloc(1 << 20, 1 << 20, 1 << 20, 1 << 20, 1 << 20, 1 << 20, 4,
                                   32, 2, 128, 64, 16, 8, 0.1, stream)
    assert rc == L.PA_ERR_WORKSPACE
    assert b"static scratch" in lib.pa_last_error()
