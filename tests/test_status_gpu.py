"""GPU: recovery of a decode workspace after a device-side error.

A decode warp that gives up on a bounded wait stops part-way, so arrival counters of the
segments it shared can stay set in its workspace. Reading a non-zero status through
ops.read_status resets the workspace's counters (pa_reset_workspace), and the next decode on
the same workspace is correct. The error is produced without a fault: the bounded-wait
self-test sets PA_ERR_TIMEOUT after about a second, and the counters a stopped decode would
leave behind are written by the test.
"""

import ctypes

import pytest
import torch

from pa_testlib import BLOCK_SIZE, assert_close, fp16_case, oracle_out, scale_for, to_cuda

pytestmark = pytest.mark.gpu


def test_status_read_resets_counters_after_a_timeout():
    from pa_b200 import _lib, ops
    L = _lib.lib()
    c = fp16_case(5, 3, 32, 8, [3000, 2000, 2500])
    q, kc, vc, bt, cl = to_cuda(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                c["context_lens"])
    B, H, D = q.shape
    KVH = kc.shape[1]
    need = L.pa_decode_workspace_bytes(B, H, KVH, D, bt.shape[1], BLOCK_SIZE, _lib.PA_DTYPE_F16,
                                       0)
    ws = ops.workspace(q.device, need)  # the workspace ops.decode uses on this stream
    assert ops.read_status(q.device) == 0
    stream = torch.cuda.current_stream().cuda_stream
    assert L.pa_selftest_bounded_wait(ws.data_ptr(), stream) == _lib.PA_OK
    # Counters as a decode that stopped part-way would leave them (every segment of the batch
    # claims three earlier arrivals).
    ws[256:256 + 4 * B * KVH].view(torch.int32).fill_(3)
    st = ops.read_status(q.device)
    assert st & _lib.PA_ERR_TIMEOUT, st
    assert int(ws[256:256 + 4 * B * KVH].view(torch.int32).abs().sum()) == 0
    out = torch.full_like(q, float("nan"))
    ops.decode(out, q, kc, vc, bt, cl, scale_for(), BLOCK_SIZE)
    assert_close(out, oracle_out(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                 c["context_lens"]))
    assert ops.read_status(q.device) == 0


def test_reset_workspace_zeroes_status_and_counters_only():
    from pa_b200 import _lib
    L = _lib.lib()
    n = (1 << 20) + 256 + 4096
    ws = torch.full((n,), 7, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert L.pa_reset_workspace(ws.data_ptr(), n, stream) == _lib.PA_OK
    torch.cuda.synchronize()
    head = (1 << 20) + 256
    assert int(ws[:head].sum()) == 0
    assert bool((ws[head:] == 7).all())
    st = ctypes.c_int(-1)
    assert L.pa_read_status(ws.data_ptr(), ctypes.byref(st), stream) == _lib.PA_OK
    assert st.value == 0
