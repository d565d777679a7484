"""GPU: decode with bf16 activations (q and out bf16; fp16 or per-token INT8 cache) against the
numpy oracle run on the same bf16 q values, the fp16-range check of q, and the failure path of
the bounded device waits (a wait that nothing completes must time out and report it)."""

import ctypes

import numpy as np
import pytest
import torch

import pa_oracle
from pa_testlib import (BLOCK_SIZE, assert_close, fp16_case, int8_case, oracle_out,
                        scale_for, to_cuda)

pytestmark = pytest.mark.gpu


def _ops():
    from pa_b200 import ops
    return ops


def _bf16_q(c):
    q = torch.from_numpy(np.ascontiguousarray(c["q"])).to(torch.bfloat16)
    return q, q.float().numpy()  # the values the kernel sees, for the oracle


@pytest.mark.parametrize("splitk", [False, True])
@pytest.mark.parametrize("kind", ["fp16", "int8"])
@pytest.mark.parametrize("lens,heads", [([1, 17, 500], (8, 2)), ([1500, 33], (32, 8)),
                                        ([700, 4096], (12, 2))])
def test_bf16_q_matches_oracle(kind, splitk, lens, heads):
    H, KVH = heads
    c = fp16_case(71, len(lens), H, KVH, lens)
    qb, qf = _bf16_q(c)
    q = qb.cuda()
    bt, cl = to_cuda(c["block_table"], c["context_lens"])
    out = torch.empty_like(q)
    if kind == "fp16":
        kc, vc = to_cuda(c["k_cache"], c["v_cache"])
        _ops().decode_bf16(out, q, kc, vc, bt, cl, scale_for(), BLOCK_SIZE, splitk=splitk)
        ref = oracle_out(qf, c["k_cache"], c["v_cache"], c["block_table"], c["context_lens"])
    else:
        qc = int8_case(c, "per_token")
        kc, vc, ks, vs = to_cuda(qc["k_cache"], qc["v_cache"], qc["k_scales"], qc["v_scales"])
        _ops().decode_bf16(out, q, kc, vc, bt, cl, scale_for(), BLOCK_SIZE, k_scales=ks,
                           v_scales=vs, splitk=splitk)
        kd, vd = pa_oracle.dequantize_kv(qc["k_cache"], qc["v_cache"], qc["k_scales"],
                                         qc["v_scales"])
        ref = oracle_out(qf, kd, vd, c["block_table"], c["context_lens"])
    assert out.dtype == torch.bfloat16
    assert_close(out, ref)
    _ops().check_status(q.device)


def test_bf16_q_rejects_fp16_arguments():
    c = fp16_case(3, 1, 8, 2, [40])
    q16, kc, vc, bt, cl = to_cuda(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                  c["context_lens"])
    with pytest.raises(RuntimeError, match="q must be bf16"):
        _ops().decode_bf16(torch.empty_like(q16), q16, kc, vc, bt, cl, scale_for(), BLOCK_SIZE)


def test_bf16_q_outside_fp16_range_is_flagged():
    c = fp16_case(5, 1, 8, 2, [64])
    qb, _ = _bf16_q(c)
    qb[0, 0, 0] = 1.0e5  # representable in bf16, not in fp16
    q = qb.cuda()
    kc, vc, bt, cl = to_cuda(c["k_cache"], c["v_cache"], c["block_table"], c["context_lens"])
    ops = _ops()
    ops.read_status(q.device)  # start from a clean status word
    ops.decode_bf16(torch.empty_like(q), q, kc, vc, bt, cl, scale_for(), BLOCK_SIZE)
    from pa_b200 import _lib
    assert ops.read_status(q.device) & _lib.PA_ERR_Q_RANGE


def test_bounded_wait_gives_up_and_reports_timeout():
    """A device wait on a barrier that nothing completes ends after about a second with
    PA_ERR_TIMEOUT in the status word, and the context stays usable afterwards."""
    from pa_b200 import _lib
    L = _lib.lib()
    ws = torch.zeros(256, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert L.pa_selftest_bounded_wait(ws.data_ptr(), stream) == _lib.PA_OK
    torch.cuda.synchronize()
    st = ctypes.c_int(0)
    assert L.pa_read_status(ws.data_ptr(), ctypes.byref(st), stream) == _lib.PA_OK
    assert st.value & _lib.PA_ERR_TIMEOUT
    # The context still runs kernels correctly.
    c = fp16_case(9, 2, 8, 2, [100, 37])
    q, kc, vc, bt, cl = to_cuda(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                c["context_lens"])
    out = torch.empty_like(q)
    _ops().decode(out, q, kc, vc, bt, cl, scale_for(), BLOCK_SIZE)
    assert_close(out, oracle_out(c["q"], c["k_cache"], c["v_cache"], c["block_table"],
                                 c["context_lens"]))
