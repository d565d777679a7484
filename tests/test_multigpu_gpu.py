"""GPU, two ranks over NCCL (skipped with fewer than two GPUs): the multi-GPU decode paths.

* Context split (shard.SplitContextDecode): each rank holds a block-aligned token range of every
  sequence, computes partials with the CUDA partial decode, all-gathers them over NCCL and
  merges them with the CUDA merge kernel; every rank's output must equal the oracle's one-pass
  decode of the whole context.
* kv-head sharding (shard.kv_head_slice): each rank decodes its kv heads' q heads; the
  all-gathered outputs must equal the oracle's.
One process per GPU (spawned), process group timeout 60 s, NVLS off.
"""

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

needs_two = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                               reason="needs two GPUs")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _excess(out, ref):
    """Largest amount by which |out - ref| exceeds the tolerance 2e-3 + 1e-2 |ref| (<= 0: ok)."""
    r = torch.from_numpy(ref)
    return float(((out.float().cpu() - r).abs() - (2e-3 + 1e-2 * r.abs())).max())


def _worker(rank, world, port, kind, result_q):
    import datetime

    import torch.distributed as dist

    import pa_oracle
    from pa_b200 import ops, shard
    from pa_testlib import fp16_case, int8_case, scale_for
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        H, KVH = 64, 8
        lens = [3000, 700, 1, 1500, 33]
        c = fp16_case(17, len(lens), H, KVH, lens, dist="lognormal_outlier")
        if kind == "int8":
            qc = int8_case(c, "per_token")
            kc, vc, ks, vs = qc["k_cache"], qc["v_cache"], qc["k_scales"], qc["v_scales"]
            kd, vd = pa_oracle.dequantize_kv(kc, vc, ks, vs)
        else:
            kc, vc, ks, vs = c["k_cache"], c["v_cache"], None, None
            kd, vd = kc, vc
        ref = pa_oracle.paged_decode_attention(c["q"], kd, vd, c["block_table"],
                                               c["context_lens"])
        t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
        q, kct, vct, kst, vst = t(c["q"]), t(kc), t(vc), t(ks), t(vs)
        errs = {}

        # Context split: this rank's token range of every sequence.
        S = len(lens)
        bt_local = np.zeros_like(c["block_table"])
        cl_local = np.zeros(S, np.int32)
        for b in range(S):
            blocks, n = shard.local_view(c["block_table"][b], lens[b], world, rank)
            bt_local[b, :len(blocks)] = blocks
            cl_local[b] = n
        dec = shard.SplitContextDecode()
        out = torch.empty_like(q)
        for _ in range(2):  # the second step reuses the gather buffer
            dec.step(out, q, kct, vct, t(bt_local), t(cl_local), scale_for(), 16, k_scales=kst,
                     v_scales=vst)
        torch.cuda.synchronize()
        errs["context_split"] = _excess(out, ref)

        # kv-head sharding: this rank's kv heads (cache slice) and their q heads.
        qh, kh = shard.kv_head_slice(H, KVH, world, rank)
        sl = slice(kh.start, kh.stop)
        kc_r, vc_r = kct[:, sl].contiguous(), vct[:, sl].contiguous()
        ks_r = None if kst is None else kst[:, sl].contiguous()
        vs_r = None if vst is None else vst[:, sl].contiguous()
        q_r = q[:, qh.start:qh.stop].contiguous()
        out_r = torch.empty_like(q_r)
        ops.decode(out_r, q_r, kc_r, vc_r, t(c["block_table"]), t(c["context_lens"]),
                   scale_for(), 16, k_scales=ks_r, v_scales=vs_r, splitk=True)
        gathered = [torch.empty_like(out_r) for _ in range(world)]
        dist.all_gather(gathered, out_r)
        full = torch.cat(gathered, dim=1)
        errs["kv_head_shard"] = _excess(full, ref)
        ops.check_status(dev)
        result_q.put((rank, errs))
    finally:
        dist.destroy_process_group()


@needs_two
@pytest.mark.parametrize("kind", ["fp16", "int8"])
def test_two_rank_context_split_and_kv_head_shard(kind):
    import torch.multiprocessing as mp
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, kind, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=10) for _ in range(2))
    for rank, errs in res:
        for name, err in errs.items():
            assert err <= 0.0, (rank, name, err)
