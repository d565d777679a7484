"""CPU: multi-GPU sharding logic (pa_b200.shard) and the cross-rank split-context exchange
(shard.SplitContextDecode.step itself), run as world-size-2 gloo process groups with the
oracle standing in for the two GPU kernels of the step."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import gen
import pa_oracle
from pa_b200 import shard


def test_lpt_partition_covers_and_balances():
    rng = np.random.default_rng(0)
    for world in (1, 2, 3, 4, 8):
        lens = rng.integers(1, 5000, size=97).tolist()
        parts = shard.lpt_partition(lens, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(len(lens)))
        loads = [sum(lens[i] for i in p) for p in parts]
        # LPT bound: max load <= 4/3 * optimum <= 4/3 * max(mean, largest item)
        lower = max(sum(lens) / world, max(lens))
        assert max(loads) <= 4 / 3 * lower + 1e-9


def test_lpt_partition_deterministic():
    lens = [5, 5, 5, 5, 3, 3]
    assert shard.lpt_partition(lens, 2) == shard.lpt_partition(lens, 2)


def test_kv_head_slice():
    q_heads, kv_heads = set(), set()
    for r in range(4):
        qs, ks = shard.kv_head_slice(64, 8, 4, r)
        q_heads |= set(qs)
        kv_heads |= set(ks)
        assert len(qs) == 16 and len(ks) == 2
        assert all(h // 8 in ks for h in qs)  # q head h belongs to kv head h // 8
    assert q_heads == set(range(64)) and kv_heads == set(range(8))
    with pytest.raises(ValueError):
        shard.kv_head_slice(12, 2, 4, 0)


@pytest.mark.parametrize("ctx", [1, 15, 16, 17, 100, 4096])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_token_ranges_are_block_aligned_and_cover(ctx, world):
    rs = shard.token_ranges(ctx, world)
    assert rs[0][0] == 0 and rs[-1][1] == ctx
    for (a, b), (c, d) in zip(rs, rs[1:]):
        assert b == c
    for a, b in rs:
        assert a % 16 == 0 and a <= b


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_partial(q, k_cache, v_cache, block_table, context_lens, scale, block_size=16,
                    k_scales=None, v_scales=None):
    """The partial decode step of SplitContextDecode, computed by the oracle on CPU tensors
    and returned in the CUDA kernel's slot layout."""
    kc, vc = k_cache.numpy(), v_cache.numpy()
    if k_scales is not None:
        kc, vc = pa_oracle.dequantize_kv(kc, vc, k_scales.numpy(), v_scales.numpy())
    cl = context_lens.numpy()
    m, l, acc = pa_oracle.range_partials(q.numpy(), kc, vc, block_table.numpy(), cl,
                                         np.zeros_like(cl), cl, scale)
    return torch.from_numpy(pa_oracle.pack_slots(m, l, acc, k_cache.shape[1]))


def _oracle_merge(out, gathered, num_heads, num_kv_heads):
    """The merge step: [world, num_seqs, per_seq] partials -> fp16 out, by the oracle."""
    assert gathered.dim() == 3
    m, l, acc = pa_oracle.unpack_slots(gathered.numpy(), num_heads, num_kv_heads)
    out.copy_(torch.from_numpy(pa_oracle.lse_merge(m, l, acc)).to(out.dtype))
    return out


def _split_context_worker(rank, world, port, int8, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lens = [700, 33, 1, 1500]
        H, KVH = 12, 2
        c = gen.decode_case(seed=41, num_seqs=4, num_heads=H, num_kv_heads=KVH,
                            context_lens=lens)
        kc, vc = pa_oracle.scatter_paged_cache(c["k"], c["v"], c["context_lens"],
                                               c["block_table"], c["num_blocks"])
        ks = vs = None
        if int8:
            kq, ksc = pa_oracle.quantize_per_token(c["k"], "f16")
            vq, vsc = pa_oracle.quantize_per_token(c["v"], "f16")
            nb = c["num_blocks"]
            kc, vc = pa_oracle.scatter_paged_cache(kq, vq, c["context_lens"], c["block_table"],
                                                   nb)
            ks = pa_oracle.scatter_scales(ksc, c["context_lens"], c["block_table"], nb, KVH)
            vs = pa_oracle.scatter_scales(vsc, c["context_lens"], c["block_table"], nb, KVH)
        scale = 1 / np.sqrt(128)
        # This rank's share: block ids and context length of its token range per sequence.
        S = len(lens)
        bt_local = np.zeros_like(c["block_table"])
        cl_local = np.zeros(S, np.int32)
        for b in range(S):
            blocks, n = shard.local_view(c["block_table"][b], lens[b], world, rank)
            bt_local[b, :len(blocks)] = blocks
            cl_local[b] = n
        dec = shard.SplitContextDecode(partial_fn=_oracle_partial, merge_fn=_oracle_merge)
        out = torch.empty(S, H, 128, dtype=torch.float16)
        t = torch.from_numpy
        dec.step(out, t(c["q"]), t(kc), t(vc), t(bt_local), t(cl_local), scale, 16,
                 k_scales=None if ks is None else t(ks), v_scales=None if vs is None else t(vs))
        if int8:
            kc, vc = pa_oracle.dequantize_kv(kc, vc, ks, vs)
        full = pa_oracle.paged_decode_attention(c["q"], kc, vc, c["block_table"],
                                                c["context_lens"], scale=scale)
        result_q.put((rank, float(np.abs(out.float().numpy() - full).max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("int8", [False, True])
def test_split_context_exchange_gloo_world2(int8):
    """Two ranks each own a block-aligned half of every sequence and run
    SplitContextDecode.step: local partials, all_gather over the process group, LSE merge. The
    result on every rank equals the one-pass decode (fp16 output rounding)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_split_context_worker, args=(r, 2, port, int8, q))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=5) for _ in range(2))
    assert all(err < 1e-3 for _, err in res), res


def test_slot_packing_round_trips():
    rng = np.random.default_rng(3)
    for H, KVH in ((12, 2), (8, 8), (40, 2), (7, 1)):
        S = 3
        m = rng.standard_normal((S, H))
        l = rng.random((S, H)) + 0.5
        acc = rng.standard_normal((S, H, 128))
        slots = pa_oracle.pack_slots(m, l, acc, KVH)
        G = H // KVH
        GT = 8 if G <= 8 else 16
        assert slots.shape == (S, KVH * -(-G // GT) * 130 * GT)
        m2, l2, a2 = pa_oracle.unpack_slots(slots, H, KVH)
        np.testing.assert_allclose(m2, m, rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(l2, l, rtol=1e-6)
        np.testing.assert_allclose(a2, acc, rtol=1e-6, atol=1e-6)


def _dead_peer_worker(rank, world, port, result_q):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        # This rank fails between steps, before the exchange, without joining it.
        os._exit(3)
    local = torch.zeros(8)
    gathered = [torch.empty_like(local) for _ in range(world)]
    try:
        dist.all_gather(gathered, local)
        result_q.put((rank, "completed"))
    except Exception as e:  # noqa: BLE001 - any backend error is the expected outcome
        result_q.put((rank, "error: " + type(e).__name__))
    # Flush the queue's feeder thread before leaving without the process group's teardown.
    result_q.close()
    result_q.join_thread()
    os._exit(0)


def test_split_context_exchange_reports_a_dead_peer():
    """A rank that dies before the all-gather of partials makes the surviving rank's exchange
    fail with an error (within the process group's short timeout) instead of hanging."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dead_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert procs[1].exitcode == 3
    assert procs[0].exitcode == 0, procs[0].exitcode
    rank, outcome = q.get(timeout=5)
    assert rank == 0 and outcome.startswith("error"), outcome


def test_split_context_single_rank_without_process_group():
    """With no process group the step runs on one rank (the gather is a copy)."""
    assert not dist.is_initialized()
    lens = [300, 17]
    c = gen.decode_case(seed=8, num_seqs=2, num_heads=8, num_kv_heads=2, context_lens=lens)
    kc, vc = pa_oracle.scatter_paged_cache(c["k"], c["v"], c["context_lens"], c["block_table"],
                                           c["num_blocks"])
    dec = shard.SplitContextDecode(partial_fn=_oracle_partial, merge_fn=_oracle_merge)
    assert dec.world == 1
    out = torch.empty(2, 8, 128, dtype=torch.float16)
    t = torch.from_numpy
    dec.step(out, t(c["q"]), t(kc), t(vc), t(c["block_table"]), t(c["context_lens"]),
             1 / np.sqrt(128))
    full = pa_oracle.paged_decode_attention(c["q"], kc, vc, c["block_table"], c["context_lens"])
    assert float(np.abs(out.float().numpy() - full).max()) < 1e-3
