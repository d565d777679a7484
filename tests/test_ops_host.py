"""CPU: the torch-facing ops reject cache tensors whose layout the write kernels would address
out of bounds (the kernels receive only num_blocks and block_size)."""

import pytest
import torch

from pa_b200 import ops


def _cache(nb=4, kvh=2, d=128, bs=16, dt=torch.int8):
    return (torch.zeros(nb, kvh, d // 8, bs, 8, dtype=dt), torch.zeros(nb, kvh, d, bs, dtype=dt),
            torch.zeros(nb, kvh, bs), torch.zeros(nb, kvh, bs))


def test_layout_accepts_the_paged_layout():
    kc, vc, ks, vs = _cache()
    assert ops._check_cache_layout(kc, vc, 2, 128, 16, ks, vs) == 4
    kc, vc, _, _ = _cache(nb=7, kvh=8, bs=32, dt=torch.float16)
    assert ops._check_cache_layout(kc, vc, 8, 128, 32) == 7


@pytest.mark.parametrize("case", ["kv_heads", "block_size", "head_dim", "v_blocks", "v_dims",
                                  "k_rank", "scales"])
def test_layout_rejects_mismatches(case):
    kc, vc, ks, vs = _cache()
    args = dict(num_kv_heads=2, head_dim=128, block_size=16)
    if case == "kv_heads":
        args["num_kv_heads"] = 4
    elif case == "block_size":
        args["block_size"] = 32
    elif case == "head_dim":
        args["head_dim"] = 64
    elif case == "v_blocks":
        vc = vc[:3]
    elif case == "v_dims":
        vc = torch.zeros(4, 2, 16, 128, dtype=torch.int8)  # [.., bs, D] instead of [.., D, bs]
    elif case == "k_rank":
        kc = kc.reshape(4, 2, 128, 16)
    elif case == "scales":
        ks = torch.zeros(4, 2, 8)
    with pytest.raises(RuntimeError):
        ops._check_cache_layout(kc, vc, args["num_kv_heads"], args["head_dim"],
                                args["block_size"], ks, vs)


def test_context_length_check():
    ops._check_lengths(torch.tensor([1, 5, 16], dtype=torch.int32), 16)
    ops._check_lengths(torch.tensor([], dtype=torch.int32), 16)
    with pytest.raises(RuntimeError, match=">= 1"):
        ops._check_lengths(torch.tensor([3, 0], dtype=torch.int32), 16)
    with pytest.raises(RuntimeError, match="exceeds"):
        ops._check_lengths(torch.tensor([17, 2], dtype=torch.int32), 16)
