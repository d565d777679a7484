"""CPU: the pieces of bench.py that do not need a GPU.

bench.py checks every timed output against an fp32 restatement of the reference decode in
torch (_dense_seq + _ref_decode). That restatement is pinned here to the oracle on seeded
paged caches (FP16, per-token INT8, FP8), so the parity figure in the bench line means what it
says. The workload specs and the reference arm's line are checked too.
"""

import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import gen
import pa_oracle
from pa_testlib import int8_case

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)
import bench  # noqa: E402


def _case(kind):
    lens = [300, 17, 1, 77]
    c = gen.decode_case(seed=12, num_seqs=4, num_heads=12, num_kv_heads=2, context_lens=lens,
                        dist="lognormal_outlier")
    kc, vc = pa_oracle.scatter_paged_cache(c["k"], c["v"], c["context_lens"], c["block_table"],
                                           c["num_blocks"])
    ks = vs = None
    if kind == "i8":
        q8 = int8_case(c, "per_token")
        kc, vc, ks, vs = q8["k_cache"], q8["v_cache"], q8["k_scales"], q8["v_scales"]
    elif kind == "f8":
        kq, ksc = pa_oracle.quantize_per_token_fp8(c["k"])
        vq, vsc = pa_oracle.quantize_per_token_fp8(c["v"])
        nb = c["num_blocks"]
        kc, vc = pa_oracle.scatter_paged_cache(kq, vq, c["context_lens"], c["block_table"], nb)
        ks = pa_oracle.scatter_scales(ksc, c["context_lens"], c["block_table"], nb, 2)
        vs = pa_oracle.scatter_scales(vsc, c["context_lens"], c["block_table"], nb, 2)
    return c, kc, vc, ks, vs


@pytest.mark.parametrize("kind", ["f16", "i8", "f8"])
def test_bench_reference_decode_matches_the_oracle(kind):
    c, kc, vc, ks, vs = _case(kind)
    if kind == "f8":
        kd, vd = pa_oracle.dequantize_fp8(kc, vc, ks, vs)
        tk = torch.from_numpy(kc.view(np.uint8)).view(torch.float8_e4m3fn)
        tv = torch.from_numpy(vc.view(np.uint8)).view(torch.float8_e4m3fn)
    elif kind == "i8":
        kd, vd = pa_oracle.dequantize_kv(kc, vc, ks, vs)
        tk, tv = torch.from_numpy(kc), torch.from_numpy(vc)
    else:
        kd, vd = kc, vc
        tk, tv = torch.from_numpy(kc), torch.from_numpy(vc)
    ref = pa_oracle.paged_decode_attention(c["q"], kd, vd, c["block_table"], c["context_lens"])
    tks = None if ks is None else torch.from_numpy(ks)
    tvs = None if vs is None else torch.from_numpy(vs)
    bt = torch.from_numpy(c["block_table"])
    for b, n in enumerate(c["context_lens"]):
        k, v = bench._dense_seq(torch, tk, tv, tks, tvs, bt[b], int(n))
        out = bench._ref_decode(torch, torch.from_numpy(c["q"][b]), k, v)
        np.testing.assert_allclose(out.numpy(), ref[b], atol=1e-4, rtol=1e-4)  # fp32 vs fp64


def test_bench_compare_flags_a_planted_error():
    ref = torch.linspace(-1, 1, 128).view(1, 128)
    out = ref.clone().half()
    assert bench._compare(torch, out, ref)[1] <= 0
    out[0, 5] += 0.05
    m, excess = bench._compare(torch, out, ref)
    assert m > 0.04 and excess > 0


def test_bench_specs_and_lengths():
    assert set(bench.SECONDARY_1GPU) <= set(bench.SPECS)
    assert set(bench.SECONDARY_MULTI) <= set(bench.SPECS)
    for name, spec in bench.SPECS.items():
        lens = bench._global_lens(spec)
        assert len(lens) == spec["B"] and lens.min() >= 1, name
    l5 = bench._global_lens(bench.SPECS["cfg5"]) + 1
    assert l5.min() >= 16 and l5.max() <= 32768
    l4 = bench._global_lens(bench.SPECS["cfg4"])
    assert l4.min() >= 65536 and l4.max() <= 131072
    assert bench.scaling_of("cfg2") == "weak" and bench.scaling_of("cfg5") == "strong"
    assert bench.config_name(3) == "cfg3" and bench.config_name("cfg4") == "cfg4"


def test_reference_arm_prints_one_line():
    res = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "1"], capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0, res.stderr
    lines = [x for x in res.stdout.splitlines() if x.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["value"] > 0
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and "cpu_model" in cb
    assert d["e2e"]["h2d_bytes_per_step"] == 0
