"""CPU: the FP8 (e4m3) cache format of the oracle. Its e4m3 rounding (torch's float8_e4m3fn
conversion of values clamped to +-448) is pinned against CUDA's own conversion
(__nv_cvt_float_to_fp8, saturating, round-to-nearest-even) run on the host, and the
per-token quantiser is checked for its scale, saturation and zero-row rules."""

import os
import shutil
import subprocess
import tempfile

import numpy as np
import pytest

import pa_oracle

HERE = os.path.dirname(os.path.abspath(__file__))


def _nvcc():
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    return None


@pytest.mark.skipif(_nvcc() is None, reason="nvcc not available")
def test_oracle_e4m3_rounding_matches_cuda_conversion():
    import torch
    rng = np.random.default_rng(11)
    x = np.concatenate([
        (rng.standard_normal(40000) * 100).astype(np.float32),
        rng.uniform(-460, 460, 40000).astype(np.float32),
        (rng.standard_normal(40000) * 1e-3).astype(np.float32),
        # ties, the saturation edge, subnormals and signed zero
        np.array([0.0, -0.0, 448.0, -448.0, 449.0, 464.0, 465.0, 1e-9, 2.0 ** -9,
                  2.0 ** -10, 1.0625, 1.1875, -1.0625, 0.013671875], dtype=np.float32),
    ])
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "cvt")
        subprocess.run([_nvcc(), "-o", exe, os.path.join(HERE, "fp8_pin", "cvt_e4m3.cu"),
                        "-Wno-deprecated-gpu-targets"], check=True, capture_output=True)
        x.tofile(os.path.join(d, "in.bin"))
        subprocess.run([exe, os.path.join(d, "in.bin"), os.path.join(d, "out.bin")], check=True)
        cuda = np.fromfile(os.path.join(d, "out.bin"), dtype=np.uint8)
    ours = torch.from_numpy(np.clip(x, -448, 448)).to(torch.float8_e4m3fn).view(torch.uint8)
    assert np.array_equal(cuda, ours.numpy())


def test_quantize_per_token_fp8_rules():
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((5, 3, 128)) * 7).astype(np.float16)
    x[1, 2] = 0  # a zero row
    q, s = pa_oracle.quantize_per_token_fp8(x)
    assert q.dtype == np.uint8 and s.dtype == np.float32 and q.shape == x.shape
    amax = np.abs(x.astype(np.float32)).max(-1)
    assert np.array_equal(s, (amax / np.float32(448)).astype(np.float32))
    assert s[1, 2] == 0 and not q[1, 2].any()
    deq = pa_oracle.fp8_to_float(q) * s[..., None]
    # e4m3 keeps 3 mantissa bits: relative error at most 2^-4 per element (normal range)
    xf = x.astype(np.float32)
    big = np.abs(xf) > s[..., None] * 2.0 ** -6
    assert np.all(np.abs(deq - xf)[big] <= np.abs(xf)[big] * 2.0 ** -4 + 1e-12)
    # the row maximum maps to +-448 exactly
    i = np.abs(xf).argmax(-1)
    top = np.take_along_axis(pa_oracle.fp8_to_float(q), i[..., None], -1)[..., 0]
    nz = s > 0
    assert np.all(np.abs(top[nz]) == 448.0)
