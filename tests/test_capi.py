"""CPU: the C-ABI library builds, loads, exports every function include/pa_b200.h declares,
and rejects bad arguments on the host (no GPU work is launched here)."""

import os
import re
import shutil
import subprocess

import pytest

from pa_b200 import _lib, build

HEADER = os.path.join(build.INCLUDE_DIR, "pa_b200.h")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    protos = {}
    for m in re.finditer(r"\b(pa_\w+)\s*\(([^;{]*?)\)\s*;", src):
        name, args = m.group(1), m.group(2).strip()
        n = 0 if args in ("", "void") else args.count(",") + 1
        protos[name] = n
    return protos


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.lib()


def test_header_declares_entry_points():
    names = set(_declared())
    for must in ("pa_decode_f16", "pa_decode_i8", "pa_splitk_f16", "pa_splitk_i8",
                 "pa_quantize_into_cache", "pa_decode_workspace_bytes"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    for name, nargs in _declared().items():
        assert hasattr(lib, name), f"{name} not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
        assert len(_lib.SIGNATURES[name][1]) == nargs, f"{name}: arity mismatch"


def test_version_and_status_strings(lib):
    assert lib.pa_version() >= 100
    assert lib.pa_status_string(0) == b"ok"
    assert b"context_lens" in lib.pa_status_string(_lib.PA_ERR_EMPTY_CONTEXT)
    assert lib.pa_partial_floats(12, 2, 128) == 130 * 8
    assert lib.pa_partial_floats(32, 1, 128) == 130 * 16 * 2
    assert lib.pa_partial_floats(12, 5, 128) == 0


def _decode_f16(lib, **kw):
    a = dict(out=1 << 20, q=1 << 20, k=1 << 20, v=1 << 20, bt=1 << 20, cl=1 << 20, B=1, H=8,
             KVH=2, D=128, NB=4, bs=16, mb=2, scale=0.1, ws=1 << 20, wsb=1 << 30)
    a.update(kw)
    return lib.pa_decode_f16(a["out"], a["q"], a["k"], a["v"], a["bt"], a["cl"], a["B"], a["H"],
                             a["KVH"], a["D"], a["NB"], a["bs"], a["mb"], a["scale"], a["ws"],
                             a["wsb"], None)


def test_host_argument_checks(lib):
    assert _decode_f16(lib, D=64) == _lib.PA_ERR_UNSUPPORTED
    assert b"head_dim" in lib.pa_last_error()
    assert _decode_f16(lib, H=7, KVH=2) == _lib.PA_ERR_INVALID_ARG
    assert _decode_f16(lib, bs=8) == _lib.PA_ERR_INVALID_ARG
    assert b"block_size" in lib.pa_last_error()
    assert _decode_f16(lib, bs=48) == _lib.PA_ERR_INVALID_ARG
    assert _decode_f16(lib, KVH=0) == _lib.PA_ERR_INVALID_ARG
    assert _decode_f16(lib, NB=1 << 26, KVH=4) == _lib.PA_ERR_UNSUPPORTED  # 2^28 page rows
    assert b"page rows" in lib.pa_last_error()
    assert _decode_f16(lib, B=0) == _lib.PA_OK  # empty batch: nothing to do
    rc = lib.pa_quantize_into_cache(1 << 20, 1 << 20, 9, 256, 1 << 20, 4, 2, 128, 1 << 20,
                                    1 << 20, 1 << 20, 1 << 20, 4, 16, None, None, None, None)
    assert rc == _lib.PA_ERR_UNSUPPORTED
    rc = lib.pa_absmax_scale(1 << 20, 0, 10, 1 << 20, 7, 1 << 20, None)
    assert rc == _lib.PA_ERR_INVALID_ARG


def test_extension_entry_points_check_arguments_on_the_host(lib):
    names = set(_declared())
    for must in ("pa_decode_fp8", "pa_splitk_fp8", "pa_quantize_into_cache_fp8",
                 "pa_decode_bf16q", "pa_decode_bf16q_workspace_bytes",
                 "pa_selftest_bounded_wait", "pa_decode_f16_noalloc",
                 "pa_decode_f16_noalloc_read_status", "pa_reset_workspace",
                 "pa_decode_step"):
        assert must in names
    assert b"fp16 range" in lib.pa_status_string(_lib.PA_ERR_Q_RANGE)
    p = 1 << 20
    # bf16 activations: only fp16 / int8 / fp8 caches
    rc = lib.pa_decode_bf16q(p, p, p, p, p, p, p, p, 1, 8, 2, 128, 4, 16, 2, _lib.PA_DTYPE_F32, 0,
                             0.1, p, 1 << 30, None)
    assert rc == _lib.PA_ERR_UNSUPPORTED and b"kv_dtype" in lib.pa_last_error()
    rc = lib.pa_decode_bf16q(p, p, p, p, p, p, p, p, 1, 7, 2, 128, 4, 16, 2, _lib.PA_DTYPE_F16, 0,
                             0.1, p, 1 << 30, None)
    assert rc == _lib.PA_ERR_INVALID_ARG
    # fp8 decode: the same shape rules as the other decode ops
    rc = lib.pa_decode_fp8(p, p, p, p, p, p, p, p, 1, 8, 2, 64, 4, 16, 2, 0.1, p, 1 << 30, None)
    assert rc == _lib.PA_ERR_UNSUPPORTED
    rc = lib.pa_splitk_fp8(p, p, p, p, p, p, p, p, 1, 8, 2, 128, 4, 24, 2, 0.1, p, 1 << 30, None)
    assert rc == _lib.PA_ERR_INVALID_ARG
    # fp8 write: input dtype and null pointers
    rc = lib.pa_quantize_into_cache_fp8(p, p, 9, 256, p, 4, 2, 128, p, p, p, p, 4, 16, None, None)
    assert rc == _lib.PA_ERR_UNSUPPORTED
    rc = lib.pa_quantize_into_cache_fp8(p, p, _lib.PA_DTYPE_F16, 256, p, 4, 2, 128, p, p, None, p,
                                        4, 16, None, None)
    assert rc == _lib.PA_ERR_INVALID_ARG
    # decode step: cache dtype, new-token rows, per-tensor scales only with int8
    rc = lib.pa_decode_step(_lib.PA_DTYPE_F32, p, p, p, p, _lib.PA_DTYPE_F16, 256, p, p, p, p,
                            None, None, p, p, 1, 8, 2, 128, 4, 16, 2, 0.1, 0, 1, p, 1 << 30, None)
    assert rc == _lib.PA_ERR_UNSUPPORTED
    rc = lib.pa_decode_step(_lib.PA_DTYPE_I8, p, p, None, p, _lib.PA_DTYPE_F16, 256, p, p, p, p,
                            None, None, p, p, 1, 8, 2, 128, 4, 16, 2, 0.1, 0, 1, p, 1 << 30, None)
    assert rc == _lib.PA_ERR_INVALID_ARG
    rc = lib.pa_decode_step(_lib.PA_DTYPE_F16, p, p, p, p, _lib.PA_DTYPE_F16, 256, p, p, None,
                            None, p, p, p, p, 1, 8, 2, 128, 4, 16, 2, 0.1, 0, 1, p, 1 << 30, None)
    assert rc == _lib.PA_ERR_INVALID_ARG and b"fixed scales" in lib.pa_last_error()
    rc = lib.pa_decode_step(_lib.PA_DTYPE_I8, p, p, p, p, _lib.PA_DTYPE_F16, 100, p, p, p, p,
                            None, None, p, p, 1, 8, 2, 128, 4, 16, 2, 0.1, 0, 1, p, 1 << 30, None)
    assert rc == _lib.PA_ERR_INVALID_ARG and b"new_token_stride" in lib.pa_last_error()
    # the wait self-test needs a status word; reset and status reads need their buffers
    assert lib.pa_selftest_bounded_wait(None, None) == _lib.PA_ERR_INVALID_ARG
    assert lib.pa_reset_workspace(None, 1024, None) == _lib.PA_ERR_INVALID_ARG
    assert lib.pa_decode_f16_noalloc_read_status(None, None) == _lib.PA_ERR_INVALID_ARG


def test_plain_c_caller(lib, tmp_path):
    """tests/c_abi_check.c, a C99 program that includes only include/pa_b200.h and links the
    library, compiles with -Wall -Wextra -pedantic -Werror and passes its host-side checks."""
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    src = os.path.join(os.path.dirname(os.path.abspath(__file__)), "c_abi_check.c")
    libdir = os.path.dirname(build.LIB_PATH)
    exe = str(tmp_path / "c_abi_check")
    subprocess.run([gcc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I",
                    build.INCLUDE_DIR, src, "-L", libdir, "-lpa_b200", "-Wl,-rpath," + libdir,
                    "-o", exe], check=True, capture_output=True, text=True)
    res = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stderr
    assert "c abi ok" in res.stdout
