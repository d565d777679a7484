"""ctypes binding of libpa_b200.so (the C ABI declared in include/pa_b200.h).

This is the only module that touches the shared library. There is no fallback: if the
library cannot be built or loaded, importing the ops raises.
"""

import ctypes
import fcntl
import os
import threading

from . import build as _build

# Status codes (include/pa_b200.h).
PA_OK = 0
PA_ERR_INVALID_ARG = 1
PA_ERR_UNSUPPORTED = 2
PA_ERR_CUDA = 4
PA_ERR_WORKSPACE = 8
PA_ERR_EMPTY_CONTEXT = 16
PA_ERR_CONTEXT_RANGE = 32
PA_ERR_BLOCK_ID = 64
PA_ERR_TIMEOUT = 128
PA_ERR_SLOT = 256
PA_ERR_Q_RANGE = 512

PA_DTYPE_F16 = 0
PA_DTYPE_BF16 = 1
PA_DTYPE_F32 = 2
PA_DTYPE_I8 = 3
PA_DTYPE_FP8E4M3 = 4

PA_SCALE_CLAMP_THEN_DIVIDE = 0
PA_SCALE_DIVIDE_THEN_CLAMP = 1

_vp = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); must match include/pa_b200.h
SIGNATURES = {
    "pa_version": (_i, []),
    "pa_last_error": (ctypes.c_char_p, []),
    "pa_status_string": (ctypes.c_char_p, [_i]),
    "pa_decode_workspace_bytes": (_sz, [_i, _i, _i, _i, _i, _i, _i, _i]),
    "pa_read_status": (_i, [_vp, ctypes.POINTER(ctypes.c_int), _vp]),
    "pa_reset_workspace": (_i, [_vp, _sz, _vp]),
    "pa_decode_f16": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f, _vp,
                           _sz, _vp]),
    "pa_decode_i8": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f,
                          _vp, _sz, _vp]),
    "pa_splitk_f16": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f, _vp,
                           _sz, _vp]),
    "pa_decode_f16_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f,
                                   _vp]),
    "pa_decode_f16_noalloc_read_status": (_i, [ctypes.POINTER(ctypes.c_int), _vp]),
    "pa_splitk_i8": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f,
                          _vp, _sz, _vp]),
    "pa_decode_bf16q_workspace_bytes": (_sz, [_i, _i, _i, _i, _i, _i, _i, _i]),
    "pa_decode_bf16q": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i,
                             _i, _i, _f, _vp, _sz, _vp]),
    "pa_selftest_bounded_wait": (_i, [_vp, _vp]),
    "pa_decode_fp8": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f,
                           _vp, _sz, _vp]),
    "pa_splitk_fp8": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f,
                           _vp, _sz, _vp]),
    "pa_quantize_into_cache_fp8": (_i, [_vp, _vp, _i, _i64, _vp, _i, _i, _i, _vp, _vp, _vp, _vp,
                                        _i, _i, _vp, _vp]),
    "pa_decode_step": (_i, [_i, _vp, _vp, _vp, _vp, _i, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                            _vp, _i, _i, _i, _i, _i, _i, _i, _f, _i, _i, _vp, _sz, _vp]),
    "pa_partial_floats": (_i, [_i, _i, _i]),
    "pa_decode_partial": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i,
                               _i, _i, _f, _vp, _sz, _vp]),
    "pa_merge_partials": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _vp, _vp]),
    "pa_quantize_into_cache": (_i, [_vp, _vp, _i, _i64, _vp, _i, _i, _i, _vp, _vp, _vp, _vp, _i,
                                    _i, _vp, _vp, _vp, _vp]),
    "pa_write_into_cache_f16": (_i, [_vp, _vp, _i, _i64, _vp, _i, _i, _i, _vp, _vp, _i, _i, _vp,
                                     _vp]),
    "pa_prefill_into_cache": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _i, _i, _vp, _vp, _vp,
                                   _vp, _i, _i, _vp, _vp, _vp, _vp]),
    "pa_absmax_scale": (_i, [_vp, _i, _i64, _vp, _i, _vp, _vp]),
}

_lock = threading.Lock()
_lib = None


def _load():
    path = _build.LIB_PATH
    if not os.path.exists(path):
        # Build once, serialised across processes (torchrun ranks) with a file lock.
        lock_path = path + ".lock"
        with open(lock_path, "w") as lf:
            fcntl.flock(lf, fcntl.LOCK_EX)
            try:
                if not os.path.exists(path):
                    _build.build()
            finally:
                fcntl.flock(lf, fcntl.LOCK_UN)
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def lib():
    """The loaded library (built on first use if absent)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                _lib = _load()
    return _lib


def last_error():
    msg = lib().pa_last_error()
    return msg.decode() if msg else ""


def check(rc, what):
    """Raise RuntimeError for a non-zero C-ABI return code."""
    if rc != PA_OK:
        raise RuntimeError(f"{what}: {last_error() or lib().pa_status_string(rc).decode()}")
