"""Torch-facing wrappers of the C ABI.

Each op checks its arguments with the error conditions of the reference launchers
(kernels/paged_attention_v4_splitk.cu:197-205, kernels/paged_attention_v6_splitk_int8.cu:
201-221 and siblings) and raises RuntimeError like their TORCH_CHECKs, then calls the
library on the current CUDA stream of the tensors' device. Temporaries (split partials,
arrival counters, the device status word) live in a per-(device, stream) workspace that is
zero-filled once when allocated and kept for later calls.
"""

import ctypes

import torch

from . import _lib

HEAD_DIM = 128
X = 8

_DTYPE_CODE = {
    torch.float16: _lib.PA_DTYPE_F16,
    torch.bfloat16: _lib.PA_DTYPE_BF16,
    torch.float32: _lib.PA_DTYPE_F32,
}

_workspaces = {}


def _ptr(t):
    return t.data_ptr() if t is not None else None


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


def workspace(device, nbytes):
    """The zero-initialised workspace of (device, current stream), grown to nbytes.

    Growing replaces the buffer, and a CUDA graph keeps the address it captured: run the
    largest shape once on a stream before capturing graphs on it, so no later call on that
    stream replaces the buffer a graph uses."""
    stream = _stream(device)
    key = (device.index, stream)
    ws = _workspaces.get(key)
    nbytes = max(int(nbytes), 256)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def read_status(device=None):
    """OR of the device status words of this device's workspaces, which are then cleared
    (synchronises). Bits are the PA_ERR_* codes of include/pa_b200.h. A workspace that
    reports an error also gets its arrival counters zeroed, since a kernel that stopped
    part-way can leave some of them set."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    status = 0
    L = _lib.lib()
    for (idx, stream), ws in list(_workspaces.items()):
        if idx != device.index:
            continue
        out = ctypes.c_int(0)
        _lib.check(L.pa_read_status(ws.data_ptr(), ctypes.byref(out), stream), "pa_read_status")
        if out.value:
            _lib.check(L.pa_reset_workspace(ws.data_ptr(), ws.numel(), stream),
                       "pa_reset_workspace")
            torch.cuda.synchronize(device)
        status |= out.value
    return status


def check_status(device=None):
    """Raise RuntimeError if a kernel on `device` recorded an error since the last check."""
    status = read_status(device)
    if status:
        raise RuntimeError("paged-attention kernel reported: " +
                           _lib.lib().pa_status_string(status).decode() + f" (status {status})")


class _Guard:
    """Make `device` current for the duration of a call (no-op when it already is)."""

    def __init__(self, device):
        self.device = device
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.device.index:
            self.prev = cur
            torch.cuda.set_device(self.device)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False


def _require(cond, msg):
    if not cond:
        raise RuntimeError(msg)


_FP8 = getattr(torch, "float8_e4m3fn", None)


def _kv_kind(k_cache, k_scales):
    """'f8' for an fp8 e4m3 cache, 'i8' for int8 (or whenever scales are given), else 'f16'."""
    if _FP8 is not None and k_cache.dtype == _FP8:
        return "f8"
    return "i8" if (k_scales is not None or k_cache.dtype == torch.int8) else "f16"


_KV_CODE = {"f16": _lib.PA_DTYPE_F16, "i8": _lib.PA_DTYPE_I8, "f8": _lib.PA_DTYPE_FP8E4M3}


def _check_lengths(context_lens, capacity, host_context_lens=None):
    """The reference's context_lens >= 1 check (and this library's upper bound). It reads
    host_context_lens, a CPU copy of the lengths, when the caller has one (no
    synchronisation); otherwise one device-to-host copy of context_lens, which synchronises
    the current stream."""
    if host_context_lens is not None:
        _require(host_context_lens.device.type == "cpu" and
                 host_context_lens.numel() == context_lens.numel(),
                 "host_context_lens must be a CPU tensor with one length per sequence")
        cl = host_context_lens
    else:
        cl = context_lens.cpu()
    if cl.numel() == 0:
        return
    a = cl.numpy()  # a view: numpy's reductions cost less per call than torch's on the CPU
    _require(int(a.min()) >= 1, "context_lens must be >= 1 (empty sequences unsupported)")
    _require(int(a.max()) <= capacity, "context_lens exceeds max_blocks_per_seq * block_size")


def _check_decode_args(out, q, k_cache, v_cache, block_table, context_lens, block_size,
                       kind, k_scales, v_scales, act_dtype=torch.float16):
    scaled = kind != "f16"  # one-byte cache with per-token scales (int8 or fp8)
    _require(q.is_cuda and (out is None or out.is_cuda), "tensors must be on CUDA")
    act_name = "fp16" if act_dtype == torch.float16 else "bf16"
    _require(q.dtype == act_dtype, f"q must be {act_name}")
    if kind == "f8":
        _require(k_cache.dtype == _FP8, "k_cache must be float8_e4m3fn")
        _require(v_cache.dtype == _FP8, "v_cache must be float8_e4m3fn")
    if kind == "i8":
        _require(k_cache.dtype == torch.int8, "k_cache must be int8")
        _require(v_cache.dtype == torch.int8, "v_cache must be int8")
    if scaled:
        _require(k_scales is not None and k_scales.dtype == torch.float32,
                 "k_scales must be fp32")
        _require(v_scales is not None and v_scales.dtype == torch.float32,
                 "v_scales must be fp32")
    else:
        _require(k_cache.dtype == torch.float16, "k_cache must be fp16")
        _require(v_cache.dtype == torch.float16, "v_cache must be fp16")
    _require(block_table.dtype == torch.int32, "block_table must be int32")
    _require(context_lens.dtype == torch.int32, "context_lens must be int32")
    dev = q.device
    tensors = [q, k_cache, v_cache, block_table, context_lens]
    if out is not None:
        tensors.append(out)
    if scaled:
        tensors += [k_scales, v_scales]
    for t in tensors:
        _require(t.device == dev, "all tensors must be on the same CUDA device")
        _require(t.is_contiguous(), "all tensors must be contiguous")
    _require(q.dim() == 3, "q must be [num_seqs, num_heads, head_dim]")
    B, H, D = q.shape
    if out is not None:
        _require(tuple(out.shape) == (B, H, D) and out.dtype == act_dtype,
                 f"out must be {act_name} with the shape of q")
    _require(k_cache.dim() == 5,
             "k_cache must be [num_blocks, kv_heads, head_dim/x, block_size, x]")
    NB, KVH, DX, BS, x = k_cache.shape
    if scaled:
        _require(x == 8, "int8 K cache requires x == 8")
    _require(x == X, "K cache requires x == 8")
    _require(D == HEAD_DIM, f"head_dim {D} unsupported (this build: {HEAD_DIM})")
    _require(DX * x == D, "k_cache head_dim/x does not match q")
    _require(block_size % 16 == 0 and 128 % block_size == 0,
             "block_size must divide TILE (multiple of 16)")
    _require(BS == block_size, f"k_cache block dimension {BS} != block_size {block_size}")
    _require(tuple(v_cache.shape) == (NB, KVH, D, block_size),
             "v_cache must be [num_blocks, kv_heads, head_dim, block_size]")
    if scaled:
        _require(tuple(k_scales.shape) == (NB, KVH, block_size) and
                 tuple(v_scales.shape) == (NB, KVH, block_size),
                 "scales must be [num_blocks, kv_heads, block_size]")
    _require(KVH > 0 and H % KVH == 0, "num_heads must be a multiple of num_kv_heads")
    _require(block_table.dim() == 2 and block_table.shape[0] == B,
             "block_table must be [num_seqs, max_blocks_per_seq]")
    _require(context_lens.dim() == 1 and context_lens.shape[0] == B,
             "context_lens must be [num_seqs]")
    return B, H, KVH, D, NB


def decode(out, q, k_cache, v_cache, block_table, context_lens, scale, block_size=16, *,
           k_scales=None, v_scales=None, splitk=False, validate=True, kv_kind=None,
           host_context_lens=None):
    """Paged decode attention into `out` (fp16 [num_seqs, num_heads, head_dim]).

    The cache type follows the tensors: fp16; int8 or float8_e4m3fn, each with per-token fp32
    k_scales/v_scales (an int8 cache is assumed whenever scales are given). splitk
    selects the partition + LSE-reduce kernel pair (512-token splits); otherwise the
    single-pass kernel with the fused combine runs. validate=False skips the one host sync
    that checks context_lens (the kernels still flag bad lengths in the status word).
    kv_kind ('f16', 'i8' or 'f8') pins the cache type instead of inferring it from the
    tensors, so a cache of another type is rejected (the reference-named ops use this).
    host_context_lens, a CPU tensor holding the same lengths (for instance the pinned copy the
    lengths were uploaded from), moves that check to the host: the call then does not
    synchronise.
    """
    kind = kv_kind or _kv_kind(k_cache, k_scales)
    B, H, KVH, D, NB = _check_decode_args(out, q, k_cache, v_cache, block_table, context_lens,
                                          block_size, kind, k_scales, v_scales)
    if B == 0:
        return out
    L = _lib.lib()
    max_blocks = block_table.shape[1]
    with _Guard(q.device):
        kv = _KV_CODE[kind]
        need = L.pa_decode_workspace_bytes(B, H, KVH, D, max_blocks, block_size, kv,
                                           1 if splitk else 0)
        _require(need > 0, "unsupported decode shape: " + _lib.last_error())
        ws = workspace(q.device, need)
        stream = _stream(q.device)
        if kind != "f16":
            if kind == "f8":
                fn = L.pa_splitk_fp8 if splitk else L.pa_decode_fp8
            else:
                fn = L.pa_splitk_i8 if splitk else L.pa_decode_i8
            args = (out.data_ptr(), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                    k_scales.data_ptr(), v_scales.data_ptr(), block_table.data_ptr(),
                    context_lens.data_ptr(), B, H, KVH, D, NB, block_size, max_blocks,
                    float(scale), ws.data_ptr(), ws.numel(), stream)
        else:
            fn = L.pa_splitk_f16 if splitk else L.pa_decode_f16
            args = (out.data_ptr(), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                    block_table.data_ptr(), context_lens.data_ptr(), B, H, KVH, D, NB,
                    block_size, max_blocks, float(scale), ws.data_ptr(), ws.numel(), stream)
        # The one host sync (if any) comes last, so the launch follows it with no Python work
        # between.
        if validate:
            _check_lengths(context_lens, max_blocks * block_size, host_context_lens)
        _lib.check(fn(*args), "paged decode")
    return out


class DecodePlan:
    """decode() for a serving loop: the argument checks run once, at construction.

    Construction takes the same arguments as decode() and validates them the same way; it
    resolves the entry point, the launch sizes and the cache pointers. run() launches the
    decode on the current stream, with the tensors given at construction or, per call, other
    out / q / block_table / context_lens tensors of the same shape, dtype and device (checked
    cheaply; anything else raises RuntimeError). The cache tensors stay those of construction.
    Results are identical to decode()'s. host_context_lens / validate behave as in decode().
    """

    def __init__(self, out, q, k_cache, v_cache, block_table, context_lens, scale, block_size=16,
                 *, k_scales=None, v_scales=None, splitk=False):
        kind = _kv_kind(k_cache, k_scales)
        B, H, KVH, D, NB = _check_decode_args(out, q, k_cache, v_cache, block_table,
                                              context_lens, block_size, kind, k_scales,
                                              v_scales)
        L = _lib.lib()
        self.max_blocks = block_table.shape[1]
        kv = _KV_CODE[kind]
        self.need = L.pa_decode_workspace_bytes(B, H, KVH, D, self.max_blocks, block_size, kv,
                                                1 if splitk else 0)
        _require(B == 0 or self.need > 0, "unsupported decode shape: " + _lib.last_error())
        if kind == "f8":
            self.fn = L.pa_splitk_fp8 if splitk else L.pa_decode_fp8
        elif kind == "i8":
            self.fn = L.pa_splitk_i8 if splitk else L.pa_decode_i8
        else:
            self.fn = L.pa_splitk_f16 if splitk else L.pa_decode_f16
        self.scaled = kind != "f16"
        self.device = q.device
        self.sizes = (B, H, KVH, D, NB, block_size, self.max_blocks, float(scale))
        self.caches = ((k_cache.data_ptr(), v_cache.data_ptr()) +
                       ((k_scales.data_ptr(), v_scales.data_ptr()) if self.scaled else ()))
        self._keep = (k_cache, v_cache, k_scales, v_scales)  # the cache tensors stay alive
        self.capacity = self.max_blocks * block_size
        self.tensors = [out, q, block_table, context_lens]
        self.specs = [(tuple(t.shape), t.dtype) for t in self.tensors]

    def _match(self, i, t):
        if t is None:
            return self.tensors[i]
        shape, dtype = self.specs[i]
        _require(t.dtype == dtype and tuple(t.shape) == shape and t.device == self.device and
                 t.is_contiguous(),
                 "DecodePlan.run: tensors must match the plan's shapes, dtypes and device")
        return t

    def run(self, out=None, q=None, block_table=None, context_lens=None, *,
            host_context_lens=None, validate=True):
        out, q = self._match(0, out), self._match(1, q)
        block_table, context_lens = self._match(2, block_table), self._match(3, context_lens)
        B, H, KVH, D, NB, bs, mb, scale = self.sizes
        if B == 0:
            return out
        with _Guard(self.device):
            ws = workspace(self.device, self.need)
            ptrs = (out.data_ptr(), q.data_ptr()) + self.caches[:2]
            if self.scaled:
                ptrs += self.caches[2:]
            args = ptrs + (block_table.data_ptr(), context_lens.data_ptr(), B, H, KVH, D, NB,
                           bs, mb, scale, ws.data_ptr(), ws.numel(), _stream(self.device))
            if validate:
                _check_lengths(context_lens, self.capacity, host_context_lens)
            _lib.check(self.fn(*args), "paged decode")
        return out


def decode_step(out, q, new_k, new_v, k_cache, v_cache, block_table, context_lens, scale,
                block_size=16, *, k_scales=None, v_scales=None, k_scale=None, v_scale=None,
                splitk=False, fused=None, validate=True, host_context_lens=None):
    """One decode step: append every sequence's new token to the cache, then decode.

    context_lens already counts the new token: new_k / new_v [num_seqs, kv_heads, head_dim]
    (fp16, bf16 or fp32 rows) go to position context_lens[b] - 1 of sequence b through
    block_table, written like quantize_into_cache (int8 cache, per-token scales or the
    per-tensor k_scale / v_scale), its FP8 counterpart or write_into_cache (fp16 cache); then
    the decode of decode() runs over the whole context. This is the bridge's
    PagedKVCache.decode_append + split-K op (benchmarks/int8_bridge/paged_cache.py:132-156,
    qwen_paged_attn.py:61-73) for a whole batch in one call. With fused=True (and at most 16 q
    heads per kv head) the decode kernel writes each token itself just before reading its
    page, so a step is one launch (two with splitk); fused=False runs the write as its own
    kernel first. Both give bit-identical caches and outputs. The default (fused=None) fuses
    small batches (at most 64 sequence x kv-head rows), where the saved launch dominates, and
    writes larger ones first: on a B200 the separate write measured 0.4 % faster at 128 rows
    and 2 % faster at 1024 rows, because the fused write lengthens the warps that carry it.

    With validate=False the call does no host synchronisation and allocates nothing once the
    stream's workspace exists, so after one call on a stream it can be captured in a CUDA
    graph (the kernels still flag bad lengths in the status word). host_context_lens (a CPU
    copy of the lengths) checks them on the host without synchronising, as in decode().
    """
    kind = _kv_kind(k_cache, k_scales)
    B, H, KVH, D, NB = _check_decode_args(out, q, k_cache, v_cache, block_table, context_lens,
                                          block_size, kind, k_scales, v_scales)
    _check_rows(new_k, new_v)
    if fused is None:
        fused = B * KVH <= 64
    _require(tuple(new_k.shape) == (B, KVH, D), "new_k/new_v must be [num_seqs, kv_heads, "
             "head_dim]")
    _require(new_k.device == q.device, "new_k/new_v must be on q's device")
    if k_scale is not None or v_scale is not None:
        _require(kind == "i8" and k_scale is not None and v_scale is not None,
                 "per-tensor scales need an int8 cache and both of k_scale and v_scale")
        for t in (k_scale, v_scale):
            _require(t.dtype == torch.float32 and t.numel() == 1 and t.device == q.device,
                     "fixed scales must be one fp32 element on q's device")
    if B == 0:
        return out
    L = _lib.lib()
    max_blocks = block_table.shape[1]
    with _Guard(q.device):
        kv = _KV_CODE[kind]
        need = L.pa_decode_workspace_bytes(B, H, KVH, D, max_blocks, block_size, kv,
                                           1 if splitk else 0)
        _require(need > 0, "unsupported decode shape: " + _lib.last_error())
        ws = workspace(q.device, need)
        args = (kv, out.data_ptr(), q.data_ptr(), new_k.data_ptr(), new_v.data_ptr(),
                _DTYPE_CODE[new_k.dtype], new_k.stride(0), k_cache.data_ptr(),
                v_cache.data_ptr(), _ptr(k_scales), _ptr(v_scales), _ptr(k_scale),
                _ptr(v_scale), block_table.data_ptr(), context_lens.data_ptr(), B, H, KVH, D, NB,
                block_size, max_blocks, float(scale), 1 if splitk else 0, 1 if fused else 0,
                ws.data_ptr(), ws.numel(), _stream(q.device))
        if validate:
            _check_lengths(context_lens, max_blocks * block_size, host_context_lens)
        _lib.check(L.pa_decode_step(*args), "paged decode step")
    return out


def decode_bf16(out, q, k_cache, v_cache, block_table, context_lens, scale, block_size=16, *,
                k_scales=None, v_scales=None, splitk=False, validate=True):
    """decode() with bf16 activations: q and out are bf16, the cache fp16, per-token INT8 or
    per-token FP8 (e4m3).

    q is converted to fp16 on the device (exact for magnitudes in the fp16 normal range; larger
    values saturate and set the PA_ERR_Q_RANGE status bit), the fp16 decode runs, and the output
    is rounded once to bf16.
    """
    kind = _kv_kind(k_cache, k_scales)
    int8 = kind != "f16"
    B, H, KVH, D, NB = _check_decode_args(out, q, k_cache, v_cache, block_table, context_lens,
                                          block_size, kind, k_scales, v_scales,
                                          act_dtype=torch.bfloat16)
    if B == 0:
        return out
    L = _lib.lib()
    max_blocks = block_table.shape[1]
    with _Guard(q.device):
        kv = _KV_CODE[kind]
        need = L.pa_decode_bf16q_workspace_bytes(B, H, KVH, D, max_blocks, block_size, kv,
                                                 1 if splitk else 0)
        _require(need > 0, "unsupported decode shape: " + _lib.last_error())
        ws = workspace(q.device, need)
        if validate:
            _check_lengths(context_lens, max_blocks * block_size)
        rc = L.pa_decode_bf16q(out.data_ptr(), q.data_ptr(), k_cache.data_ptr(),
                               v_cache.data_ptr(), _ptr(k_scales) if int8 else None,
                               _ptr(v_scales) if int8 else None, block_table.data_ptr(),
                               context_lens.data_ptr(), B, H, KVH, D, NB, block_size, max_blocks,
                               kv, 1 if splitk else 0, float(scale), ws.data_ptr(), ws.numel(),
                               _stream(q.device))
        _lib.check(rc, "paged decode (bf16 q)")
    return out


def partial_floats(num_heads, num_kv_heads, head_dim=HEAD_DIM):
    return _lib.lib().pa_partial_floats(num_heads, num_kv_heads, head_dim)


def decode_partial(q, k_cache, v_cache, block_table, context_lens, scale, block_size=16, *,
                   k_scales=None, v_scales=None, partials=None):
    """Un-normalised per-(sequence, kv-head) partials (O, m, l) for this device's token
    ranges: fp32 [num_seqs, num_kv_heads * slot]. Sequences with context 0 give empty
    partials. Used to split one sequence's context across GPUs."""
    kind = _kv_kind(k_cache, k_scales)
    B, H, KVH, D, NB = _check_decode_args(None, q, k_cache, v_cache, block_table, context_lens,
                                          block_size, kind, k_scales, v_scales)
    per = partial_floats(H, KVH, D) * KVH  # floats per sequence: kv_heads x head tiles x slot
    if partials is None:
        partials = torch.empty(B, per, dtype=torch.float32, device=q.device)
    _require(partials.dtype == torch.float32 and partials.is_contiguous() and
             partials.numel() == B * per, "partials must be fp32 [num_seqs, per_seq_floats]")
    if B == 0:
        return partials
    L = _lib.lib()
    max_blocks = block_table.shape[1]
    with _Guard(q.device):
        kv = _KV_CODE[kind]
        need = L.pa_decode_workspace_bytes(B, H, KVH, D, max_blocks, block_size, kv, 0)
        _require(need > 0, "unsupported decode shape: " + _lib.last_error())
        ws = workspace(q.device, need)
        rc = L.pa_decode_partial(kv, partials.data_ptr(), q.data_ptr(), k_cache.data_ptr(),
                                 v_cache.data_ptr(), _ptr(k_scales), _ptr(v_scales),
                                 block_table.data_ptr(), context_lens.data_ptr(), B, H, KVH, D,
                                 NB, block_size, max_blocks, float(scale), ws.data_ptr(),
                                 ws.numel(), _stream(q.device))
        _lib.check(rc, "partial decode")
    return partials


def merge_partials(out, partials, num_heads, num_kv_heads):
    """LSE-merge partials gathered from several GPUs, fp32 [num_parts, num_seqs, ...], into
    out fp16 [num_seqs, num_heads, head_dim]."""
    _require(out.is_cuda and partials.is_cuda, "tensors must be on CUDA")
    _require(partials.dtype == torch.float32 and partials.is_contiguous(),
             "partials must be contiguous fp32")
    P, B = partials.shape[0], partials.shape[1]
    _require(tuple(out.shape) == (B, num_heads, HEAD_DIM) and out.dtype == torch.float16,
             "out must be fp16 [num_seqs, num_heads, head_dim]")
    per = partial_floats(num_heads, num_kv_heads, HEAD_DIM) * num_kv_heads
    _require(per > 0 and partials.numel() == P * B * per,
             "partials must be fp32 [num_parts, num_seqs, per_seq_floats]")
    _require(partials.device == out.device, "partials and out must be on the same device")
    with _Guard(out.device):
        ws = workspace(out.device, 256)
        rc = _lib.lib().pa_merge_partials(out.data_ptr(), partials.data_ptr(), P, B, num_heads,
                                          num_kv_heads, HEAD_DIM, ws.data_ptr(),
                                          _stream(out.device))
        _lib.check(rc, "merge partials")
    return out


# ---------------------------------------------------------------------------------------
# Cache writes
# ---------------------------------------------------------------------------------------
def _check_cache_layout(k_cache, v_cache, num_kv_heads, head_dim, block_size, k_scales=None,
                        v_scales=None):
    """The paged layout the write kernels address, given the rows' kv-head count and head_dim:
    K [num_blocks, kv_heads, head_dim/8, block_size, 8], V [num_blocks, kv_heads, head_dim,
    block_size], scales [num_blocks, kv_heads, block_size] (tests/paged_decode_attn.py:76-81,
    156-164). The kernels take only num_blocks and block_size, so any other shape would be
    written out of bounds; it is rejected here. Returns num_blocks."""
    _require(k_cache.dim() == 5,
             "k_cache must be [num_blocks, kv_heads, head_dim/x, block_size, x]")
    NB = k_cache.shape[0]
    _require(head_dim % X == 0 and tuple(k_cache.shape) == (NB, num_kv_heads, head_dim // X,
                                                             block_size, X),
             f"k_cache must be [num_blocks, {num_kv_heads}, {head_dim // X}, {block_size}, {X}] "
             f"for these rows; got {tuple(k_cache.shape)}")
    _require(tuple(v_cache.shape) == (NB, num_kv_heads, head_dim, block_size),
             f"v_cache must be [{NB}, {num_kv_heads}, {head_dim}, {block_size}]; "
             f"got {tuple(v_cache.shape)}")
    for name, t in (("k_scales", k_scales), ("v_scales", v_scales)):
        if t is not None:
            _require(tuple(t.shape) == (NB, num_kv_heads, block_size),
                     f"{name} must be [{NB}, {num_kv_heads}, {block_size}]; got {tuple(t.shape)}")
    return NB


def _check_rows(key, value):
    _require(key.is_cuda and value.is_cuda, "tensors must be on CUDA")
    _require(key.dtype in _DTYPE_CODE and value.dtype == key.dtype,
             "key/value must both be fp16, bf16 or fp32")
    _require(key.dim() == 3 and key.shape == value.shape,
             "key/value must be [num_tokens, num_kv_heads, head_dim]")
    _require(key.stride(2) == 1 and key.stride(1) == key.shape[2] and
             value.stride() == key.stride(), "key/value rows must be contiguous")


def quantize_into_cache(key, value, k_cache, v_cache, k_scales, v_scales, slot_mapping,
                        block_size=16, *, k_scale=None, v_scale=None):
    """Per-token symmetric INT8 write of key/value [num_tokens, kv_heads, head_dim] into the
    paged cache at slot_mapping (int32, block*block_size+offset; negative = skip).

    Values and scales are bit-identical to quantize_per_token
    (tests/paged_decode_attn.py:106-112). With k_scale/v_scale (one fp32 device scalar each)
    the given per-tensor scale is used instead, as PagedKVCache.decode_append does in
    per-tensor mode (benchmarks/int8_bridge/paged_cache.py:142-145).
    """
    _check_rows(key, value)
    fp8 = _FP8 is not None and k_cache.dtype == _FP8
    if fp8:
        _require(v_cache.dtype == _FP8, "v_cache must be float8_e4m3fn like k_cache")
        _require(k_scale is None and v_scale is None,
                 "the fp8 cache write has per-token scales only")
    else:
        _require(k_cache.dtype == torch.int8 and v_cache.dtype == torch.int8,
                 "cache must be int8")
    _require(k_scales.dtype == torch.float32 and v_scales.dtype == torch.float32,
             "scales must be fp32")
    _require(slot_mapping.dtype == torch.int32 and slot_mapping.is_cuda,
             "slot_mapping must be int32 on CUDA")
    N, KVH, D = key.shape
    _require(slot_mapping.numel() == N, "slot_mapping must have one entry per token")
    _check_cache_layout(k_cache, v_cache, KVH, D, block_size, k_scales, v_scales)
    for t in (k_cache, v_cache, k_scales, v_scales, slot_mapping):
        _require(t.is_contiguous() and t.device == key.device,
                 "cache tensors must be contiguous and on the key's device")
    for t in (k_scale, v_scale):
        if t is not None:
            _require(t.dtype == torch.float32 and t.numel() == 1 and t.device == key.device,
                     "fixed scales must be one fp32 element on the key's device")
    with _Guard(key.device):
        ws = workspace(key.device, 256)
        if fp8:
            rc = _lib.lib().pa_quantize_into_cache_fp8(
                key.data_ptr(), value.data_ptr(), _DTYPE_CODE[key.dtype], key.stride(0),
                slot_mapping.data_ptr(), N, KVH, D, k_cache.data_ptr(), v_cache.data_ptr(),
                k_scales.data_ptr(), v_scales.data_ptr(), k_cache.shape[0], block_size,
                ws.data_ptr(), _stream(key.device))
            _lib.check(rc, "quantize_into_cache (fp8)")
            return
        rc = _lib.lib().pa_quantize_into_cache(
            key.data_ptr(), value.data_ptr(), _DTYPE_CODE[key.dtype], key.stride(0),
            slot_mapping.data_ptr(), N, KVH, D, k_cache.data_ptr(), v_cache.data_ptr(),
            k_scales.data_ptr(), v_scales.data_ptr(), k_cache.shape[0], block_size,
            _ptr(k_scale), _ptr(v_scale), ws.data_ptr(), _stream(key.device))
        _lib.check(rc, "quantize_into_cache")


def write_into_cache(key, value, k_cache, v_cache, slot_mapping, block_size=16):
    """FP16 copy of key/value [num_tokens, kv_heads, head_dim] into an fp16 paged cache."""
    _check_rows(key, value)
    _require(k_cache.dtype == torch.float16 and v_cache.dtype == torch.float16,
             "cache must be fp16")
    _require(slot_mapping.dtype == torch.int32 and slot_mapping.is_cuda,
             "slot_mapping must be int32 on CUDA")
    N, KVH, D = key.shape
    _require(slot_mapping.numel() == N, "slot_mapping must have one entry per token")
    _check_cache_layout(k_cache, v_cache, KVH, D, block_size)
    for t in (k_cache, v_cache, slot_mapping):
        _require(t.is_contiguous() and t.device == key.device,
                 "cache tensors must be contiguous and on the key's device")
    with _Guard(key.device):
        ws = workspace(key.device, 256)
        rc = _lib.lib().pa_write_into_cache_f16(
            key.data_ptr(), value.data_ptr(), _DTYPE_CODE[key.dtype], key.stride(0),
            slot_mapping.data_ptr(), N, KVH, D, k_cache.data_ptr(), v_cache.data_ptr(),
            k_cache.shape[0], block_size, ws.data_ptr(), _stream(key.device))
        _lib.check(rc, "write_into_cache")


def prefill_into_cache(k, v, k_cache, v_cache, block_table, context_lens, block_size=16, *,
                       k_scales=None, v_scales=None, k_scale=None, v_scale=None):
    """Bulk write of contiguous per-sequence K/V [num_seqs, max_len, kv_heads, head_dim] into
    the blocks listed by block_table (a warp per 16-token group of one page, K or V, its rows
    loaded into registers together; 16-byte stores into the page layout). INT8
    caches are quantised per token (or with k_scale/v_scale); FP16 caches get a copy.
    Tokens past a sequence's context inside its last block are written as zeros."""
    _require(k.is_cuda and v.is_cuda, "tensors must be on CUDA")
    _require(k.dtype in _DTYPE_CODE and v.dtype == k.dtype, "k/v must be fp16, bf16 or fp32")
    _require(k.dim() == 4 and k.shape == v.shape and k.is_contiguous() and v.is_contiguous(),
             "k/v must be contiguous [num_seqs, max_len, kv_heads, head_dim]")
    S, Lmax, KVH, D = k.shape
    int8 = k_cache.dtype == torch.int8
    _require(int8 or k_cache.dtype == torch.float16, "cache must be int8 or fp16")
    _require(block_table.dtype == torch.int32 and context_lens.dtype == torch.int32,
             "block_table and context_lens must be int32")
    _require(block_table.dim() == 2 and block_table.shape[0] == S and context_lens.numel() == S,
             "block_table must be [num_seqs, max_blocks] and context_lens [num_seqs]")
    tensors = [k_cache, v_cache, block_table, context_lens]
    if int8:
        _require(k_scales is not None and v_scales is not None, "int8 cache needs scales")
        tensors += [k_scales, v_scales]
    _check_cache_layout(k_cache, v_cache, KVH, D, block_size, k_scales if int8 else None,
                        v_scales if int8 else None)
    for t in tensors:
        _require(t.is_contiguous() and t.device == k.device,
                 "cache tensors must be contiguous and on k's device")
    with _Guard(k.device):
        ws = workspace(k.device, 256)
        rc = _lib.lib().pa_prefill_into_cache(
            k.data_ptr(), v.data_ptr(), _DTYPE_CODE[k.dtype], S, Lmax, KVH, D,
            block_table.data_ptr(), context_lens.data_ptr(), block_table.shape[1],
            _lib.PA_DTYPE_I8 if int8 else _lib.PA_DTYPE_F16, k_cache.data_ptr(),
            v_cache.data_ptr(), _ptr(k_scales), _ptr(v_scales), k_cache.shape[0], block_size,
            _ptr(k_scale), _ptr(v_scale), ws.data_ptr(), _stream(k.device))
        _lib.check(rc, "prefill_into_cache")


def absmax_scale(x, semantics=_lib.PA_SCALE_CLAMP_THEN_DIVIDE):
    """Per-tensor INT8 scale of x as a 0-d fp32 device tensor.

    CLAMP_THEN_DIVIDE matches quantize_per_tensor (tests/paged_decode_attn.py:118-119);
    DIVIDE_THEN_CLAMP matches PagedKVCache.prefill's per-tensor scale
    (benchmarks/int8_bridge/paged_cache.py:101-102)."""
    _require(x.is_cuda and x.dtype in _DTYPE_CODE and x.is_contiguous(),
             "x must be a contiguous fp16/bf16/fp32 CUDA tensor")
    out = torch.empty((), dtype=torch.float32, device=x.device)
    with _Guard(x.device):
        scratch = torch.empty(1, dtype=torch.int32, device=x.device)
        rc = _lib.lib().pa_absmax_scale(x.data_ptr(), _DTYPE_CODE[x.dtype], x.numel(),
                                        out.data_ptr(), semantics, scratch.data_ptr(),
                                        _stream(x.device))
        _lib.check(rc, "absmax_scale")
    return out
