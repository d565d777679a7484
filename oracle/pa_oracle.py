"""CPU oracle for the paged-attention decode path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference algorithm (Yevsquant/cuda-PA-INT8). Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg may import it; the product path
(pa_b200) never does. Parity is pinned: tests/test_oracle_golden.py checks every function
here against golden vectors that tests/golden/make_golden.py produced by running the
reference's own torch implementation.

Each function cites the reference lines it restates:
  quantize_per_token     tests/paged_decode_attn.py:106-112
  quantize_per_tensor    tests/paged_decode_attn.py:115-121
  dequantize_kv          tests/paged_decode_attn.py:202-216
  paged_decode_attention tests/paged_decode_attn.py:4-49 (scale as a parameter, as the CUDA
                         launchers take it; the reference oracle hard-codes 1/sqrt(D) at :45)
  scatter_paged_cache    the scatter of build_paged_kv_cache{,_int8} (:84-99, :178-197) with a
                         caller-supplied block table
  split_partials/lse_merge  split-K partition + reduce (kernels/paged_attention_v4_splitk.cu:
                         28-153, 156-187)
  BridgeCacheOracle      benchmarks/int8_bridge/paged_cache.py:41-156
  quantize_per_token_fp8 / dequantize_fp8: the FP8 (e4m3) cache format of this library,
                         which has no reference counterpart (the reference lists FP8 KV as
                         future work, report/benchmark_report.md:196-197); its e4m3 rounding
                         is torch's float8_e4m3fn conversion, pinned against CUDA's own
                         conversion by tests/test_fp8_cpu.py
Dtypes: "f16" inputs are np.float16 arrays; "f32" np.float32; "bf16" are np.float32 arrays
holding bfloat16-representable values (numpy has no bfloat16).
"""

import math

import numpy as np

LOG2E = 1.4426950408889634


# ---------------------------------------------------------------------------------------
# Rounding helpers
# ---------------------------------------------------------------------------------------
def round_to_bf16(x):
    """Round float32 values to the nearest bfloat16 (ties to even); returns float32."""
    x = np.asarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, r).astype(np.float32)


def round_to(x32, in_dtype):
    """Round float32 values into the input dtype and widen back to float32."""
    x32 = np.asarray(x32, dtype=np.float32)
    if in_dtype == "f16":
        return x32.astype(np.float16).astype(np.float32)
    if in_dtype == "bf16":
        return round_to_bf16(x32)
    if in_dtype == "f32":
        return x32
    raise ValueError(in_dtype)


def clamp_floor(in_dtype):
    """The reference's clamp_min(1e-8) bound, as represented in the input dtype."""
    return round_to(np.float32(1e-8), in_dtype)


# ---------------------------------------------------------------------------------------
# Quantisation (tests/paged_decode_attn.py:106-121)
# ---------------------------------------------------------------------------------------
def scale_from_amax(amax32, in_dtype):
    """scale = T(max(amax, T(1e-8)) / 127) in fp32 (paged_decode_attn.py:109-110)."""
    a = np.maximum(np.asarray(amax32, dtype=np.float32), clamp_floor(in_dtype))
    return round_to((a / np.float32(127.0)).astype(np.float32), in_dtype)


def quantize_with_scale(x32, scale):
    """round-half-even(x / scale) clamped to [-127, 127] as int8; NaN (0/0) becomes 0 as it
    does in the reference's CPU cast (paged_decode_attn.py:111, paged_cache.py:34-38)."""
    x32 = np.asarray(x32, dtype=np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        r = np.rint((x32 / np.asarray(scale, dtype=np.float32)).astype(np.float32))
    r = np.clip(r, -127, 127)
    return np.where(np.isnan(r), 0, r).astype(np.int8)


def quantize_per_token(x, in_dtype):
    """Per-token symmetric INT8 over the last axis: (int8 values, fp32 scales)."""
    x32 = np.asarray(x).astype(np.float32)
    amax = np.abs(x32).max(axis=-1)
    s = scale_from_amax(amax, in_dtype)
    return quantize_with_scale(x32, s[..., None]), s


def quantize_per_tensor(x, in_dtype):
    """One scale for the whole tensor (paged_decode_attn.py:115-121)."""
    x32 = np.asarray(x).astype(np.float32)
    s = scale_from_amax(np.abs(x32).max() if x32.size else np.float32(0), in_dtype)
    return quantize_with_scale(x32, s), np.float32(s)


def bridge_tensor_scale(x, in_dtype):
    """PagedKVCache.prefill per-tensor scale: T(amax/127) -> fp32 -> clamp_min(1e-8)
    (benchmarks/int8_bridge/paged_cache.py:101-102)."""
    x32 = np.asarray(x).astype(np.float32)
    amax = np.abs(x32).max() if x32.size else np.float32(0)
    s = round_to((np.float32(amax) / np.float32(127.0)).astype(np.float32), in_dtype)
    return np.float32(max(np.float32(s), np.float32(1e-8)))


def dequantize_kv(k_cache, v_cache, k_scales, v_scales):
    """fp32 K/V from int8 + per-token scales (paged_decode_attn.py:202-216)."""
    k = k_cache.astype(np.float32) * k_scales[:, :, None, :, None]
    v = v_cache.astype(np.float32) * v_scales[:, :, None, :]
    return k, v


FP8_MAX = 448.0  # largest finite e4m3 value


def quantize_per_token_fp8(x):
    """Per-token e4m3: scale = amax / 448 (fp32, IEEE divide), q = e4m3(x / scale) with
    round-to-nearest-even and saturation to +-448; zero rows give scale 0 and zeros. Returns
    (q as uint8 e4m3 bit patterns, fp32 scales over all but the last axis)."""
    import torch
    xf = np.asarray(x, dtype=np.float32)
    amax = np.abs(xf).max(axis=-1)
    scale = (amax / np.float32(FP8_MAX)).astype(np.float32)
    safe = np.where(scale > 0, scale, np.float32(1)).astype(np.float32)
    y = np.clip(xf / safe[..., None], -FP8_MAX, FP8_MAX).astype(np.float32)
    q = torch.from_numpy(np.ascontiguousarray(y)).to(torch.float8_e4m3fn).view(torch.uint8)
    q = np.where(scale[..., None] > 0, q.numpy(), 0).astype(np.uint8)
    return q, scale


def fp8_to_float(q_u8):
    """float32 values of uint8 e4m3 bit patterns."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(q_u8, dtype=np.uint8)).view(torch.float8_e4m3fn)
    return t.float().numpy()


def dequantize_fp8(k_cache, v_cache, k_scales, v_scales):
    """fp32 K/V from an e4m3 (uint8 bit patterns) paged cache + per-token scales."""
    k = fp8_to_float(k_cache) * k_scales[:, :, None, :, None]
    v = fp8_to_float(v_cache) * v_scales[:, :, None, :]
    return k, v


# ---------------------------------------------------------------------------------------
# Paged layout
# ---------------------------------------------------------------------------------------
def gather_seq(k_cache, v_cache, block_table, ctx, b):
    """Contiguous K, V [ctx, kv_heads, D] of sequence b from the paged cache."""
    NB, KVH, DX, BS, X = k_cache.shape
    t = np.arange(ctx)
    blk = block_table[b, t // BS]
    off = t % BS
    k = k_cache[blk, :, :, off, :].reshape(ctx, KVH, DX * X)
    v = v_cache[blk, :, :, off]
    return k, v


def scatter_paged_cache(k, v, context_lens, block_table, num_blocks, block_size=16, x=8,
                        dtype=None):
    """Write contiguous per-sequence K/V [S, L, KVH, D] into a zeroed paged cache at the
    physical blocks of block_table (the scatter of paged_decode_attn.py:84-99)."""
    S, L, KVH, D = k.shape
    dtype = dtype or k.dtype
    k_cache = np.zeros((num_blocks, KVH, D // x, block_size, x), dtype=dtype)
    v_cache = np.zeros((num_blocks, KVH, D, block_size), dtype=dtype)
    for b in range(S):
        n = int(context_lens[b])
        t = np.arange(n)
        blk = block_table[b, t // block_size]
        off = t % block_size
        k_cache[blk, :, :, off, :] = k[b, :n].reshape(n, KVH, D // x, x)
        v_cache[blk, :, :, off] = v[b, :n]
    return k_cache, v_cache


def scatter_scales(scales, context_lens, block_table, num_blocks, kv_heads, block_size=16):
    """Per-token scales [S, L, KVH] into [num_blocks, KVH, block_size] (paged_decode_attn.py:
    195-197)."""
    out = np.zeros((num_blocks, kv_heads, block_size), dtype=np.float32)
    for b in range(scales.shape[0]):
        n = int(context_lens[b])
        t = np.arange(n)
        out[block_table[b, t // block_size], :, t % block_size] = scales[b, :n]
    return out


# ---------------------------------------------------------------------------------------
# Decode attention (tests/paged_decode_attn.py:4-49)
# ---------------------------------------------------------------------------------------
def paged_decode_attention(q, k_cache, v_cache, block_table, context_lens, scale=None,
                           acc=np.float64):
    """Vectorised per-sequence restatement; returns float32 [S, H, D]."""
    S, H, D = q.shape
    KVH = k_cache.shape[1]
    G = H // KVH
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    out = np.zeros((S, H, D), dtype=np.float32)
    for b in range(S):
        n = int(context_lens[b])
        k, v = gather_seq(k_cache, v_cache, block_table, n, b)
        k = k.astype(acc).transpose(1, 0, 2)            # [KVH, n, D]
        v = v.astype(acc).transpose(1, 0, 2)
        qb = q[b].astype(acc).reshape(KVH, G, D)
        s = np.matmul(qb, k.transpose(0, 2, 1)) * scale    # [KVH, G, n]
        s -= s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=-1, keepdims=True)
        out[b] = np.matmul(p, v).reshape(H, D).astype(np.float32)
    return out


def paged_decode_attention_loop(q, k_cache, v_cache, block_table, context_lens, block_size=16):
    """Token-by-token restatement with the reference's control flow and its fixed
    1/sqrt(head_dim) scale (paged_decode_attn.py:17-47); pure Python, small cases only."""
    S, H, D = q.shape
    KVH = k_cache.shape[1]
    qpk = H // KVH
    out = np.zeros((S, H, D), dtype=np.float32)
    for b in range(S):
        n = int(context_lens[b])
        ks, vs = [], []
        for i in range(n):
            blk = int(block_table[b, i // block_size])
            off = i % block_size
            ks.append(k_cache[blk, :, :, off, :].reshape(KVH, D).astype(np.float32))
            vs.append(v_cache[blk, :, :, off].astype(np.float32))
        ks = np.stack(ks, axis=1)
        vs = np.stack(vs, axis=0)
        for h in range(H):
            kvh = h // qpk
            sc = (ks[kvh] @ q[b, h].astype(np.float32)) / np.float32(math.sqrt(D))
            sc = sc - sc.max()
            p = np.exp(sc)
            p = p / p.sum()
            out[b, h] = (p[:, None] * vs[:, kvh, :]).sum(axis=0)
    return out


# ---------------------------------------------------------------------------------------
# Split-K partials and the LSE merge (kernels/paged_attention_v4_splitk.cu:28-187)
# ---------------------------------------------------------------------------------------
def range_partials(q, k_cache, v_cache, block_table, context_lens, t_lo, t_hi, scale):
    """Un-normalised partial over tokens [t_lo[b], t_hi[b]) of every sequence, natural-log
    units: (m [S, H], l [S, H], acc [S, H, D]); an empty range gives m=-inf, l=0, acc=0."""
    S, H, D = q.shape
    KVH = k_cache.shape[1]
    G = H // KVH
    m = np.full((S, H), -np.inf)
    l = np.zeros((S, H))
    acc = np.zeros((S, H, D))
    for b in range(S):
        lo, hi = int(t_lo[b]), int(t_hi[b])
        if hi <= lo:
            continue
        k, v = gather_seq(k_cache, v_cache, block_table, hi, b)
        k = k[lo:hi].astype(np.float64).transpose(1, 0, 2)
        v = v[lo:hi].astype(np.float64).transpose(1, 0, 2)
        qb = q[b].astype(np.float64).reshape(KVH, G, D)
        s = np.einsum("kgd,knd->kgn", qb, k) * scale
        mb = s.max(axis=-1)
        p = np.exp(s - mb[..., None])
        m[b] = mb.reshape(H)
        l[b] = p.sum(axis=-1).reshape(H)
        acc[b] = np.einsum("kgn,knd->kgd", p, v).reshape(H, D)
    return m, l, acc


LOG2E = 1.4426950408889634


def _slot_shape(num_heads, num_kv_heads, head_dim=128):
    G = num_heads // num_kv_heads
    GT = 8 if G <= 8 else 16
    HT = -(-G // GT)
    return G, GT, HT, (head_dim + 2) * GT


def pack_slots(m, l, acc, num_kv_heads):
    """Partials (m, l [S, H] natural-log units, acc [S, H, D]) in the slot layout the CUDA
    partial decode writes: fp32 [S, num_kv_heads * head_tiles * slot], a slot per (kv head,
    head tile) holding O[D][GT], then m[GT] in log2 units, then l[GT]; head rows past the
    group are empty (m = -inf, l = 0)."""
    S, H, D = acc.shape
    G, GT, HT, SLOT = _slot_shape(H, num_kv_heads, D)
    out = np.zeros((S, num_kv_heads * HT, SLOT), np.float32)
    for kvh in range(num_kv_heads):
        for ht in range(HT):
            seg = kvh * HT + ht
            o = np.zeros((S, D, GT), np.float32)
            mm = np.full((S, GT), -np.inf, np.float32)
            ll = np.zeros((S, GT), np.float32)
            for h in range(min(GT, G - ht * GT)):
                qh = kvh * G + ht * GT + h
                o[:, :, h] = acc[:, qh, :]
                mm[:, h] = m[:, qh] * LOG2E
                ll[:, h] = l[:, qh]
            out[:, seg, :D * GT] = o.reshape(S, D * GT)
            out[:, seg, D * GT:D * GT + GT] = mm
            out[:, seg, D * GT + GT:] = ll
    return out.reshape(S, -1)


def unpack_slots(slots, num_heads, num_kv_heads, head_dim=128):
    """Inverse of pack_slots: (m, l, acc) in natural-log units from [..., S, per_seq]."""
    slots = np.asarray(slots, np.float64)
    lead = slots.shape[:-1]
    G, GT, HT, SLOT = _slot_shape(num_heads, num_kv_heads, head_dim)
    x = slots.reshape(lead + (num_kv_heads * HT, SLOT))
    D = head_dim
    m = np.full(lead + (num_heads,), -np.inf)
    l = np.zeros(lead + (num_heads,))
    acc = np.zeros(lead + (num_heads, D))
    for kvh in range(num_kv_heads):
        for ht in range(HT):
            seg = x[..., kvh * HT + ht, :]
            o = seg[..., :D * GT].reshape(lead + (D, GT))
            for h in range(min(GT, G - ht * GT)):
                qh = kvh * G + ht * GT + h
                acc[..., qh, :] = o[..., :, h]
                m[..., qh] = seg[..., D * GT + h] / LOG2E
                l[..., qh] = seg[..., D * GT + GT + h]
    return m, l, acc


def lse_merge(ms, ls, accs):
    """Merge partials stacked on axis 0: out = sum acc_s e^{m_s-M} / sum l_s e^{m_s-M}."""
    ms, ls, accs = np.asarray(ms), np.asarray(ls), np.asarray(accs)
    M = ms.max(axis=0)
    w = np.where(np.isneginf(ms), 0.0, np.exp(ms - M[None]))
    L = (w * ls).sum(axis=0)
    O = (w[..., None] * accs).sum(axis=0)
    return (O / L[..., None]).astype(np.float32)


def split_partials(q, k_cache, v_cache, block_table, context_lens, scale, split=512):
    """Per-split partials of the split-K partition kernel: lists over splits of (m, l, acc)."""
    n_split = max(1, -(-int(np.max(context_lens)) // split))
    parts = []
    for s in range(n_split):
        lo = np.minimum(context_lens, s * split)
        hi = np.minimum(context_lens, (s + 1) * split)
        parts.append(range_partials(q, k_cache, v_cache, block_table, context_lens, lo, hi,
                                    scale))
    return parts


# ---------------------------------------------------------------------------------------
# Bridge cache (benchmarks/int8_bridge/paged_cache.py:41-156), single layer
# ---------------------------------------------------------------------------------------
class BridgeCacheOracle:
    def __init__(self, num_kv_heads, head_dim, max_len, block_size=16, x=8, variant="fp16",
                 in_dtype="f16"):
        self.H, self.D, self.bs, self.x = num_kv_heads, head_dim, block_size, x
        self.variant = variant
        self.in_dtype = in_dtype
        self.is_int8 = variant != "fp16"
        nb = (max_len + block_size - 1) // block_size
        self.num_blocks = nb
        st = np.int8 if self.is_int8 else np.float16
        self.k_cache = np.zeros((nb, num_kv_heads, head_dim // x, block_size, x), dtype=st)
        self.v_cache = np.zeros((nb, num_kv_heads, head_dim, block_size), dtype=st)
        self.k_scales = np.zeros((nb, num_kv_heads, block_size), dtype=np.float32)
        self.v_scales = np.zeros((nb, num_kv_heads, block_size), dtype=np.float32)
        self.k_tensor_scale = None
        self.v_tensor_scale = None
        self.length = 0

    def _rows(self, k, v):
        if self.variant == "int8_per_token":
            kq, ks = quantize_per_token(k, self.in_dtype)
            vq, vs = quantize_per_token(v, self.in_dtype)
        elif self.variant == "int8_per_tensor":
            kq = quantize_with_scale(np.asarray(k).astype(np.float32), self.k_tensor_scale)
            vq = quantize_with_scale(np.asarray(v).astype(np.float32), self.v_tensor_scale)
            ks = np.full(kq.shape[:-1], self.k_tensor_scale, dtype=np.float32)
            vs = np.full(vq.shape[:-1], self.v_tensor_scale, dtype=np.float32)
        else:
            kq = np.asarray(k).astype(np.float32).astype(np.float16)
            vq = np.asarray(v).astype(np.float32).astype(np.float16)
            ks = vs = None
        return kq, vq, ks, vs

    def prefill(self, k, v):
        L = k.shape[0]
        if self.variant == "int8_per_tensor":
            self.k_tensor_scale = bridge_tensor_scale(k, self.in_dtype)
            self.v_tensor_scale = bridge_tensor_scale(v, self.in_dtype)
        kq, vq, ks, vs = self._rows(k, v)
        nb = (L + self.bs - 1) // self.bs
        P = nb * self.bs
        kp = np.zeros((P, self.H, self.D), dtype=kq.dtype)
        vp = np.zeros((P, self.H, self.D), dtype=vq.dtype)
        kp[:L], vp[:L] = kq, vq
        self.k_cache[:nb] = kp.reshape(nb, self.bs, self.H, self.D // self.x, self.x).transpose(
            0, 2, 3, 1, 4)
        self.v_cache[:nb] = vp.reshape(nb, self.bs, self.H, self.D).transpose(0, 2, 3, 1)
        if self.is_int8:
            ksp = np.zeros((P, self.H), dtype=np.float32)
            vsp = np.zeros((P, self.H), dtype=np.float32)
            ksp[:L], vsp[:L] = ks, vs
            self.k_scales[:nb] = ksp.reshape(nb, self.bs, self.H).transpose(0, 2, 1)
            self.v_scales[:nb] = vsp.reshape(nb, self.bs, self.H).transpose(0, 2, 1)
        self.length = L

    def decode_append(self, k, v):
        t = self.length
        blk, off = t // self.bs, t % self.bs
        kq, vq, ks, vs = self._rows(k, v)
        self.k_cache[blk, :, :, off, :] = kq.reshape(self.H, self.D // self.x, self.x)
        self.v_cache[blk, :, :, off] = vq
        if self.is_int8:
            self.k_scales[blk, :, off] = ks
            self.v_scales[blk, :, off] = vs
        self.length = t + 1
        return t + 1
