"""Per-layer paged K/V cache with the interface of the reference bridge cache
(benchmarks/int8_bridge/paged_cache.py:41-183), written by this library's kernels.

Same constructor, variants ("fp16", "int8_per_token", "int8_per_tensor"), layouts and
methods (prefill, decode_append, context_lens, kv_bytes, kv_bytes_for_len, reset). The
reference quantises and scatters with torch ops; here prefill is one block-granular kernel
(pa_prefill_into_cache) and decode_append one token-granular kernel (pa_quantize_into_cache
or pa_write_into_cache_f16), with bit-identical cache contents.
"""

import torch

from . import _lib, ops


class PagedKVCache:
    def __init__(self, num_layers, num_kv_heads, head_dim, max_len, block_size=16, x=8,
                 variant="fp16", device="cuda"):
        assert variant in ("fp16", "int8_per_token", "int8_per_tensor")
        assert head_dim % x == 0
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.block_size = block_size
        self.x = x
        self.variant = variant
        self.is_int8 = variant != "fp16"
        self.device = device

        self.num_blocks = (max_len + block_size - 1) // block_size
        store_dtype = torch.int8 if self.is_int8 else torch.float16
        self.k_cache = torch.zeros(num_layers, self.num_blocks, num_kv_heads, head_dim // x,
                                   block_size, x, dtype=store_dtype, device=device)
        self.v_cache = torch.zeros(num_layers, self.num_blocks, num_kv_heads, head_dim,
                                   block_size, dtype=store_dtype, device=device)
        if self.is_int8:
            self.k_scales = torch.zeros(num_layers, self.num_blocks, num_kv_heads, block_size,
                                        dtype=torch.float32, device=device)
            self.v_scales = torch.zeros(num_layers, self.num_blocks, num_kv_heads, block_size,
                                        dtype=torch.float32, device=device)
            self._k_tensor_scale = [None] * num_layers
            self._v_tensor_scale = [None] * num_layers
        # Contiguous identity block table shared across layers (batch = 1).
        self.block_table = torch.arange(self.num_blocks, dtype=torch.int32,
                                        device=device).view(1, -1)
        self.lengths = [0] * num_layers

    def reset(self):
        self.lengths = [0] * self.num_layers
        if self.is_int8:
            self._k_tensor_scale = [None] * self.num_layers
            self._v_tensor_scale = [None] * self.num_layers

    # --- write path -------------------------------------------------------------------------
    def prefill(self, layer_idx, k, v):
        """Scatter the prompt's K/V [L, num_kv_heads, head_dim] into positions [0, L)."""
        L, H, D = k.shape
        assert H == self.num_kv_heads and D == self.head_dim
        k4 = k.contiguous().view(1, L, H, D)
        v4 = v.contiguous().view(1, L, H, D)
        lens = torch.tensor([L], dtype=torch.int32, device=self.device)
        kw = {}
        if self.is_int8:
            kw = dict(k_scales=self.k_scales[layer_idx], v_scales=self.v_scales[layer_idx])
        if self.variant == "int8_per_tensor":
            sk = ops.absmax_scale(k.contiguous(), _lib.PA_SCALE_DIVIDE_THEN_CLAMP)
            sv = ops.absmax_scale(v.contiguous(), _lib.PA_SCALE_DIVIDE_THEN_CLAMP)
            self._k_tensor_scale[layer_idx] = sk
            self._v_tensor_scale[layer_idx] = sv
            kw.update(k_scale=sk, v_scale=sv)
        ops.prefill_into_cache(k4, v4, self.k_cache[layer_idx], self.v_cache[layer_idx],
                               self.block_table, lens, self.block_size, **kw)
        self.lengths[layer_idx] = L

    def decode_append(self, layer_idx, k, v):
        """Append one token's K/V [num_kv_heads, head_dim]; returns the new length."""
        t = self.lengths[layer_idx]
        H, D = self.num_kv_heads, self.head_dim
        slot = torch.tensor([t], dtype=torch.int32, device=self.device)
        k3 = k.contiguous().view(1, H, D)
        v3 = v.contiguous().view(1, H, D)
        if self.is_int8:
            kw = {}
            if self.variant == "int8_per_tensor":
                kw = dict(k_scale=self._k_tensor_scale[layer_idx],
                          v_scale=self._v_tensor_scale[layer_idx])
            ops.quantize_into_cache(k3, v3, self.k_cache[layer_idx], self.v_cache[layer_idx],
                                    self.k_scales[layer_idx], self.v_scales[layer_idx], slot,
                                    self.block_size, **kw)
        else:
            ops.write_into_cache(k3, v3, self.k_cache[layer_idx], self.v_cache[layer_idx], slot,
                                 self.block_size)
        self.lengths[layer_idx] = t + 1
        return t + 1

    def append_and_decode(self, layer_idx, k, v, q, scale, out=None):
        """decode_append(layer_idx, k, v) followed by the split-K decode of q [1, num_q_heads,
        head_dim] over the layer's cache -- the bridge's decode step
        (benchmarks/int8_bridge/qwen_paged_attn.py:61-73) -- as one call (for this one
        sequence the token is written by the decode kernel itself). Returns out
        [1, num_q_heads, head_dim] fp16."""
        t = self.lengths[layer_idx]
        H, D = self.num_kv_heads, self.head_dim
        q = q.contiguous()
        out = torch.empty_like(q) if out is None else out
        ctx = torch.tensor([t + 1], dtype=torch.int32, device=self.device)
        kw = {}
        if self.is_int8:
            kw = dict(k_scales=self.k_scales[layer_idx], v_scales=self.v_scales[layer_idx])
            if self.variant == "int8_per_tensor":
                kw.update(k_scale=self._k_tensor_scale[layer_idx],
                          v_scale=self._v_tensor_scale[layer_idx])
        ops.decode_step(out, q, k.contiguous().view(1, H, D), v.contiguous().view(1, H, D),
                        self.k_cache[layer_idx], self.v_cache[layer_idx], self.block_table, ctx,
                        scale, self.block_size, splitk=True, validate=False, **kw)
        self.lengths[layer_idx] = t + 1
        return out

    # --- read path --------------------------------------------------------------------------
    def context_lens(self, layer_idx):
        return torch.tensor([self.lengths[layer_idx]], dtype=torch.int32, device=self.device)

    def kv_bytes(self):
        b = self.k_cache.element_size() * self.k_cache.nelement()
        b += self.v_cache.element_size() * self.v_cache.nelement()
        if self.is_int8:
            b += self.k_scales.element_size() * self.k_scales.nelement()
            b += self.v_scales.element_size() * self.v_scales.nelement()
        return b

    def kv_bytes_for_len(self, n):
        blocks = (n + self.block_size - 1) // self.block_size
        elem = 1 if self.is_int8 else 2
        per_blk = 2 * self.num_kv_heads * self.head_dim * self.block_size
        b = blocks * per_blk * elem * self.num_layers
        if self.is_int8:
            b += blocks * 2 * self.num_kv_heads * self.block_size * 4 * self.num_layers
        return b
