"""Drop-in replacement for the reference's op module tests/cuda_ext.py.

Same names, call signatures and error conditions as the reference registry
(tests/cuda_ext.py:104-141 of Yevsquant/cuda-PA-INT8): `paged_decode_attention`, `VARIANTS`
(naive, vec, online, warp, splitk) and `VARIANTS_INT8` (warp_int8, splitk_int8). Underneath,
every name runs this library's sm_100a kernels through the C ABI (include/pa_b200.h):

  naive / vec / online / warp  -> pa_decode_f16  (single pass, fused split combine)
  splitk                       -> pa_splitk_f16  (512-token partitions + LSE reduce kernel)
  warp_int8                    -> pa_decode_i8
  splitk_int8                  -> pa_splitk_i8

The reference's four FP16 single-pass names are optimisation stages of one op; they share
one kernel here. The quantize-into-cache write has no reference op (the reference quantises
in torch); it is exported as `quantize_into_cache` in the style of the decode ops.
"""

from . import ops as _ops

# Reference op names per variant (tests/cuda_ext.py:38-49), kept for callers that print them.
_OPT_OPS = {
    "vec": "paged_decode_attn_vec",
    "online": "paged_decode_attn_online",
    "warp": "paged_decode_attn_warp",
    "splitk": "paged_decode_attn_splitk",
}
_OPT_OPS_INT8 = {
    "warp_int8": "paged_decode_attn_warp_int8",
    "splitk_int8": "paged_decode_attn_splitk_int8",
}


def paged_decode_attention(out, q, k_cache, v_cache, block_table, context_lens, scale,
                           block_size=16):
    _ops.decode(out, q, k_cache, v_cache, block_table, context_lens, scale, block_size,
                kv_kind="f16")
    return out


def _make_variant(op_name, splitk):
    def run(out, q, k_cache, v_cache, block_table, context_lens, scale, block_size=16):
        _ops.decode(out, q, k_cache, v_cache, block_table, context_lens, scale, block_size,
                    splitk=splitk, kv_kind="f16")
        return out
    run.__name__ = op_name
    return run


def _make_variant_int8(op_name, splitk):
    def run(out, q, k_cache, v_cache, k_scales, v_scales, block_table, context_lens, scale,
            block_size=16):
        _ops.decode(out, q, k_cache, v_cache, block_table, context_lens, scale, block_size,
                    k_scales=k_scales, v_scales=v_scales, splitk=splitk, kv_kind="i8")
        return out
    run.__name__ = op_name
    return run


VARIANTS = {"naive": paged_decode_attention}
VARIANTS.update({name: _make_variant(op, name == "splitk") for name, op in _OPT_OPS.items()})

VARIANTS_INT8 = {name: _make_variant_int8(op, name == "splitk_int8")
                 for name, op in _OPT_OPS_INT8.items()}


def quantize_into_cache(key, value, k_cache, v_cache, k_scales, v_scales, slot_mapping,
                        block_size=16):
    """Per-token INT8 quantize-into-cache (bit-exact with quantize_per_token)."""
    _ops.quantize_into_cache(key, value, k_cache, v_cache, k_scales, v_scales, slot_mapping,
                             block_size)
