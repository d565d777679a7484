"""pa_b200: B200-native (sm_100a) paged-attention decode with FP16 and per-token INT8 KV.

Public surface:
  pa_b200.cuda_ext     drop-in for the reference op registry (VARIANTS, VARIANTS_INT8, ...)
  pa_b200.ops          torch wrappers of the C ABI (decode, cache writes, partial merge)
  pa_b200.paged_cache  PagedKVCache with the reference bridge's interface, written by kernels
  pa_b200.shard        multi-GPU sharding by sequence / kv-head and cross-GPU split-K
"""

__version__ = "0.1.0"
