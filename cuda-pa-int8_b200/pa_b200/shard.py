"""Multi-GPU sharding of the decode path: one process per GPU, torch.distributed for plumbing.

Decode shards with no data exchange in two ways:
  * by sequence (lpt_partition): each rank owns a subset of the sequences and their blocks,
    balanced by context length with the longest-processing-time rule;
  * by kv-head (kv_head_slice): each rank holds num_kv_heads/world kv heads of every page and
    computes the q heads of those groups.
Only when one sequence's context is split across GPUs is there an exchange: each rank
computes un-normalised partials (O, m, l) for its token range (ops.decode_partial), the
partials are all-gathered over NCCL (a few hundred KB), and every rank merges them with the
log-sum-exp rule (ops.merge_partials). No kernel reads another GPU's memory: remote data
arrives through NCCL.
"""

import heapq


def lpt_partition(lengths, world):
    """Indices of `lengths` per rank, longest first onto the least-loaded rank; each rank's
    list is returned sorted. Ties break toward the lower rank, so the result is
    deterministic."""
    heap = [(0, r) for r in range(world)]
    parts = [[] for _ in range(world)]
    order = sorted(range(len(lengths)), key=lambda i: (-lengths[i], i))
    for i in order:
        load, r = heapq.heappop(heap)
        parts[r].append(i)
        heapq.heappush(heap, (load + lengths[i], r))
    return [sorted(p) for p in parts]


def kv_head_slice(num_heads, num_kv_heads, world, rank):
    """(q head range, kv head range) owned by `rank` when sharding by kv head."""
    if num_kv_heads % world != 0:
        raise ValueError(f"num_kv_heads {num_kv_heads} not divisible by world size {world}")
    per = num_kv_heads // world
    g = num_heads // num_kv_heads
    return (range(rank * per * g, (rank + 1) * per * g), range(rank * per, (rank + 1) * per))


def token_ranges(context_len, world, block_size=16):
    """Block-aligned [lo, hi) token ranges of one sequence, one per rank (possibly empty)."""
    nblk = (int(context_len) + block_size - 1) // block_size
    out = []
    for r in range(world):
        lo = (nblk * r) // world
        hi = (nblk * (r + 1)) // world
        out.append((min(lo * block_size, context_len), min(hi * block_size, context_len)))
    return out


def local_view(block_table_row, context_len, world, rank, block_size=16):
    """This rank's (block ids, context length) for its token range of one sequence."""
    lo, hi = token_ranges(context_len, world, block_size)[rank]
    b0 = lo // block_size
    nb = (hi - lo + block_size - 1) // block_size
    return list(block_table_row[b0:b0 + nb]), hi - lo


class SplitContextDecode:
    """Decode where each rank holds a block-aligned token range of every sequence.

    step(out, q, ...) runs the local partial decode, all-gathers the partials over the
    process group and merges them; every rank ends with the full output. The collective is
    the only cross-GPU traffic: num_seqs * num_kv_heads * slot floats per rank.

    partial_fn and merge_fn default to the CUDA ops (ops.decode_partial, ops.merge_partials);
    they take the same arguments as those, so the exchange itself can be driven with other
    implementations of the two steps (the CPU tests pass the oracle's).
    """

    def __init__(self, group=None, partial_fn=None, merge_fn=None):
        import torch.distributed as dist
        # Without an initialised process group the step runs on one rank: the gather is a copy.
        self.dist = dist if (dist.is_available() and dist.is_initialized()) else None
        self.group = group
        self.world = self.dist.get_world_size(group) if self.dist else 1
        if partial_fn is None or merge_fn is None:
            from . import ops
            partial_fn = partial_fn or ops.decode_partial
            merge_fn = merge_fn or ops.merge_partials
        self.partial_fn = partial_fn
        self.merge_fn = merge_fn
        self._gathered = None

    def gather_buffer(self, part):
        """The [world * num_seqs, per_seq] receive buffer for partials shaped like `part`,
        kept between steps (so a captured step keeps its address)."""
        import torch
        shape = (self.world * part.shape[0],) + tuple(part.shape[1:])
        g = self._gathered
        if g is None or tuple(g.shape) != shape or g.device != part.device:
            g = torch.empty(shape, dtype=part.dtype, device=part.device)
            self._gathered = g
        return g

    def step(self, out, q, k_cache, v_cache, block_table, context_lens, scale, block_size=16,
             k_scales=None, v_scales=None):
        part = self.partial_fn(q, k_cache, v_cache, block_table, context_lens, scale,
                               block_size, k_scales=k_scales, v_scales=v_scales)
        # Gathered along dim 0 ([world * num_seqs, per]: the layout every backend accepts),
        # then viewed as [world, num_seqs, per] for the merge.
        gathered = self.gather_buffer(part)
        if self.dist is not None:
            self.dist.all_gather_into_tensor(gathered, part, group=self.group)
        else:
            gathered.copy_(part)
        self.merge_fn(out, gathered.view((self.world,) + tuple(part.shape)), q.shape[1],
                      k_cache.shape[1])
        return out
