"""Row-sharded KNN over several GPUs: one process per GPU, each holding a contiguous
slice of the rows, a local top-k per query, an all-gather of the k (score, id) pairs,
and a merge.

This is the B200 counterpart of the reference's intra-process shard bus
(src/common/lock_free.mojo:104-200) and its merge (src/commands/vector.mojo:4394-4436:
concatenate up to k per shard, keep the best k), over NCCL instead of shared memory.
Ids are global (each shard registers its rows with id_base = its first row), and the
merge orders by (score, id), so the result equals the single-index result.
"""
from __future__ import annotations

from typing import Callable, Tuple


def shard_bounds(n_rows: int, world: int, rank: int) -> Tuple[int, int]:
    """Rows [lo, hi) held by `rank` of `world` equal contiguous shards."""
    return n_rows * rank // world, n_rows * (rank + 1) // world


class ShardedSearch:
    """One step of a row-sharded search.

    local_search(inputs) -> (ids int32 [B, k], scores float32 [B, k]) for this shard,
    global ids, ordered.  merge(scores [W, B, k], ids [W, B, k]) -> (ids, scores): the
    k best per query of the gathered lists (on the GPU: pion_b200.merge_topk with
    lists_major=True).  `group` is a torch.distributed process group (None: default).
    """

    def __init__(self, local_search: Callable, k: int, merge: Callable, group=None):
        import torch.distributed as dist

        self.local_search = local_search
        self.k = k
        self.merge = merge
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self._bufs = None

    def _gather(self, t):
        import torch
        import torch.distributed as dist

        out = torch.empty((self.world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        if t.is_cuda:
            dist.all_gather_into_tensor(out, t.contiguous(), group=self.group)
        else:  # gloo: list form
            parts = list(out.unbind(0))
            dist.all_gather(parts, t.contiguous(), group=self.group)
        return out

    def __call__(self, inputs):
        ids, scores = self.local_search(inputs)
        if self.world == 1:
            return ids, scores
        return self.merge(self._gather(scores), self._gather(ids))
