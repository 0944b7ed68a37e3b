"""Row-sharded KNN over several GPUs: one process per GPU, each holding a contiguous
slice of the rows, a local top-k per query, an all-gather of the k (score, id) pairs,
and a merge.

This is the B200 counterpart of the reference's intra-process shard bus
(src/common/lock_free.mojo:104-200) and its merge (src/commands/vector.mojo:4394-4436:
concatenate up to k per shard, keep the best k), over NCCL instead of shared memory.
Ids are global (each shard registers its rows with id_base = its first row), and the
merge orders by (score, id), so the result equals the single-index result.

A shard's k results per query travel as interleaved 8-byte (f32 score, i32 id) pairs,
so one all-gather of B * k * 8 bytes per rank carries them (not one per array).
"""
from __future__ import annotations

from typing import Callable, Tuple


def shard_bounds(n_rows: int, world: int, rank: int) -> Tuple[int, int]:
    """Rows [lo, hi) held by `rank` of `world` equal contiguous shards."""
    return n_rows * rank // world, n_rows * (rank + 1) // world


def pack_pairs(ids, scores):
    """ids int32 [B, k] and scores float32 [B, k] -> int32 [B, k, 2]: per entry the
    score's bits, then the id (the 8-byte pair layout of PION_B200_MERGE_PAIRS)."""
    import torch
    return torch.stack((scores.contiguous().view(torch.int32), ids.contiguous()), dim=-1)


def unpack_pairs(pairs):
    """int32 [..., k, 2] pairs -> (ids int32 [..., k], scores float32 [..., k])."""
    import torch
    return pairs[..., 1].contiguous(), pairs[..., 0].contiguous().view(torch.float32)


class ShardedSearch:
    """One step of a row-sharded search.

    local_search(inputs) -> (ids int32 [B, k], scores float32 [B, k]) for this shard,
    global ids, ordered.  merge(pairs int32 [W, B, k, 2]) -> (ids, scores): the k best
    per query of the gathered (score, id) pairs (on the GPU: pion_b200.merge_topk_pairs
    with lists_major=True).  `group` is a torch.distributed process group (None: default).
    """

    def __init__(self, local_search: Callable, k: int, merge: Callable, group=None,
                 local_pairs: Callable | None = None):
        import torch.distributed as dist

        self.local_search = local_search
        self.local_pairs = local_pairs  # inputs -> int32 [B, k, 2] pairs, written directly
        self.k = k
        self.merge = merge
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1

    def _pairs(self, inputs):
        if self.local_pairs is not None:
            return self.local_pairs(inputs)
        return pack_pairs(*self.local_search(inputs))

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
        if self.world == 1:
            return self.local_search(inputs)
        return self.merge(self._gather(self._pairs(inputs)))

    def breakdown(self, inputs, steps: int):
        """Average device milliseconds per step of each phase -- local scoring and top-k
        (as pairs), all-gather, merge -- over `steps` steps timed with CUDA events on the
        current stream (GPU tensors only)."""
        import torch

        st = torch.cuda.current_stream()
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]
        for e in ev:
            e[0].record(st)
            if self.world > 1:
                pairs = self._pairs(inputs)
                e[1].record(st)
                g = self._gather(pairs)
                e[2].record(st)
                self.merge(g)
            else:
                self.local_search(inputs)
                e[1].record(st)
                e[2].record(st)
            e[3].record(st)
        torch.cuda.synchronize()
        parts = [0.0, 0.0, 0.0]
        for e in ev:
            for j in range(3):
                parts[j] += e[j].elapsed_time(e[j + 1])
        n = max(1, steps)
        return {"local_ms": parts[0] / n, "allgather_ms": parts[1] / n, "merge_ms": parts[2] / n}


class PeerExchange:
    """The library's NVLink peer-memory shard exchange (pion_v_b200_exchange_*): every rank
    creates it on its own GPU, the ranks swap its IPC handles over `group` (any
    torch.distributed backend), and each rank maps the others' receive buffers.  After
    that no collective call is needed per step: pion_v_b200_flat_i8_knn_sharded and
    pion_v_b200_exchange_merge move the pairs with peer stores and bounded flag waits."""

    def __init__(self, ctx, max_nq: int, k: int, regions: int = 2, group=None):
        import ctypes

        import torch
        import torch.distributed as dist

        from . import _lib
        self.ctx = ctx
        self.k = k
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        h = ctypes.c_void_p()
        ctx.check(ctx.lib.pion_v_b200_exchange_create(ctx.h, self.world, self.rank, regions,
                                                      max_nq, k, ctypes.byref(h)))
        self.h = h
        mine = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES)()
        ctx.check(ctx.lib.pion_v_b200_exchange_handle(self.h, mine))
        t = torch.tensor(list(mine), dtype=torch.uint8)
        if self.world > 1:
            backend = dist.get_backend(group)
            dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else None
            t = t.to(dev) if dev is not None else t
            out = torch.empty(self.world * _lib.IPC_HANDLE_BYTES, dtype=torch.uint8,
                              device=t.device)
            dist.all_gather_into_tensor(out, t, group=group)
            allh = bytes(out.cpu().tolist())
        else:
            allh = bytes(mine)
        buf = (ctypes.c_uint8 * len(allh)).from_buffer_copy(allh)
        ctx.check(ctx.lib.pion_v_b200_exchange_connect(self.h, buf))
        self.epoch = 0

    def next_epoch(self) -> int:
        self.epoch += 1
        return self.epoch

    def close(self):
        if getattr(self, "h", None):
            self.ctx.lib.pion_v_b200_exchange_free(self.h)
            self.h = None


class PeerShardedSearch:
    """One step of the row-sharded FLAT INT8 search through PeerExchange: the threshold
    sample shared by all ranks, every shard scored, the shard lists exchanged and merged
    (pion_v_b200_flat_i8_knn_sharded).  index: this rank's FlatI8Index (id_base = its first
    row); inputs: [q int8 [B, dim], q_scale float32 [B]] CUDA tensors.  local_bound: each
    rank starts from its own sample share's bound (one exchange per step instead of two)."""

    def __init__(self, index, ex: PeerExchange, local_bound: bool = False):
        from . import _lib
        self.ix = index
        self.ex = ex
        self.world = ex.world
        self.flags = _lib.OUT_PAIRS | (_lib.SHARD_LOCAL_BOUND if local_bound else 0)

    def __call__(self, inputs):
        import torch

        from . import _lib
        from .search import _TorchStream
        q, qs = inputs
        ctx = self.ix.ctx
        nq, k = q.shape[0], self.ex.k
        out = torch.empty((nq, k, 2), dtype=torch.int32, device=q.device)
        with _TorchStream(ctx, _lib.MEM_DEVICE):
            ctx.check(ctx.lib.pion_v_b200_flat_i8_knn_sharded(
                ctx.h, self.ix.h, self.ex.h, q.data_ptr(), qs.data_ptr(), nq, k,
                self.ex.next_epoch(), self.flags, None, out.data_ptr()))
        return unpack_pairs(out)
