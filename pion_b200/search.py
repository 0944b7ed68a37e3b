"""Python host API over libpion_vector_b200 — the FT.SEARCH KNN operators.

Mirrors the operator surface of Pion's vector path (pavelhorak/pion):

* ``pkm_quantize_rows_i8`` / ``pkm_scores_i8`` / ``pkm_topk_max`` /
  ``pkm_sort_desc`` / ``pkm_combine_topk`` / ``pkm_scores_f32`` /
  ``pkm_rescore_f32`` — same names and argument meaning as
  src/vector/pkm_kernels.mojo:88-266 (the C symbols the engine binds);
* ``FlatI8Index.search`` — batched FLAT INT8 inner-product KNN
  (ref_pkm_scores_i8 + ref_pkm_topk_max per query);
* ``FlatF32Index.search`` — batched ``exact_knn`` under COSINE
  (src/commands/vector.mojo:1228-1365);
* ``BQIndex.search`` — sign-bit Hamming shortlist + exact cosine rerank;
* ``HNSWGraph`` — the reference's FT.OPTIMIZE graph build on the host CPU
  (src/vector/hnsw.mojo:2540-2620) into its compact level-0 layout;
* ``HNSWIndex.search`` — batched ``search_fp32_scored`` at dim 1536: upper-level
  greedy descent, then ``beam_search_1536_ref`` per query on the GPU;
  ``metric_scores`` — the reply scores (src/vector/hnsw.mojo:4523-4651);
  ``slot_scan_topk`` / ``brute_force`` — the GPU brute-force scan of the slot buffer
  (pion_metal_search_topk_w, search_gpu_brute_force).

Arrays may be numpy (host memory: the call copies to and from the GPU) or CUDA
torch tensors (device memory: used in place on the context's stream).  Errors
raise ``PionError`` with the library's message; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import _lib
from ._lib import MEM_DEVICE, MEM_DEVICE_BORROW, MEM_HOST, PionError

try:  # torch is plumbing for device memory and streams; optional for host-only use
    import torch
except Exception:  # pragma: no cover
    torch = None


def _is_torch(x) -> bool:
    return torch is not None and isinstance(x, torch.Tensor)


def _ptr(x, dtype_np, name: str):
    """(pointer, mem kind, keep-alive object) for a numpy array or torch tensor."""
    if _is_torch(x):
        if not x.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
        want = {np.int8: torch.int8, np.float32: torch.float32, np.int32: torch.int32,
                np.uint64: torch.uint64 if hasattr(torch, "uint64") else torch.int64}[dtype_np]
        if x.dtype != want:
            raise TypeError(f"{name} must be {want}, got {x.dtype}")
        return x.data_ptr(), (MEM_DEVICE if x.is_cuda else MEM_HOST), x
    a = np.ascontiguousarray(x, dtype=dtype_np)
    return a.ctypes.data, MEM_HOST, a


def _torch_stream() -> int:
    """torch's current stream as a cudaStream_t; its legacy default stream has handle 0,
    which the C API reads as "the context's own stream", so it is passed as
    cudaStreamLegacy (0x1) instead."""
    return torch.cuda.current_stream().cuda_stream or 1


class _TorchStream:
    """For device-memory calls: run the library on torch's current CUDA stream so
    that tensors torch produced (or will consume) are ordered with our kernels."""

    def __init__(self, ctx, mem):
        self.ctx = ctx
        self.active = mem in (MEM_DEVICE, MEM_DEVICE_BORROW) and torch is not None

    def __enter__(self):
        if self.active:
            self.ctx.lib.pion_v_b200_set_stream(self.ctx.h, ctypes.c_void_p(_torch_stream()))
        return self

    def __exit__(self, *exc):
        if self.active:
            self.ctx.lib.pion_v_b200_set_stream(self.ctx.h, ctypes.c_void_p(self.ctx._stream))


def _same_mem(*mems):
    m = set(mems)
    if len(m) != 1:
        raise ValueError("all arrays of one call must live in the same memory (host or device)")
    return m.pop()


class Context:
    """One worker's CUDA stream, scratch buffers and error slot (pion_v_b200_init)."""

    def __init__(self, device: int = -1, worker_id: int = 0):
        self.lib = _lib.load()
        h = ctypes.c_void_p()
        rc = self.lib.pion_v_b200_init(device, worker_id, ctypes.byref(h))
        if rc != 0:
            raise PionError(rc, f"pion_v_b200_init(device={device}) failed")
        self.h = h
        self.device = device
        self._stream = 0  # 0: the context's own stream

    def check(self, rc: int):
        if rc != 0:
            msg = self.lib.pion_v_b200_last_error(self.h)
            raise PionError(rc, msg.decode() if msg else "")

    def use_stream(self, stream_handle: int | None):
        self._stream = stream_handle or 0
        self.check(self.lib.pion_v_b200_set_stream(self.h, ctypes.c_void_p(self._stream)))

    def use_torch_stream(self):
        """Run on torch's current CUDA stream (so torch ops and ours are ordered)."""
        self.use_stream(_torch_stream())

    def sync(self):
        self.check(self.lib.pion_v_b200_sync(self.h))

    def set_wait_budget(self, ns: int):
        """Budget of each device-side wait of the FLAT INT8 kernels (ns; <= 0: 2 s)."""
        self.check(self.lib.pion_v_b200_set_wait_budget(self.h, int(ns)))

    def reserve(self, max_nq: int, max_k: int):
        self.check(self.lib.pion_v_b200_reserve(self.h, max_nq, max_k))

    @property
    def launches(self) -> int:
        return int(self.lib.pion_v_b200_launch_count(self.h))

    def timing(self, enable: bool):
        """Record CUDA events around every scoring-kernel launch (benchmarks)."""
        self.check(self.lib.pion_v_b200_timing_enable(self.h, int(enable)))

    def timing_read(self, tag: int = 0):
        """(total ms, count) of the event pairs recorded since timing(True) for one phase:
        0 every scoring kernel of a call, 1 the FLAT INT8 threshold pass, 2 its main pass."""
        ms = ctypes.c_double()
        n = ctypes.c_int64()
        self.check(self.lib.pion_v_b200_timing_read_tag(self.h, int(tag), ctypes.byref(ms),
                                                        ctypes.byref(n)))
        return ms.value, n.value

    def close(self):
        if getattr(self, "h", None):
            self.lib.pion_v_b200_shutdown(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass


def _outputs(like_device: bool, nq: int, k: int, device=None):
    if like_device:
        ids = torch.empty((nq, k), dtype=torch.int32, device=device)
        sc = torch.empty((nq, k), dtype=torch.float32, device=device)
        return ids, sc, ids.data_ptr(), sc.data_ptr()
    ids = np.empty((nq, k), np.int32)
    sc = np.empty((nq, k), np.float32)
    return ids, sc, ids.ctypes.data, sc.ctypes.data


class _Index:
    def __init__(self, ctx: Context, handle: ctypes.c_void_p, keep=None):
        self.ctx = ctx
        self.h = handle
        self._keep = keep

    @property
    def n_rows(self) -> int:
        return int(self.ctx.lib.pion_v_b200_index_rows(self.h))

    def free(self):
        if getattr(self, "h", None):
            self.ctx.lib.pion_v_b200_index_free(self.h)
            self.h = None

    def __del__(self):  # pragma: no cover
        try:
            self.free()
        except Exception:
            pass


class FlatI8Index(_Index):
    """Device-resident FLAT INT8 index (rows int8[n, dim] + per-row fp32 scale)."""

    def __init__(self, ctx: Context, rows, row_scale, id_base: int = 0, borrow: bool = False):
        pr, mr, kr = _ptr(rows, np.int8, "rows")
        ps, ms, ks = _ptr(row_scale, np.float32, "row_scale")
        mem = _same_mem(mr, ms)
        if borrow:
            if mem != MEM_DEVICE:
                raise ValueError("borrow needs device tensors")
            mem = MEM_DEVICE_BORROW
        n, dim = (rows.shape[0], rows.shape[1])
        h = ctypes.c_void_p()
        with _TorchStream(ctx, mem):
            ctx.check(ctx.lib.pion_v_b200_register_flat_i8(ctx.h, pr, ps, n, dim, id_base, mem,
                                                           ctypes.byref(h)))
        super().__init__(ctx, h, (kr, ks) if borrow else None)
        self.dim = dim

    def search(self, q, q_scale, k: int):
        """Top-k by (score desc, id asc) per query -> (ids int32[nq,k], scores f32[nq,k])."""
        pq, mq, kq = _ptr(q, np.int8, "q")
        ps, ms, ks = _ptr(q_scale, np.float32, "q_scale")
        mem = _same_mem(mq, ms)
        nq = q.shape[0]
        ids, sc, pi, pv = _outputs(mem == MEM_DEVICE, nq, k,
                                   q.device if mem == MEM_DEVICE else None)
        with _TorchStream(self.ctx, mem):
            self.ctx.check(self.ctx.lib.pion_v_b200_flat_i8_knn(self.ctx.h, self.h, pq, ps, nq,
                                                                k, pi, pv, mem))
        return ids, sc


def _search_pairs_i8(ix, q, q_scale, k: int):
    """FlatI8Index.search into one int32 [nq, k, 2] CUDA tensor of (score bits, id)."""
    if not (_is_torch(q) and q.is_cuda):
        raise TypeError("search_pairs needs CUDA tensors")
    pq, mq, kq = _ptr(q, np.int8, "q")
    ps, ms, ks = _ptr(q_scale, np.float32, "q_scale")
    _same_mem(mq, ms)
    out = torch.empty((q.shape[0], k, 2), dtype=torch.int32, device=q.device)
    with _TorchStream(ix.ctx, MEM_DEVICE):
        ix.ctx.check(ix.ctx.lib.pion_v_b200_flat_i8_knn(ix.ctx.h, ix.h, pq, ps, q.shape[0], k,
                                                        None, out.data_ptr(),
                                                        MEM_DEVICE | _lib.OUT_PAIRS))
    return out


FlatI8Index.search_pairs = _search_pairs_i8
FlatI8Index.search_pairs.__doc__ = (
    "Top-k as interleaved (score, id) pairs, int32 [nq, k, 2] on the GPU: the layout one "
    "row shard all-gathers (pion_b200.sharded), written by the search's final merge.")


class FlatF32Index(_Index):
    """Device-resident FLAT FP32 index for COSINE exact_knn."""

    def __init__(self, ctx: Context, rows, id_base: int = 0, normalize: bool = True,
                 borrow: bool = False):
        pr, mem, kr = _ptr(rows, np.float32, "rows")
        if borrow:
            if mem != MEM_DEVICE or normalize:
                raise ValueError("borrow needs device tensors that are already normalised")
            mem = MEM_DEVICE_BORROW
        h = ctypes.c_void_p()
        with _TorchStream(ctx, mem):
            ctx.check(ctx.lib.pion_v_b200_register_flat_f32(ctx.h, pr, rows.shape[0],
                                                            rows.shape[1], id_base,
                                                            int(normalize), mem,
                                                            ctypes.byref(h)))
        super().__init__(ctx, h, kr if borrow else None)
        self.dim = rows.shape[1]

    def search(self, q, k: int):
        """k smallest `1 - cos` by (score asc, id asc) -> (ids, scores)."""
        pq, mem, kq = _ptr(q, np.float32, "q")
        nq = q.shape[0]
        ids, sc, pi, pv = _outputs(mem == MEM_DEVICE, nq, k,
                                   q.device if mem == MEM_DEVICE else None)
        with _TorchStream(self.ctx, mem):
            self.ctx.check(self.ctx.lib.pion_v_b200_flat_f32_knn(self.ctx.h, self.h, pq, nq, k,
                                                                 pi, pv, mem))
        return ids, sc

    def merge_delta(self, q, built: int, ids, scores, k: int, cosine: bool = True,
                    ctx: Context | None = None):
        """merge_delta (src/commands/vector.mojo:1368-1456) with this index as the FP32
        ingest rows: ids / scores [nq, kg] (the graph's results, -1 ends a list) are
        rescored in place; returns the merge with the exact scan of rows [built, n)
        as (ids int32 [nq, k], scores float32 [nq, k])."""
        c = ctx or self.ctx
        pq, mq, kq = _ptr(q, np.float32, "q")
        if _is_torch(ids):
            pi, mi = ids.data_ptr(), MEM_DEVICE if ids.is_cuda else MEM_HOST
            ps, ms = scores.data_ptr(), MEM_DEVICE if scores.is_cuda else MEM_HOST
        else:
            for a, nm, dt in ((ids, "ids", np.int32), (scores, "scores", np.float32)):
                if not (isinstance(a, np.ndarray) and a.dtype == dt and a.flags["C_CONTIGUOUS"]):
                    raise TypeError(f"{nm} must be a contiguous {np.dtype(dt)} array "
                                    "(updated in place)")
            pi, mi, ps, ms = ids.ctypes.data, MEM_HOST, scores.ctypes.data, MEM_HOST
        m = _same_mem(mq, mi, ms)
        nq, kg = ids.shape
        oi, osc, poi, pos = _outputs(m == MEM_DEVICE, nq, k, q.device if m == MEM_DEVICE else None)
        with _TorchStream(c, m):
            c.check(c.lib.pion_v_b200_merge_delta(c.h, self.h, built, 1 if cosine else 0, pq, nq,
                                                   kg, pi, ps, k, poi, pos, m))
        return oi, osc


class BQIndex(_Index):
    """Sign-bit codes + fp32 rows: Hamming shortlist, exact cosine rerank."""

    def __init__(self, ctx: Context, rows, id_base: int = 0, normalize: bool = True):
        pr, mem, kr = _ptr(rows, np.float32, "rows")
        h = ctypes.c_void_p()
        with _TorchStream(ctx, mem):
            ctx.check(ctx.lib.pion_v_b200_register_bq(ctx.h, pr, rows.shape[0], rows.shape[1],
                                                      id_base, int(normalize), mem,
                                                      ctypes.byref(h)))
        super().__init__(ctx, h)
        self.dim = rows.shape[1]

    def search(self, q, k: int, shortlist: int = 100):
        pq, mem, kq = _ptr(q, np.float32, "q")
        nq = q.shape[0]
        ids, sc, pi, pv = _outputs(mem == MEM_DEVICE, nq, k,
                                   q.device if mem == MEM_DEVICE else None)
        with _TorchStream(self.ctx, mem):
            self.ctx.check(self.ctx.lib.pion_v_b200_bq_rerank_knn(self.ctx.h, self.h, pq, nq,
                                                                  shortlist, k, pi, pv, mem))
        return ids, sc


# --------------------------------------------------------------- functions --

def quantize_rows_i8(ctx: Context, src, d: int | None = None):
    """pkm_quantize_rows_i8 on the GPU (src/vector/pkm_kernels.mojo:152-191)."""
    ps, mem, ks = _ptr(src, np.float32, "src")
    n, d_pad = src.shape
    d = d_pad if d is None else d
    if mem == MEM_DEVICE:
        out = torch.empty((n, d_pad), dtype=torch.int8, device=src.device)
        sc = torch.empty(n, dtype=torch.float32, device=src.device)
        po, psc = out.data_ptr(), sc.data_ptr()
    else:
        out = np.empty((n, d_pad), np.int8)
        sc = np.empty(n, np.float32)
        po, psc = out.ctypes.data, sc.ctypes.data
    with _TorchStream(ctx, mem):
        ctx.check(ctx.lib.pion_v_b200_quantize_rows_i8(ctx.h, ps, n, d, d_pad, po, psc, mem))
    return out, sc


def l2_normalize_rows(ctx: Context, src):
    """l2_normalize_fp32 of every row on the GPU (src/vector/kernels.mojo:318-357)."""
    ps, mem, ks = _ptr(src, np.float32, "src")
    n, dim = src.shape
    if mem == MEM_DEVICE:
        out = torch.empty_like(src)
        po = out.data_ptr()
    else:
        out = np.empty((n, dim), np.float32)
        po = out.ctypes.data
    with _TorchStream(ctx, mem):
        ctx.check(ctx.lib.pion_v_b200_l2_normalize_rows(ctx.h, ps, n, dim, po, mem))
    return out


def merge_topk(ctx: Context, cand_scores, cand_ids, k: int, descending: bool = True,
               lists_major: bool = False):
    """Merge sorted candidate lists into the k best per query: input [nq, n_lists, k],
    or [n_lists, nq, k] with lists_major (an all-gather of per-shard results)."""
    pv, mv, kv = _ptr(cand_scores, np.float32, "cand_scores")
    pi, mi, ki = _ptr(cand_ids, np.int32, "cand_ids")
    mem = _same_mem(mv, mi)
    if lists_major:
        n_lists, nq, kk = cand_scores.shape
    else:
        nq, n_lists, kk = cand_scores.shape
    if kk != k:
        raise ValueError("candidate lists must hold exactly k entries")
    ids, sc, po_i, po_v = _outputs(mem == MEM_DEVICE, nq, k,
                                   cand_scores.device if mem == MEM_DEVICE else None)
    with _TorchStream(ctx, mem):
        flags = (_lib.MERGE_DESC if descending else 0) | (_lib.MERGE_LISTS_MAJOR if lists_major
                                                           else 0)
        ctx.check(ctx.lib.pion_v_b200_merge_topk(ctx.h, pv, pi, nq, n_lists, k, flags, po_v,
                                                 po_i, mem))
    return ids, sc


def merge_topk_pairs(ctx: Context, pairs, k: int, descending: bool = True,
                     lists_major: bool = True):
    """merge_topk over interleaved (f32 score, i32 id) pairs: `pairs` int32 [n_lists, nq,
    k, 2] (lists_major, the all-gather of pion_b200.sharded.pack_pairs) or [nq, n_lists,
    k, 2]; numpy (host) or a CUDA tensor.  Returns (ids [nq, k], scores [nq, k])."""
    if _is_torch(pairs):
        if not pairs.is_contiguous() or pairs.dtype != torch.int32:
            raise TypeError("pairs must be a contiguous int32 tensor")
        p, mem = pairs.data_ptr(), (MEM_DEVICE if pairs.is_cuda else MEM_HOST)
        keep = pairs
    else:
        keep = np.ascontiguousarray(pairs, dtype=np.int32)
        p, mem = keep.ctypes.data, MEM_HOST
    if keep.ndim != 4 or keep.shape[-1] != 2:
        raise ValueError("pairs must have shape [lists, nq, k, 2] or [nq, lists, k, 2]")
    if lists_major:
        n_lists, nq, kk = keep.shape[:3]
    else:
        nq, n_lists, kk = keep.shape[:3]
    if kk != k:
        raise ValueError("candidate lists must hold exactly k entries")
    ids, sc, po_i, po_v = _outputs(mem == MEM_DEVICE, nq, k,
                                   pairs.device if mem == MEM_DEVICE else None)
    with _TorchStream(ctx, mem):
        flags = ((_lib.MERGE_DESC if descending else 0) |
                 (_lib.MERGE_LISTS_MAJOR if lists_major else 0) | _lib.MERGE_PAIRS)
        ctx.check(ctx.lib.pion_v_b200_merge_topk(ctx.h, p, None, nq, n_lists, k, flags, po_v,
                                                 po_i, mem))
    return ids, sc


# -------------------------------------------------------------------- HNSW --

_LAYOUT_ARRAYS = {
    # name: (dtype, shape from (n, stride, M, upper_rows))
    "compact_buffer": (np.int8, lambda n, st, m, ur: (n, st)),
    "l0_compact": (np.uint32, lambda n, st, m, ur: (n, 33)),
    "l0_slots": (np.uint32, lambda n, st, m, ur: (n, 33)),
    "node_slot": (np.uint32, lambda n, st, m, ur: (n,)),
    "node_ids": (np.int32, lambda n, st, m, ur: (n,)),
    "node_level": (np.int8, lambda n, st, m, ur: (n,)),
    "upper_offset": (np.int64, lambda n, st, m, ur: (n,)),
    "upper_links": (np.uint32, lambda n, st, m, ur: (ur, 1 + m)),
}
_LAYOUT_SCALARS = ("num_nodes", "dim", "M", "entry_point", "max_level", "global_min",
                   "global_max", "metric", "compact_stride", "compact_hdr", "upper_rows")


def hnsw_layout_struct(arrays: dict):
    """(pion_b200_hnsw_layout, keep-alive list) from a dict of numpy arrays and scalars
    (the keys of HNSWGraph.arrays(); "deleted" optional)."""
    lay = _lib.HnswLayout()
    keep = []
    for name in _LAYOUT_SCALARS:
        setattr(lay, name, arrays[name])
    for name, (dt, _) in _LAYOUT_ARRAYS.items():
        a = np.ascontiguousarray(arrays[name], dtype=dt)
        keep.append(a)
        setattr(lay, name, a.ctypes.data if a.size else None)
    dele = arrays.get("deleted")
    if dele is not None:
        d = np.ascontiguousarray(dele, dtype=np.uint8)
        keep.append(d)
        lay.deleted = d.ctypes.data
    return lay, keep


class HNSWGraph:
    """An HNSW INT8 graph built on the host CPU as the reference's FT.OPTIMIZE builds
    it (calibrate, quantize, parallel link lanes, relink and level-0 repair, compact),
    held by the library in the compact level-0 layout.

    rows: float32 [n, dim] host array.  metric: "cosine" (rows and queries are
    unit-normalised) or "l2".  threads <= 0 uses every online CPU; one thread builds
    the same graph every time.  batch > 0: batched insertion of up to `batch` nodes at a
    time (the same graph for any thread count; batch = 1 is the one-lane build)."""

    def __init__(self, rows, M: int = 16, ef_construction: int = 200, metric: str = "cosine",
                 id_base: int = 0, threads: int = 0, batch: int = 0, gpu: "Context" = None):
        """gpu: a Context whose device plans the batches (needs batch > 0); the graph is
        the one the host's batched build makes."""
        self.lib = _lib.load()
        a = np.ascontiguousarray(rows, dtype=np.float32)
        h = ctypes.c_void_p()
        mt = 1 if metric == "cosine" else 0
        if gpu is not None:
            if batch <= 0:
                raise ValueError("the GPU build is a batched build: give batch > 0")
            gpu.check(self.lib.pion_v_b200_hnsw_build_gpu(gpu.h, a.ctypes.data, a.shape[0],
                                                          a.shape[1], M, ef_construction, mt,
                                                          id_base, threads, batch,
                                                          ctypes.byref(h)))
            rc = 0
        elif batch > 0:  # batched insertion (deterministic for any thread count)
            rc = self.lib.pion_v_b200_hnsw_build_batched(a.ctypes.data, a.shape[0], a.shape[1],
                                                         M, ef_construction, mt, id_base,
                                                         threads, batch, ctypes.byref(h))
        else:
            rc = self.lib.pion_v_b200_hnsw_build(a.ctypes.data, a.shape[0], a.shape[1], M,
                                                 ef_construction, mt, id_base, threads,
                                                 ctypes.byref(h))
        if rc != 0:
            raise PionError(rc, "hnsw_build failed")
        self._adopt(h)

    def _adopt(self, h):
        self.h = h
        self.layout = _lib.HnswLayout()
        self.lib.pion_v_b200_hnsw_graph_layout(self.h, ctypes.byref(self.layout))

    @classmethod
    def load(cls, path: str) -> "HNSWGraph":
        """A graph from the reference's index file pion.hnsw.0 (format v3 to v5,
        HNSWGraph.load_from_disk, src/vector/hnsw.mojo:1485-1700)."""
        self = cls.__new__(cls)
        self.lib = _lib.load()
        h = ctypes.c_void_p()
        rc = self.lib.pion_v_b200_hnsw_load(os.fsencode(path), ctypes.byref(h))
        if rc != 0:
            raise PionError(rc, f"hnsw_load {path} failed")
        self._adopt(h)
        return self

    @classmethod
    def load_quant(cls, path: str):
        """A graph and its block-quantised slots from the reference's index file (compact
        format INT4 / INT3 / INT2 with the FP32 rerank and QJL sections it carries) ->
        (HNSWGraph, HNSWQuant); the HNSWQuant is None for a plain INT8 file."""
        self = cls.__new__(cls)
        self.lib = _lib.load()
        h, q = ctypes.c_void_p(), ctypes.c_void_p()
        rc = self.lib.pion_v_b200_hnsw_load_quant(os.fsencode(path), ctypes.byref(h),
                                                  ctypes.byref(q))
        if rc != 0:
            raise PionError(rc, f"hnsw_load_quant {path} failed")
        self._adopt(h)
        return self, (HNSWQuant._adopt(self.lib, q) if q.value else None)

    def save(self, path: str, max_elements: int = 0, quant=None):
        """Write the graph as the reference's index file (format v5, _save_body,
        src/vector/hnsw.mojo:1209-1440); max_elements: the engine's capacity.  With
        `quant` (an HNSWQuant of this graph) the file holds its block format and
        sections instead of INT8 slots."""
        if quant is not None:
            rc = self.lib.pion_v_b200_hnsw_save_quant(self.h, quant.h, os.fsencode(path),
                                                      max_elements)
        else:
            rc = self.lib.pion_v_b200_hnsw_save(self.h, os.fsencode(path), max_elements)
        if rc != 0:
            raise PionError(rc, f"hnsw_save {path} failed")

    def stats(self) -> dict:
        """lanes, link_drops, relinked, repaired_exits, repaired_links, gpu_planned (nodes
        whose insertion a GPU planned)."""
        out = (ctypes.c_int64 * 6)()
        self.lib.pion_v_b200_hnsw_graph_stats6(self.h, out)
        return dict(zip(("lanes", "link_drops", "relinked", "repaired_exits",
                         "repaired_links", "gpu_planned"), list(out)))

    def arrays(self) -> dict:
        """The layout as numpy views of the library's buffers (each view keeps the graph
        alive) plus its scalars."""
        L = self.layout
        n, st, m, ur = L.num_nodes, L.compact_stride, L.M, L.upper_rows
        out = {name: getattr(L, name) for name in _LAYOUT_SCALARS}
        ctype = {np.int8: ctypes.c_int8, np.uint32: ctypes.c_uint32, np.int32: ctypes.c_int32,
                 np.int64: ctypes.c_int64}
        for name, (dt, shape_of) in _LAYOUT_ARRAYS.items():
            shape = shape_of(n, st, m, ur)
            ptr = getattr(L, name)
            if not ptr or int(np.prod(shape)) == 0:
                out[name] = np.zeros(shape, dt)
                continue
            out[name] = _view(ptr, ctype[dt], shape, dt, self)
        out["deleted"] = None
        return out

    def free(self):
        if getattr(self, "h", None):
            self.lib.pion_v_b200_hnsw_graph_free(self.h)
            self.h = None

    def __del__(self):  # pragma: no cover
        try:
            self.free()
        except Exception:
            pass


class HNSWIndex(_Index):
    """An HNSW graph copied to the GPU: batched search_fp32_scored at dim 1536."""

    def __init__(self, ctx: Context, graph):
        if isinstance(graph, HNSWGraph):
            lay, keep = graph.layout, [graph]
        else:
            lay, keep = hnsw_layout_struct(graph)
        h = ctypes.c_void_p()
        ctx.check(ctx.lib.pion_v_b200_register_hnsw(ctx.h, ctypes.byref(lay), ctypes.byref(h)))
        super().__init__(ctx, h)
        self.dim = lay.dim

    def search(self, q, k: int, ef: int, ctx: Context | None = None):
        """q float32 [nq, 1536] -> (node ids int32 [nq, k], pool distances float32).
        `ctx`: another context on the same device (a registered graph is read-only and
        may serve every worker's context at once); default the registering one."""
        c = ctx or self.ctx
        pq, mem, kq = _ptr(q, np.float32, "q")
        nq = q.shape[0]
        ids, dist, pi, pv = _outputs(mem == MEM_DEVICE, nq, k,
                                     q.device if mem == MEM_DEVICE else None)
        with _TorchStream(c, mem):
            c.check(c.lib.pion_v_b200_hnsw_search(c.h, self.h, pq, nq, k, ef, pi, pv, mem))
        return ids, dist

    def metric_scores(self, q, ids, scores, ctx: Context | None = None):
        """metric_scores (src/vector/hnsw.mojo:4523-4651): the reply scores of `ids`
        (external ids, as search returns them) in the index metric (squared L2, or
        1 - cos under COSINE) from the INT8 codes; `scores` is updated in place and
        returned (entries whose id names no node keep their value)."""
        c = ctx or self.ctx
        pq, mem, kq = _ptr(q, np.float32, "q")
        pi, mi, ki = _ptr(ids, np.int32, "ids")
        if _is_torch(scores):
            ps, ms = scores.data_ptr(), MEM_DEVICE if scores.is_cuda else MEM_HOST
        else:
            if not (isinstance(scores, np.ndarray) and scores.dtype == np.float32 and
                    scores.flags["C_CONTIGUOUS"]):
                raise TypeError("scores must be a contiguous float32 array (updated in place)")
            ps, ms = scores.ctypes.data, MEM_HOST
        m = _same_mem(mem, mi, ms)
        nq, k = ids.shape
        with _TorchStream(c, m):
            c.check(c.lib.pion_v_b200_hnsw_metric_scores(c.h, self.h, pq, nq, k, pi, ps, m))
        return scores

    def beam_batch(self, q_codes, q_norm, pools, sizes, cursors=None,
                   ctx: Context | None = None):
        """The level-0 beam from caller-seeded pools for a batch (pion_v_beam_1536's
        contract): q_codes int8 [nq, 1536], q_norm float32 [nq], pools a structured or
        uint64 array [nq, ef] of (f32 dist, u32 node) entries and sizes int32 [nq], both
        updated in place; cursors int32 [nq] or None."""
        c = ctx or self.ctx
        pq, mq, kq = _ptr(q_codes, np.int8, "q_codes")
        pn, mn, kn = _ptr(q_norm, np.float32, "q_norm")
        if _is_torch(pools):
            pp, mp = pools.data_ptr(), MEM_DEVICE if pools.is_cuda else MEM_HOST
            ps, ms = sizes.data_ptr(), MEM_DEVICE if sizes.is_cuda else MEM_HOST
        else:
            for a, nm in ((pools, "pools"), (sizes, "sizes")):
                if not (isinstance(a, np.ndarray) and a.flags["C_CONTIGUOUS"]):
                    raise TypeError(f"{nm} must be a contiguous array (updated in place)")
            if pools.dtype.itemsize * (pools.shape[1] if pools.ndim > 1 else 1) % 8:
                raise TypeError("pools entries must be 8 bytes")
            if sizes.dtype != np.int32:
                raise TypeError("sizes must be int32")
            pp, mp = pools.ctypes.data, MEM_HOST
            ps, ms = sizes.ctypes.data, MEM_HOST
        pc, kc = None, None
        mems = [mq, mn, mp, ms]
        if cursors is not None:
            pc, mc, kc = _ptr(cursors, np.int32, "cursors")
            mems.append(mc)
        m = _same_mem(*mems)
        nq = q_codes.shape[0]
        ef = pools.shape[1] if (pools.ndim > 1 and pools.dtype.itemsize == 8) else \
            pools.nbytes // (8 * max(1, nq))
        with _TorchStream(c, m):
            c.check(c.lib.pion_v_b200_hnsw_beam_batch(c.h, self.h, pq, pn, nq, ef, pp, ps, pc,
                                                       m))
        return pools, sizes

    def slot_scan_topk(self, q_codes, k: int, q_norm=None, num_vectors: int | None = None,
                       ctx: Context | None = None):
        """The GPU brute-force slot scan (pion_metal_search_topk_w, src/ffi/metal_wrap.m:
        495-580) for a batch: int8 codes [nq, 1536] (and optionally their norms) ->
        (slots int32 [nq, k], INT8 L2 distances float32) in the order the worst-replace
        loop leaves them; -1 / +inf past min(k, num_vectors)."""
        c = ctx or self.ctx
        pq, mem, kq = _ptr(q_codes, np.int8, "q_codes")
        pn, kn = None, None
        if q_norm is not None:
            pn, mn, kn = _ptr(q_norm, np.float32, "q_norm")
            mem = _same_mem(mem, mn)
        nq = q_codes.shape[0]
        nv = self.n_rows if num_vectors is None else int(num_vectors)
        slots, dist, ps, pd = _outputs(mem == MEM_DEVICE, nq, k,
                                       q_codes.device if mem == MEM_DEVICE else None)
        with _TorchStream(c, mem):
            c.check(c.lib.pion_v_b200_slot_scan_topk(c.h, self.h, pq, pn, nq, nv, k, ps, pd,
                                                      mem))
        return slots, dist

    def slot_stats(self, ctx: Context | None = None) -> dict:
        """Work of the context's last slot scan or brute-force call: queries that took
        the exact CUDA-core scan, candidate slots replayed through the top-k loop."""
        c = ctx or self.ctx
        out = (ctypes.c_int64 * 2)()
        c.check(c.lib.pion_v_b200_slot_last_stats(c.h, out))
        return dict(zip(("exact_queries", "replayed"), list(out)))

    def set_rerank_rows(self, rows):
        """FP32 rows [slots, 1536] by slot for brute_force's rerank
        (pion_metal_register_rerank_buffer); None drops them."""
        if rows is None:
            self.ctx.check(self.ctx.lib.pion_v_b200_hnsw_set_rerank_rows(
                self.ctx.h, self.h, None, 0, 0, MEM_HOST))
            return
        pr, mem, kr = _ptr(rows, np.float32, "rows")
        with _TorchStream(self.ctx, mem):
            self.ctx.check(self.ctx.lib.pion_v_b200_hnsw_set_rerank_rows(
                self.ctx.h, self.h, pr, rows.shape[0], rows.shape[1], mem))

    def brute_force(self, q, k: int, ctx: Context | None = None):
        """search_gpu_brute_force (src/vector/hnsw.mojo:3916-3992) for a batch: q float32
        [nq, 1536] -> (external ids int32 [nq, k], scores float32 [nq, k], found int32
        [nq]); scores are INT8 L2 distances, or FP32 squared L2 with rerank rows."""
        c = ctx or self.ctx
        pq, mem, kq = _ptr(q, np.float32, "q")
        nq = q.shape[0]
        dev = mem == MEM_DEVICE
        ids, sc, pi, pv = _outputs(dev, nq, k, q.device if dev else None)
        if dev:
            found = torch.empty(nq, dtype=torch.int32, device=q.device)
            pf = found.data_ptr()
        else:
            found = np.empty(nq, np.int32)
            pf = found.ctypes.data
        with _TorchStream(c, mem):
            c.check(c.lib.pion_v_b200_hnsw_brute_force(c.h, self.h, pq, nq, k, pi, pv, pf, mem))
        return ids, sc, found

    def last_stats(self, ctx: Context | None = None) -> dict:
        """Work of the context's last search: level-0 evaluations, expansions, upper-level
        evaluations."""
        c = ctx or self.ctx
        out = (ctypes.c_int64 * 3)()
        c.check(c.lib.pion_v_b200_hnsw_last_stats(c.h, out))
        return dict(zip(("evals", "expansions", "upper_evals"), list(out)))


# ------------------------------------------------------ block-quantised HNSW --

QUANT_KINDS = {"polar": 0, "nano": 1, "turbo": 2}


def _view(ptr, ctype, shape, dtype, owner=None):
    """A numpy view of library memory that keeps `owner` (the object whose buffers these
    are) alive as long as the view lives."""
    count = int(np.prod(shape))
    if not ptr or count == 0:
        return np.zeros(shape, dtype)
    buf = (ctype * count).from_address(ptr)
    buf._owner = owner
    return np.frombuffer(buf, dtype).reshape(shape)


class HNSWQuant:
    """A graph's block-quantised slots in one of the reference's compact formats
    ("polar": PolarQuant INT4, "nano": NanoQuant INT2, "turbo": TurboQuant INT3 + QJL),
    quantised on the host from the rows the graph was built from (node order; normalised
    first under COSINE), with those rows kept as the FP32 rerank buffer."""

    def __init__(self, graph: HNSWGraph, rows, kind: str):
        if kind not in QUANT_KINDS:
            raise ValueError(f"kind must be one of {sorted(QUANT_KINDS)}")
        self.lib = _lib.load()
        a = np.ascontiguousarray(rows, dtype=np.float32)
        h = ctypes.c_void_p()
        rc = self.lib.pion_v_b200_hnsw_quantize(graph.h, a.ctypes.data, a.shape[0],
                                                QUANT_KINDS[kind], ctypes.byref(h))
        if rc != 0:
            raise PionError(rc, "hnsw_quantize failed")
        self.h = h
        self.kind = kind
        self.layout = _lib.HnswQuantLayout()
        self.lib.pion_v_b200_hnsw_quant_layout(self.h, ctypes.byref(self.layout))

    @classmethod
    def _adopt(cls, lib, h):
        self = cls.__new__(cls)
        self.lib, self.h = lib, h
        self.layout = _lib.HnswQuantLayout()
        lib.pion_v_b200_hnsw_quant_layout(h, ctypes.byref(self.layout))
        self.kind = {v: k for k, v in QUANT_KINDS.items()}[self.layout.kind]
        return self

    def arrays(self) -> dict:
        """numpy views of the buffers (each keeps this object alive): kind, stride,
        compact [n * stride] int8 by slot, rerank [n, 1536] by node, and for "turbo" qjl
        [n, 24] uint64, qjl_res_norms [n], qjl_random_signs [24], qjl_lambda."""
        L = self.layout
        n = L.num_nodes
        out = {"kind": self.kind, "stride": L.stride,
               "compact": _view(L.compact, ctypes.c_int8, (n * L.stride,), np.int8, self),
               "rerank": _view(L.rerank, ctypes.c_float, (n, 1536), np.float32, self)
               if L.rerank else None}
        if L.qjl:
            out.update(qjl=_view(L.qjl, ctypes.c_uint64, (n, 24), np.uint64, self),
                       qjl_res_norms=_view(L.qjl_res_norms, ctypes.c_float, (n,), np.float32,
                                           self),
                       qjl_random_signs=_view(L.qjl_random_signs, ctypes.c_uint64, (24,),
                                              np.uint64, self),
                       qjl_lambda=L.qjl_lambda)
        return out

    def free(self):
        if getattr(self, "h", None):
            self.lib.pion_v_b200_hnsw_quant_free(self.h)
            self.h = None

    def __del__(self):  # pragma: no cover
        try:
            self.free()
        except Exception:
            pass


def hnsw_quant_layout_struct(arrays: dict, num_nodes: int):
    """(pion_b200_hnsw_quant_layout, keep-alive list) from a dict with HNSWQuant.arrays()'
    keys (kind as a name or number; qjl keys and rerank optional)."""
    lay = _lib.HnswQuantLayout()
    keep = []

    def ptr(name, dt):
        a = arrays.get(name)
        if a is None:
            return None
        a = np.ascontiguousarray(a, dtype=dt)
        keep.append(a)
        return a.ctypes.data if a.size else None

    kind = arrays["kind"]
    lay.kind = QUANT_KINDS[kind] if isinstance(kind, str) else int(kind)
    lay.num_nodes = num_nodes
    lay.stride = arrays["stride"]
    lay.compact = ptr("compact", np.int8)
    lay.qjl = ptr("qjl", np.uint64)
    lay.qjl_res_norms = ptr("qjl_res_norms", np.float32)
    lay.qjl_random_signs = ptr("qjl_random_signs", np.uint64)
    lay.qjl_lambda = float(arrays.get("qjl_lambda", 1.0))
    lay.rerank = ptr("rerank", np.float32)
    return lay, keep


class HNSWQuantIndex(_Index):
    """An HNSW graph with block-quantised slots copied to the GPU: the block-quant
    branches of search_fp32_scored (src/vector/hnsw.mojo:4136-4330) with the FP32 rerank
    tail, batched.  graph: HNSWGraph or a layout dict; quant: HNSWQuant or a dict of its
    arrays; rerank=False registers no rerank rows (results keep their block distances)."""

    def __init__(self, ctx: Context, graph, quant, rerank: bool = True):
        if isinstance(graph, HNSWGraph):
            glay, keep = graph.layout, [graph]
        else:
            glay, keep = hnsw_layout_struct(graph)
        if isinstance(quant, HNSWQuant):
            qlay = _lib.HnswQuantLayout.from_buffer_copy(quant.layout)
            keep.append(quant)
        else:
            qlay, k2 = hnsw_quant_layout_struct(quant, glay.num_nodes)
            keep += k2
        if not rerank:
            qlay.rerank = None
        h = ctypes.c_void_p()
        ctx.check(ctx.lib.pion_v_b200_register_hnsw_quant(ctx.h, ctypes.byref(glay),
                                                          ctypes.byref(qlay), ctypes.byref(h)))
        super().__init__(ctx, h)
        self.dim = glay.dim

    def search(self, q, k: int, ef: int, ctx: Context | None = None):
        """q float32 [nq, 1536] -> (external ids int32 [nq, k], scores float32 [nq, k],
        found int32 [nq]); scores are FP32 squared L2 after the rerank, else the block
        distances; -1 / +inf past found."""
        c = ctx or self.ctx
        pq, mem, kq = _ptr(q, np.float32, "q")
        nq = q.shape[0]
        dev = mem == MEM_DEVICE
        ids, sc, pi, pv = _outputs(dev, nq, k, q.device if dev else None)
        if dev:
            found = torch.empty(nq, dtype=torch.int32, device=q.device)
            pf = found.data_ptr()
        else:
            found = np.empty(nq, np.int32)
            pf = found.ctypes.data
        with _TorchStream(c, mem):
            c.check(c.lib.pion_v_b200_hnsw_quant_search(c.h, self.h, pq, nq, k, ef, pi, pv, pf,
                                                         mem))
        return ids, sc, found

    def metric_scores(self, q, ids, scores, ctx: Context | None = None):
        """metric_scores (src/vector/hnsw.mojo:4523-4651) from the FP32 copy: the reply
        scores of `ids` (external ids) in the index metric (squared L2, or 1 - cos under
        COSINE); `scores` (contiguous float32, host) is updated in place.  Returns False,
        leaving the scores, when the graph was registered without FP32 rows."""
        c = ctx or self.ctx
        pq, mem, kq = _ptr(q, np.float32, "q")
        pi, mi, ki = _ptr(ids, np.int32, "ids")
        if not (isinstance(scores, np.ndarray) and scores.dtype == np.float32 and
                scores.flags["C_CONTIGUOUS"]):
            raise TypeError("scores must be a contiguous float32 array (updated in place)")
        m = _same_mem(mem, mi, MEM_HOST)
        nq, k = ids.shape
        rc = c.lib.pion_v_b200_hnsw_metric_scores(c.h, self.h, pq, nq, k, pi,
                                                  scores.ctypes.data, m)
        if rc == 1:
            return False
        c.check(rc)
        return True

    def last_stats(self, ctx: Context | None = None) -> dict:
        """Work of the context's last search: distance evaluations, level-0 expansions,
        queries re-run with room for every node in the candidate heap."""
        c = ctx or self.ctx
        out = (ctypes.c_int64 * 3)()
        c.check(c.lib.pion_v_b200_hnsw_last_stats(c.h, out))
        return dict(zip(("evals", "expansions", "reruns"), list(out)))


def rescore_knn(index, q, ids, scores, ctx: Context | None = None):
    """_rescore_knn (src/commands/vector.mojo:1091-1105) for a batch: the reply scores of
    `ids` in the index metric (metric_scores on the GPU), then each row re-sorted by them,
    ascending and stable (the reference's insertion sort), ids alongside.  `ids` int32
    [nq, k] and `scores` float32 [nq, k], host arrays, are updated in place; when the index
    has no source for metric scores (a block-quantised graph without FP32 rows) both stay
    as they are.  Returns (ids, scores).

    A stable argsort equals the insertion sort on rows without NaN; a row holding a NaN
    is sorted by the insertion loop itself (`<` is false against NaN, so a NaN stops the
    entries behind it where the reference stops them)."""
    if not isinstance(ids, np.ndarray) or not isinstance(scores, np.ndarray):
        raise TypeError("rescore_knn: ids and scores must be host numpy arrays")
    if ids.shape != scores.shape or ids.ndim != 2:
        raise ValueError("rescore_knn: ids and scores must both be [nq, k]")
    ok = index.metric_scores(q, ids, scores, ctx=ctx)
    if ok is False:
        return ids, scores
    nan_rows = np.isnan(scores).any(axis=1)
    order = np.argsort(scores, axis=1, kind="stable")
    clean = ~nan_rows
    ids[clean] = np.take_along_axis(ids[clean], order[clean], axis=1)
    scores[clean] = np.take_along_axis(scores[clean], order[clean], axis=1)
    for t in np.nonzero(nan_rows)[0]:
        si, ss = ids[t], scores[t]
        for a in range(1, ss.shape[0]):
            b = a
            while b > 0 and ss[b] < ss[b - 1]:
                ss[b], ss[b - 1] = ss[b - 1], ss[b]
                si[b], si[b - 1] = si[b - 1], si[b]
                b -= 1
    return ids, scores
