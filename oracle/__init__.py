"""CPU oracle for Pion's FT.SEARCH KNN hot path — TEST INFRASTRUCTURE ONLY.

numpy-facing ctypes bindings over ``oracle/liboracle.so`` (built from
``oracle/pion_oracle.c`` by ``oracle/Makefile``).  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import this
package, and only as the checker; the product library ``pion_b200`` never
imports it and has no CPU fallback.

Parity status: UNPINNED — the reference path is Mojo (no toolchain here) and the
reference stores no golden vectors.  Each wrapped function names the reference
``file:line`` it restates (paths inside the pavelhorak/pion repository).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lock = threading.Lock()
_lib = None

_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_p = ctypes.c_void_p
_f32 = ctypes.c_float


def build(force: bool = False) -> str:
    """Compile the C restatement with its Makefile (gcc, no GPU needed)."""
    if force or not os.path.exists(_LIB_PATH) or _stale():
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _stale() -> bool:
    lib_t = os.path.getmtime(_LIB_PATH)
    for f in os.listdir(_HERE):
        if f.endswith((".c", ".h")) and os.path.getmtime(os.path.join(_HERE, f)) > lib_t:
            return True
    return False


def lib() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                build()
            L = ctypes.CDLL(_LIB_PATH)
            L.orc_pkm_quantize_rows_i8.argtypes = [_p, _i64, _i64, _i64, _p, _p]
            L.orc_pkm_scores_i8.argtypes = [_p, _i64, _i64, _p, _p, _p, _i64, _p]
            L.orc_pkm_scores_f32.argtypes = [_p, _i64, _i64, _p, _i64, _p]
            L.orc_pkm_rescore_f32.argtypes = [_p, _i64, _p, _p, _i64, _p]
            L.orc_pkm_sort_desc.argtypes = [_p, _p, _i64]
            L.orc_pkm_topk_max.argtypes = [_p, _i64, _i64, _p, _p]
            L.orc_pkm_topk_max.restype = _i64
            L.orc_pkm_combine_topk.argtypes = [_p, _p, _i64, _p, _p, _i64, _i64, _i64, _p, _p]
            L.orc_pkm_combine_topk.restype = _i64
            L.orc_flat_i8_knn.argtypes = [_p, _i64, _i64, _p, _p, _p, _i64, _i64, _p, _p, _i32]
            L.orc_dot_f32_4chain.argtypes = [_p, _p, _i64]
            L.orc_dot_f32_4chain.restype = _f32
            L.orc_l2sq_f32_4chain.argtypes = [_p, _p, _i64]
            L.orc_l2sq_f32_4chain.restype = _f32
            L.orc_l2_normalize_fp32.argtypes = [_p, _p, _i64]
            L.orc_exact_query_normalize.argtypes = [_p, _p, _i64, _i32]
            L.orc_exact_knn.argtypes = [_p, _i64, _i64, _p, _i64, _i32, _p, _p]
            L.orc_exact_knn.restype = _i64
            L.orc_exact_knn_batch.argtypes = [_p, _i64, _i64, _p, _i64, _i64, _i32, _p, _p, _i32]
            L.orc_bq_pack_signs.argtypes = [_p, _i64, _i64, _p]
            L.orc_hamming.argtypes = [_p, _p, _i64]
            L.orc_hamming.restype = _i64
            L.orc_bq_knn_batch.argtypes = [_p, _p, _i64, _i64, _p, _i64, _i64, _i64, _p, _p, _p,
                                           _p, _i32]
            L.orc_shard_merge_asc.argtypes = [_p, _p, _i64, _i64, _p, _p]
            L.orc_shard_merge_asc.restype = _i64
            L.orc_hnsw_search.argtypes = [_p, _p, _i64, _i64, _i64, _p, _p, _p, _i32]
            L.orc_hnsw_search.restype = _i32
            L.orc_hnsw_search_ft.argtypes = [_p, _p, _i64, _i64, _i64, _p, _p, _p, _i32]
            L.orc_hnsw_search_ft.restype = _i32
            L.orc_hnsw_query_codes.argtypes = [_p, _p, _i64, _p]
            L.orc_hnsw_beam_pool.argtypes = [_p, _p, _f32, _i64, _p, _p, _i64, _i64, _p, _p]
            L.orc_hnsw_beam_pool.restype = _i64
            L.orc_hnsw_metric_scores.argtypes = [_p, _p, _i64, _i64, _p, _p]
            L.orc_slot_scan_topk.argtypes = [_p, _p, ctypes.c_float, _i64, _i64, _p, _p]
            L.orc_slot_scan_topk.restype = _i64
            L.orc_hnsw_brute_force.argtypes = [_p, _p, _p, _i64, _i64, _p, _p, _p]
            _lib = L
    return _lib


class _HnswLayout(ctypes.Structure):
    """orc_hnsw_layout (oracle/pion_oracle.h)."""
    _fields_ = [
        ("num_nodes", _i64), ("dim", _i64), ("M", _i64), ("entry_point", _i64),
        ("max_level", _i64), ("global_min", _f32), ("global_max", _f32),
        ("metric", ctypes.c_int32), ("reserved", ctypes.c_int32),
        ("compact_buffer", _p), ("compact_stride", _i64), ("compact_hdr", _i64),
        ("l0_compact", _p), ("l0_slots", _p), ("node_slot", _p), ("node_ids", _p),
        ("deleted", _p), ("node_level", _p), ("upper_offset", _p), ("upper_links", _p),
        ("upper_rows", _i64),
    ]


_HNSW_ARRAYS = {"compact_buffer": np.int8, "l0_compact": np.uint32, "l0_slots": np.uint32,
                "node_slot": np.uint32, "node_ids": np.int32, "node_level": np.int8,
                "upper_offset": np.int64, "upper_links": np.uint32}
_HNSW_SCALARS = ("num_nodes", "dim", "M", "entry_point", "max_level", "global_min",
                 "global_max", "metric", "compact_stride", "compact_hdr", "upper_rows")


def _hnsw_layout(g: dict):
    lay = _HnswLayout()
    keep = []
    for name in _HNSW_SCALARS:
        setattr(lay, name, g[name])
    for name, dt in _HNSW_ARRAYS.items():
        a, p = _c(g[name], dt)
        keep.append(a)
        setattr(lay, name, p if a.size else None)
    if g.get("deleted") is not None:
        a, p = _c(g["deleted"], np.uint8)
        keep.append(a)
        lay.deleted = p
    return lay, keep


def _c(a, dtype):
    a = np.ascontiguousarray(a, dtype=dtype)
    return a, a.ctypes.data_as(_p)


def default_threads() -> int:
    return max(1, os.cpu_count() or 1)


# --------------------------------------------------------------------------
# PKM routines (src/vector/pkm_kernels.mojo, src/vector/reference/pkm_ref.mojo)
# --------------------------------------------------------------------------

def pkm_quantize_rows_i8(src: np.ndarray, d: int | None = None):
    """src/vector/pkm_kernels.mojo:152-191.  src: [n, d_pad] float32 -> (int8, scale)."""
    src, ps = _c(src, np.float32)
    n, d_pad = src.shape
    d = d_pad if d is None else d
    out = np.empty((n, d_pad), np.int8)
    sc = np.empty(n, np.float32)
    lib().orc_pkm_quantize_rows_i8(ps, n, d, d_pad, out.ctypes.data_as(_p), sc.ctypes.data_as(_p))
    return out, sc


def pkm_scores_i8(keys, row_scale, q, q_scale) -> np.ndarray:
    """src/vector/reference/pkm_ref.mojo:47-61.  -> [nq, S] float32."""
    keys, pk = _c(keys, np.int8)
    row_scale, pr = _c(row_scale, np.float32)
    q, pq = _c(q, np.int8)
    q_scale, pqs = _c(q_scale, np.float32)
    s, d_pad = keys.shape
    nq = q.shape[0]
    dst = np.empty((nq, s), np.float32)
    lib().orc_pkm_scores_i8(pk, s, d_pad, pr, pq, pqs, nq, dst.ctypes.data_as(_p))
    return dst


def pkm_scores_f32(keys, q) -> np.ndarray:
    """src/vector/reference/pkm_ref.mojo:22-31."""
    keys, pk = _c(keys, np.float32)
    q, pq = _c(q, np.float32)
    s, d_pad = keys.shape
    nq = q.shape[0]
    dst = np.empty((nq, s), np.float32)
    lib().orc_pkm_scores_f32(pk, s, d_pad, pq, nq, dst.ctypes.data_as(_p))
    return dst


def pkm_rescore_f32(keys, q, idx) -> np.ndarray:
    """src/vector/reference/pkm_ref.mojo:34-44."""
    keys, pk = _c(keys, np.float32)
    q, pq = _c(q, np.float32)
    idx, pi = _c(idx, np.int32)
    dst = np.empty(idx.shape[0], np.float32)
    lib().orc_pkm_rescore_f32(pk, keys.shape[1], pq, pi, idx.shape[0], dst.ctypes.data_as(_p))
    return dst


def pkm_sort_desc(val, idx):
    """src/vector/reference/pkm_ref.mojo:92-107 (in place on copies)."""
    val = np.array(val, np.float32, copy=True)
    idx = np.array(idx, np.int32, copy=True)
    lib().orc_pkm_sort_desc(val.ctypes.data_as(_p), idx.ctypes.data_as(_p), val.shape[0])
    return val, idx


def pkm_topk_max(scores, k: int):
    """src/vector/reference/pkm_ref.mojo:110-130.  -> (idx int32[kk], val float32[kk])."""
    scores, ps = _c(scores, np.float32)
    kk = max(0, min(k, scores.shape[0]))
    oi = np.empty(max(kk, 1), np.int32)
    ov = np.empty(max(kk, 1), np.float32)
    got = lib().orc_pkm_topk_max(ps, scores.shape[0], k, oi.ctypes.data_as(_p),
                                 ov.ctypes.data_as(_p))
    return oi[:got], ov[:got]


def pkm_combine_topk(s0, i0, s1, i1, s_cols: int, k: int):
    """src/vector/reference/pkm_ref.mojo:133-160."""
    s0, p0 = _c(s0, np.float32)
    i0, q0 = _c(i0, np.int32)
    s1, p1 = _c(s1, np.float32)
    i1, q1 = _c(i1, np.int32)
    cap = max(1, min(k, s0.shape[0] * s1.shape[0]))
    oi = np.empty(cap, np.int32)
    ov = np.empty(cap, np.float32)
    got = lib().orc_pkm_combine_topk(p0, q0, s0.shape[0], p1, q1, s1.shape[0], s_cols, k,
                                     oi.ctypes.data_as(_p), ov.ctypes.data_as(_p))
    return oi[:got], ov[:got]


def flat_i8_knn(keys, row_scale, q, q_scale, k: int, nthreads: int | None = None):
    """pkm_scores_i8 + pkm_topk_max per query, streamed.  -> (idx [nq,k], val [nq,k])."""
    keys, pk = _c(keys, np.int8)
    row_scale, pr = _c(row_scale, np.float32)
    q, pq = _c(q, np.int8)
    q_scale, pqs = _c(q_scale, np.float32)
    n, d_pad = keys.shape
    nq = q.shape[0]
    oi = np.empty((nq, k), np.int32)
    ov = np.empty((nq, k), np.float32)
    lib().orc_flat_i8_knn(pk, n, d_pad, pr, pq, pqs, nq, k, oi.ctypes.data_as(_p),
                          ov.ctypes.data_as(_p), nthreads or default_threads())
    return oi, ov


# --------------------------------------------------------------------------
# Exact FP32 rows (src/vector/fp32_scan.mojo, src/commands/vector.mojo)
# --------------------------------------------------------------------------

def dot_f32_4chain(q, v) -> float:
    q, pq = _c(q, np.float32)
    v, pv = _c(v, np.float32)
    return lib().orc_dot_f32_4chain(pq, pv, q.shape[0])


def l2sq_f32_4chain(a, b) -> float:
    a, pa = _c(a, np.float32)
    b, pb = _c(b, np.float32)
    return lib().orc_l2sq_f32_4chain(pa, pb, a.shape[0])


def l2_normalize_rows(x) -> np.ndarray:
    """src/vector/kernels.mojo:318-357 applied to every row."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    L = lib()
    dim = x.shape[1]
    for r in range(x.shape[0]):
        L.orc_l2_normalize_fp32(x[r].ctypes.data_as(_p), out[r].ctypes.data_as(_p), dim)
    return out


def exact_query_normalize(query, cosine: bool = True) -> np.ndarray:
    query, pq = _c(query, np.float32)
    out = np.empty_like(query)
    lib().orc_exact_query_normalize(pq, out.ctypes.data_as(_p), query.shape[0], int(cosine))
    return out


def exact_knn(rows, queries, k: int, cosine: bool = True, nthreads: int | None = None):
    """src/commands/vector.mojo:1228-1365 per query.  -> (ids int64 [nq,k], scores [nq,k])."""
    rows, pr = _c(rows, np.float32)
    queries, pq = _c(np.atleast_2d(queries), np.float32)
    n, dim = rows.shape
    nq = queries.shape[0]
    ids = np.empty((nq, k), np.int64)
    sc = np.empty((nq, k), np.float32)
    lib().orc_exact_knn_batch(pr, n, dim, pq, nq, k, int(cosine), ids.ctypes.data_as(_p),
                              sc.ctypes.data_as(_p), nthreads or default_threads())
    return ids, sc


# --------------------------------------------------------------------------
# Binary quantisation + rerank (composed)
# --------------------------------------------------------------------------

def bq_pack_signs(rows) -> np.ndarray:
    rows, pr = _c(np.atleast_2d(rows), np.float32)
    n, dim = rows.shape
    codes = np.empty((n, dim // 64), np.uint64)
    lib().orc_bq_pack_signs(pr, n, dim, codes.ctypes.data_as(_p))
    return codes


def hamming(a, b) -> int:
    a, pa = _c(a, np.uint64)
    b, pb = _c(b, np.uint64)
    return lib().orc_hamming(pa, pb, a.shape[0])


def bq_knn(codes, rows, queries, shortlist: int, k: int, nthreads: int | None = None):
    """Hamming shortlist (distance, id) then exact COSINE rerank (stable by score)."""
    codes, pc = _c(codes, np.uint64)
    rows, pr = _c(rows, np.float32)
    queries, pq = _c(np.atleast_2d(queries), np.float32)
    n, dim = rows.shape
    nq = queries.shape[0]
    ids = np.empty((nq, k), np.int64)
    sc = np.empty((nq, k), np.float32)
    sid = np.empty((nq, shortlist), np.int32)
    sd = np.empty((nq, shortlist), np.int32)
    lib().orc_bq_knn_batch(pc, pr, n, dim, pq, nq, shortlist, k, ids.ctypes.data_as(_p),
                           sc.ctypes.data_as(_p), sid.ctypes.data_as(_p), sd.ctypes.data_as(_p),
                           nthreads or default_threads())
    return ids, sc, sid, sd


def shard_merge_asc(ids, scores, k: int):
    """src/commands/vector.mojo:4394-4429 (selection sort over concatenated shards)."""
    ids, pi = _c(ids, np.int64)
    scores, ps = _c(scores, np.float32)
    n = ids.shape[0]
    oi = np.empty(max(1, k), np.int64)
    os_ = np.empty(max(1, k), np.float32)
    got = lib().orc_shard_merge_asc(pi, ps, n, k, oi.ctypes.data_as(_p), os_.ctypes.data_as(_p))
    return oi[:got], os_[:got]


def hnsw_search(graph: dict, queries, k: int, ef: int, nthreads: int | None = None,
                ft: bool = False):
    """search_fp32_scored at dim 1536 (src/vector/hnsw.mojo:4136-4521) over a graph in
    the compact layout (a dict with the fields of pion_b200_hnsw_layout as numpy arrays
    and scalars): upper-level greedy in code space (:3789-3848), then
    beam_search_1536_ref (src/vector/reference/beam_1536.mojo:85-135) over a LinearPool
    (src/common/heap.mojo:133-234).  ft=True: the FT.SEARCH composition, whose start node
    comes from _upper_level_greedy on the raw query (greedy codes of the once-normalised
    query; src/commands/vector.mojo:4514-4518).  Returns (ids int32 [nq, k], dist float32
    [nq, k], stats {evals, expansions, upper_evals})."""
    L = lib()
    lay, keep = _hnsw_layout(graph)
    q, qp = _c(queries, np.float32)
    nq = q.shape[0]
    ids = np.empty((nq, k), np.int32)
    dist = np.empty((nq, k), np.float32)
    st = np.zeros(3, np.int64)
    fn = L.orc_hnsw_search_ft if ft else L.orc_hnsw_search
    rc = fn(ctypes.byref(lay), qp, nq, k, ef, ids.ctypes.data_as(_p),
                           dist.ctypes.data_as(_p), st.ctypes.data_as(_p),
                           nthreads or default_threads())
    if rc != 0:
        raise ValueError("orc_hnsw_search: layout not supported")
    del keep
    return ids, dist, {"evals": int(st[0]), "expansions": int(st[1]), "upper_evals": int(st[2])}


def hnsw_query_codes(graph: dict, queries):
    """The int8 codes _quantize_query_to_int8 gives each query (after the search's
    normalisation), [nq, 1536]."""
    L = lib()
    lay, keep = _hnsw_layout(graph)
    q, qp = _c(queries, np.float32)
    out = np.empty(q.shape, np.int8)
    L.orc_hnsw_query_codes(ctypes.byref(lay), qp, q.shape[0], out.ctypes.data_as(_p))
    return out


def hnsw_beam_pool(graph: dict, q_codes, qn: float, ef: int, init_d, init_id, cursor: int = 0):
    """beam_search_1536_ref (src/vector/reference/beam_1536.mojo:85-135) from a seeded
    LinearPool: q_codes int8[1536], qn the query's |code|^2 as a float, the pool's
    (dist, id) entries (bit 31 of id = expanded) and cursor.  Returns the final pool as
    (dist float32 [size], id uint32 [size])."""
    L = lib()
    lay, keep = _hnsw_layout(graph)
    q, qp = _c(q_codes, np.int8)
    d0, dp = _c(init_d, np.float32)
    i0, ip = _c(init_id, np.uint32)
    out_d = np.empty(max(1, ef), np.float32)
    out_i = np.empty(max(1, ef), np.uint32)
    n = L.orc_hnsw_beam_pool(ctypes.byref(lay), qp, float(qn), ef, dp, ip, len(d0), cursor,
                             out_d.ctypes.data_as(_p), out_i.ctypes.data_as(_p))
    if n < 0:
        raise ValueError("orc_hnsw_beam_pool failed")
    del keep
    return out_d[:n].copy(), out_i[:n].copy()


def hnsw_metric_scores(graph: dict, queries, ids, scores):
    """metric_scores (src/vector/hnsw.mojo:4523-4651) for INT8 codes: returns a copy of
    `scores` with every id that names a node replaced by its metric distance."""
    L = lib()
    lay, keep = _hnsw_layout(graph)
    q, qp = _c(queries, np.float32)
    i, ip = _c(ids, np.int32)
    out = np.array(scores, dtype=np.float32, copy=True, order="C")
    L.orc_hnsw_metric_scores(ctypes.byref(lay), qp, i.shape[0], i.shape[1], ip,
                             out.ctypes.data_as(_p))
    del keep
    return out


def slot_scan_topk(graph: dict, qcodes, qnorm, num_vectors: int, k: int):
    """The GPU brute-force slot scan (src/ffi/metal_compute.metal:19-78) and its
    worst-replace top-k (src/ffi/metal_wrap.m:495-580) per query: (slots [nq, k],
    dists [nq, k]) in the order the loop leaves them; -1 / +inf past min(k, n)."""
    L = lib()
    lay, keep = _hnsw_layout(graph)
    q = np.ascontiguousarray(qcodes, dtype=np.int8)
    nq = q.shape[0]
    qn = np.ascontiguousarray(qnorm, dtype=np.float32)
    slots = np.full((nq, k), -1, np.int32)
    dists = np.full((nq, k), np.inf, np.float32)
    for t in range(nq):
        L.orc_slot_scan_topk(ctypes.byref(lay), q[t].ctypes.data_as(_p), float(qn[t]),
                             num_vectors, k, slots[t].ctypes.data_as(_p),
                             dists[t].ctypes.data_as(_p))
    del keep
    return slots, dists


def hnsw_brute_force(graph: dict, queries, k: int, rerank=None):
    """search_gpu_brute_force (src/vector/hnsw.mojo:3916-3992): (ids, scores, found)."""
    L = lib()
    lay, keep = _hnsw_layout(graph)
    q, qp = _c(queries, np.float32)
    nq = q.shape[0]
    rp = None
    if rerank is not None:
        r, rp = _c(rerank, np.float32)
        keep.append(r)
    ids = np.empty((nq, k), np.int32)
    sc = np.empty((nq, k), np.float32)
    found = np.empty(nq, np.int32)
    L.orc_hnsw_brute_force(ctypes.byref(lay), rp, qp, nq, k, ids.ctypes.data_as(_p),
                           sc.ctypes.data_as(_p), found.ctypes.data_as(_p))
    del keep
    return ids, sc, found


def merge_delta(rows, built: int, cosine: bool, queries, ids, scores, k: int):
    """merge_delta (src/commands/vector.mojo:1368-1410) per query, composed from the
    restated pieces: _exact_rescore (:1413-1456: graph results below `built` rescored from
    the FP32 rows, 1 - dot_f32_4chain(q^, row) or l2sq_f32_4chain(q, row), then the stable
    insertion sort), exact_knn over rows [built, len(rows)), and the merge loop (a graph
    entry first when its score <= the delta entry's, k kept).  ids/scores [nq, kg] with
    -1 ending a list.  Returns (rescored ids, rescored scores, merged ids [nq, k], merged
    scores [nq, k]); merged entries past the lists are -1 / +inf."""
    rows = np.ascontiguousarray(rows, np.float32)
    queries = np.ascontiguousarray(np.atleast_2d(queries), np.float32)
    nq, kg = ids.shape
    r_ids = np.array(ids, np.int32, copy=True)
    r_sc = np.array(scores, np.float32, copy=True)
    n_rows = rows.shape[0]
    b = min(built, n_rows)
    if n_rows > b:
        d_ids, d_sc = exact_knn(rows[b:], queries, k, cosine=cosine)
    out_i = np.full((nq, k), -1, np.int32)
    out_s = np.full((nq, k), np.inf, np.float32)
    for t in range(nq):
        q = exact_query_normalize(queries[t], cosine)
        n = 0
        while n < kg and r_ids[t, n] >= 0:
            n += 1
        li, ls = list(r_ids[t, :n]), list(r_sc[t, :n])
        for j in range(n):
            s = li[j]
            if 0 <= s < b:
                ls[j] = (np.float32(1.0) - np.float32(dot_f32_4chain(q, rows[s])) if cosine
                         else np.float32(l2sq_f32_4chain(q, rows[s])))
        for a in range(1, n):  # insertion sort, strict <
            j = a
            while j > 0 and ls[j] < ls[j - 1]:
                ls[j], ls[j - 1] = ls[j - 1], ls[j]
                li[j], li[j - 1] = li[j - 1], li[j]
                j -= 1
        r_ids[t, :n], r_sc[t, :n] = li, ls
        dl_i, dl_s = [], []
        if n_rows > b:
            for j in range(k):
                if d_ids[t, j] >= 0 and np.isfinite(d_sc[t, j]):
                    dl_i.append(int(d_ids[t, j]) + b)
                    dl_s.append(np.float32(d_sc[t, j]))
        a = bb = o = 0
        while o < k and (a < n or bb < len(dl_i)):
            if bb >= len(dl_i) or (a < n and ls[a] <= dl_s[bb]):
                out_i[t, o], out_s[t, o] = li[a], ls[a]
                a += 1
            else:
                out_i[t, o], out_s[t, o] = dl_i[bb], dl_s[bb]
                bb += 1
            o += 1
    return r_ids, r_sc, out_i, out_s


# --------------------------------------------------------------------------
# Block-quantised HNSW (oracle/quant_oracle.c)
# --------------------------------------------------------------------------

QUANT_KINDS = {"polar": 0, "nano": 1, "turbo": 2}


class _QuantLayout(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("metric", ctypes.c_int32),
                ("num_nodes", ctypes.c_int64), ("M", ctypes.c_int64),
                ("entry_point", ctypes.c_int64), ("max_level", ctypes.c_int64),
                ("compact", _p), ("stride", ctypes.c_int64),
                ("l0_compact", _p), ("l0_slots", _p), ("node_slot", _p), ("node_ids", _p),
                ("deleted", _p), ("node_level", _p), ("upper_offset", _p),
                ("upper_links", _p), ("qjl", _p), ("qjl_res_norms", _p),
                ("qjl_random_signs", _p), ("qjl_lambda", ctypes.c_float), ("rerank", _p)]


def _qlib():
    L = lib()
    if not getattr(L, "_quant_bound", False):
        L.orc_f32_to_f16.argtypes = [ctypes.c_float]
        L.orc_f32_to_f16.restype = ctypes.c_uint16
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_f16_to_f32.restype = ctypes.c_float
        L.orc_quant_stride.argtypes = [ctypes.c_int]
        L.orc_quant_stride.restype = _i64
        L.orc_quant_block.argtypes = [ctypes.c_int, _p, _p]
        L.orc_quant_dot.argtypes = [ctypes.c_int, _p, _p, _p]
        L.orc_quant_dot.restype = ctypes.c_float
        L.orc_query_block_int8.argtypes = [_p, _p, _p]
        L.orc_query_block_int8.restype = ctypes.c_float
        L.orc_qjl_random_signs.argtypes = [_p]
        L.orc_qjl_signs.argtypes = [_p, _p, _p]
        L.orc_qjl_signs.restype = ctypes.c_float
        L.orc_turbo_qjl_row.argtypes = [_p, _p, _p, _p]
        L.orc_turbo_qjl_row.restype = ctypes.c_float
        L.orc_quant_search.argtypes = [_p, _p, _i64, _i64, _i64, _p, _p, _p, ctypes.c_int]
        L.orc_quant_search.restype = ctypes.c_int
        L.orc_quant_beam_heaps.argtypes = [_p, _p, _p, ctypes.c_float, _p, ctypes.c_float, _i64,
                                           _p, _p, _p, _i64, _p, _p, _p, _p, _p]
        L.orc_quant_beam_heaps.restype = ctypes.c_int
        L._quant_bound = True
    return L


def f32_to_f16_bits(x):
    L = _qlib()
    return np.array([L.orc_f32_to_f16(float(v)) for v in np.ravel(x)], np.uint16)


def quant_block(kind: str, x) -> np.ndarray:
    """One vector's block slot (quantize_fp32_to_block_int4 / _int3 / _int2)."""
    L = _qlib()
    k = QUANT_KINDS[kind]
    x, px = _c(x, np.float32)
    out = np.zeros(L.orc_quant_stride(k), np.int8)
    L.orc_quant_block(k, px, out.ctypes.data_as(_p))
    return out


def quant_dot(kind: str, qcodes, qscales, slot) -> float:
    L = _qlib()
    a, pa = _c(qcodes, np.int8)
    b, pb = _c(qscales, np.float32)
    c, pc = _c(slot, np.int8)
    return L.orc_quant_dot(QUANT_KINDS[kind], pa, pb, pc)


def query_block_int8(q):
    """quantize_fp32_to_block_int8 -> (codes int8 [1536], scales f32 [48], recon |q|^2)."""
    L = _qlib()
    q, pq = _c(q, np.float32)
    codes = np.empty(1536, np.int8)
    scales = np.empty(48, np.float32)
    n = L.orc_query_block_int8(pq, codes.ctypes.data_as(_p), scales.ctypes.data_as(_p))
    return codes, scales, np.float32(n)


def qjl_random_signs() -> np.ndarray:
    out = np.empty(24, np.uint64)
    _qlib().orc_qjl_random_signs(out.ctypes.data_as(_p))
    return out


def qjl_signs(residual, signs):
    L = _qlib()
    r, pr = _c(residual, np.float32)
    s, ps = _c(signs, np.uint64)
    out = np.empty(24, np.uint64)
    n = L.orc_qjl_signs(pr, ps, out.ctypes.data_as(_p))
    return out, np.float32(n)


def quant_graph(graph: dict, rows, kind: str, rerank: bool = True):
    """The block-quant compact buffer of `graph` (slot order of its node_slot), the QJL rows
    by node (TurboQuant) and the FP32 rerank rows by node, from the rows the graph was built
    from (normalised first under COSINE)."""
    rows = np.ascontiguousarray(rows, np.float32)
    if graph["metric"] == 1:
        rows = l2_normalize_rows(rows)
    n = graph["num_nodes"]
    k = QUANT_KINDS[kind]
    L = _qlib()
    stride = L.orc_quant_stride(k)
    comp = np.zeros((n, stride), np.int8)
    slot = graph["node_slot"].astype(np.int64)
    for i in range(n):
        L.orc_quant_block(k, rows[i].ctypes.data_as(_p), comp[slot[i]].ctypes.data_as(_p))
    out = {"kind": kind, "compact": comp.reshape(-1), "stride": stride,
           "rerank": rows if rerank else None}
    if kind == "turbo":
        rs = qjl_random_signs()
        qjl = np.zeros((n, 24), np.uint64)
        norms = np.zeros(n, np.float32)
        for i in range(n):
            norms[i] = L.orc_turbo_qjl_row(rows[i].ctypes.data_as(_p),
                                           comp[slot[i]].ctypes.data_as(_p),
                                           rs.ctypes.data_as(_p), qjl[i].ctypes.data_as(_p))
        out.update(qjl=qjl, qjl_res_norms=norms, qjl_random_signs=rs, qjl_lambda=1.0)
    return out


def _quant_layout(graph: dict, quant: dict):
    """(orc_quant_layout, keep-alive list) of a graph dict and a quant dict."""
    keep = []

    def ptr(a, dt):
        if a is None:
            return None
        a = np.ascontiguousarray(a, dtype=dt)
        keep.append(a)
        return a.ctypes.data_as(_p)

    lay = _QuantLayout()
    lay.kind = QUANT_KINDS[quant["kind"]]
    lay.metric = graph["metric"]
    lay.num_nodes, lay.M = graph["num_nodes"], graph["M"]
    lay.entry_point, lay.max_level = graph["entry_point"], graph["max_level"]
    lay.compact = ptr(quant["compact"], np.int8)
    lay.stride = quant["stride"]
    lay.l0_compact = ptr(graph["l0_compact"], np.uint32)
    lay.l0_slots = ptr(graph["l0_slots"], np.uint32)
    lay.node_slot = ptr(graph["node_slot"], np.uint32)
    lay.node_ids = ptr(graph["node_ids"], np.int32)
    lay.deleted = ptr(graph.get("deleted"), np.uint8)
    lay.node_level = ptr(graph["node_level"], np.int8)
    lay.upper_offset = ptr(graph["upper_offset"], np.int64)
    lay.upper_links = ptr(graph["upper_links"], np.uint32)
    lay.qjl = ptr(quant.get("qjl"), np.uint64)
    lay.qjl_res_norms = ptr(quant.get("qjl_res_norms"), np.float32)
    lay.qjl_random_signs = ptr(quant.get("qjl_random_signs"), np.uint64)
    lay.qjl_lambda = quant.get("qjl_lambda", 1.0)
    lay.rerank = ptr(quant.get("rerank"), np.float32)
    return lay, keep


def quant_search(graph: dict, quant: dict, queries, k: int, ef: int, nthreads: int | None = None):
    """search_fp32_scored's block-quant branch (src/vector/hnsw.mojo:4136-4330) with the
    shared FP32 rerank tail -> (external ids [nq, k], scores [nq, k], counts [nq])."""
    L = _qlib()
    lay, keep = _quant_layout(graph, quant)
    q, pq = _c(np.atleast_2d(queries), np.float32)
    nq = q.shape[0]
    ids = np.empty((nq, k), np.int32)
    sc = np.empty((nq, k), np.float32)
    cnt = np.empty(nq, np.int64)
    rc = L.orc_quant_search(ctypes.byref(lay), pq, nq, k, ef, ids.ctypes.data_as(_p),
                            sc.ctypes.data_as(_p), cnt.ctypes.data_as(_p),
                            nthreads or default_threads())
    if rc != 0:
        raise RuntimeError("orc_quant_search failed")
    del keep
    return ids, sc, cnt


def quant_beam_heaps(graph: dict, quant: dict, qcodes, qscales, qnorm, qsig, qres, ef: int,
                     cand, res, worst, cand_cap: int | None = None):
    """quant_beam_search_1536_ref on a view's state: the query (codes, scales, |q|^2, QJL
    signs or None, residual norm) and the heaps as lists of (distance, node) in array order
    (their nodes visited) -> (candidates [up to cand_cap], the whole candidate count,
    results, results' cached worst)."""
    L = _qlib()
    lay, keep = _quant_layout(graph, quant)
    n = graph["num_nodes"] + len(cand) + 1
    cap = n if cand_cap is None else cand_cap
    cd = np.zeros(max(n, len(cand)), np.float32)
    ci = np.zeros(max(n, len(cand)), np.int64)
    for i, (d, j) in enumerate(cand):
        cd[i], ci[i] = d, j
    rd = np.zeros(max(ef, len(res)) + 1, np.float32)
    ri = np.zeros(max(ef, len(res)) + 1, np.int64)
    for i, (d, j) in enumerate(res):
        rd[i], ri[i] = d, j
    cn, rn, tot = ctypes.c_int64(len(cand)), ctypes.c_int64(len(res)), ctypes.c_int64(0)
    w = ctypes.c_float(worst)
    qc, pqc = _c(qcodes, np.int8)
    qs_, pqs = _c(qscales, np.float32)
    sig = None if qsig is None else np.ascontiguousarray(qsig, np.uint64)
    rc = L.orc_quant_beam_heaps(ctypes.byref(lay), pqc, pqs, float(qnorm),
                                None if sig is None else sig.ctypes.data_as(_p), float(qres), ef,
                                cd.ctypes.data_as(_p), ci.ctypes.data_as(_p), ctypes.byref(cn),
                                cap, ctypes.byref(tot), rd.ctypes.data_as(_p),
                                ri.ctypes.data_as(_p), ctypes.byref(rn), ctypes.byref(w))
    if rc != 0:
        raise RuntimeError("orc_quant_beam_heaps failed")
    del keep
    return ([(cd[i], int(ci[i])) for i in range(cn.value)], tot.value,
            [(rd[i], int(ri[i])) for i in range(rn.value)], np.float32(w.value))


def metric_scores_f32(graph: dict, rows, queries, ids, scores):
    """metric_scores' FP32-copy branch (src/vector/hnsw.mojo:4586-4600) with the rows by
    node -> new scores (ids that name no node keep theirs)."""
    L = lib()
    L.orc_metric_scores_f32.argtypes = [_p, _i64, ctypes.c_int, _p, _p, _i64, _i64, _p, _p]
    nid, pn = _c(graph["node_ids"], np.int32)
    r, pr = _c(rows, np.float32)
    q, pq = _c(np.atleast_2d(queries), np.float32)
    i, pi = _c(ids, np.int32)
    out = np.array(scores, np.float32, copy=True)
    L.orc_metric_scores_f32(pn, graph["num_nodes"], graph["metric"], pr, pq, q.shape[0],
                            i.shape[1], pi, out.ctypes.data_as(_p))
    return out
