"""The oracle's restatement of the GPU brute-force slot scan, checked on CPU against a
second, plain-Python restatement: the shader's distance (src/ffi/metal_compute.metal:
19-78), the worst-replace loop of pion_metal_search_topk_w (src/ffi/metal_wrap.m:
495-580) including where tied entries land, and the composition of
search_gpu_brute_force (src/vector/hnsw.mojo:3916-3992)."""
import numpy as np
import pytest

from pion_b200.workloads import mixture_np


def _loop(dist, k):
    """pion_metal_search_topk_w's top-k loop, statement for statement."""
    k = min(k, len(dist))
    out_d = [np.float32(np.inf)] * k
    out_i = [-1] * k
    worst, widx = np.float32(np.inf), 0
    for i, d in enumerate(dist):
        if d < worst:
            out_d[widx] = d
            out_i[widx] = i
            worst = np.float32(-np.inf)
            for j in range(k):
                if out_d[j] > worst:
                    worst, widx = out_d[j], j
    return np.array(out_i, np.int32), np.array(out_d, np.float32)


def _slot_dists(A, qc, qn):
    """d = (query_norm + cand_norm) - 2 * float(dot), float32 at every step."""
    n, stride, hdr = A["num_nodes"], A["compact_stride"], A["compact_hdr"]
    buf = A["compact_buffer"].reshape(n, stride)
    codes = buf[:, hdr:hdr + 1536].astype(np.int32)
    norms = buf[:, :4].copy().view(np.float32)[:, 0]
    dots = codes @ qc.astype(np.int32)
    return (np.float32(qn) + norms) - np.float32(2.0) * dots.astype(np.float32)


@pytest.fixture(scope="module")
def built():
    import pion_b200
    rows, qs = mixture_np(2000, 1536, 16, seed=23, n_queries=6)
    g = pion_b200.HNSWGraph(rows, M=8, ef_construction=48, threads=1)
    return g, g.arrays(), rows, qs


def test_slot_scan_matches_plain_loop(oracle, built):
    g, A, rows, qs = built
    codes = oracle.hnsw_query_codes(A, qs)
    qn = (codes.astype(np.int32) ** 2).sum(axis=1).astype(np.float32)
    for k in (1, 10, 64):
        slots, dists = oracle.slot_scan_topk(A, codes, qn, A["num_nodes"], k)
        for t in range(len(qs)):
            wi, wd = _loop(_slot_dists(A, codes[t], qn[t]), k)
            assert np.array_equal(slots[t], wi)
            assert np.array_equal(dists[t].view(np.uint32), wd.view(np.uint32))


def test_slot_scan_ties_and_limits(oracle, built):
    """Many equal distances (codes in {-1, 0, 1}): which tied slots survive and at which
    entry follows the loop; k above num_vectors is clamped."""
    g, A, rows, qs = built
    A = dict(A)
    n, stride, hdr = A["num_nodes"], A["compact_stride"], A["compact_hdr"]
    rng = np.random.Generator(np.random.PCG64(5))
    buf = A["compact_buffer"].reshape(n, stride).copy()
    c = rng.integers(-1, 2, size=(n, 1536)).astype(np.int8)
    buf[:, hdr:hdr + 1536] = c
    buf[:, :4] = (c.astype(np.int32) ** 2).sum(1).astype(np.float32)[:, None].view(np.uint8)
    A["compact_buffer"] = buf.reshape(-1)
    qc = rng.integers(-1, 2, size=(3, 1536)).astype(np.int8)
    qn = (qc.astype(np.int32) ** 2).sum(1).astype(np.float32)
    for k in (7, 33):
        slots, dists = oracle.slot_scan_topk(A, qc, qn, n, k)
        for t in range(3):
            d = _slot_dists(A, qc[t], qn[t])
            assert len(np.unique(d)) < n // 4          # ties everywhere
            wi, wd = _loop(d, k)
            assert np.array_equal(slots[t], wi) and np.array_equal(dists[t], wd)
    slots, dists = oracle.slot_scan_topk(A, qc[:1], qn[:1], 5, 9)
    wi, wd = _loop(_slot_dists(A, qc[0], qn[0])[:5], 9)
    assert np.array_equal(slots[0, :5], wi) and (slots[0, 5:] == -1).all()
    assert np.isinf(dists[0, 5:]).all()


def _rerank_l2(q, v):
    acc = np.zeros(8, np.float32)
    for i in range(0, 1536, 8):
        diff = q[i:i + 8] - v[i:i + 8]
        acc = acc + diff * diff
    while len(acc) > 1:
        h = len(acc) // 2
        acc = acc[:h] + acc[h:]
    return acc[0]


@pytest.mark.parametrize("rerank", [False, True])
def test_brute_force_composition(oracle, built, rerank):
    g, A, rows, qs = built
    n = A["num_nodes"]
    slot_ext = np.full(n, -1, np.int32)
    slot_ext[A["node_slot"]] = A["node_ids"]
    rr = None
    if rerank:
        rr = np.empty_like(rows)
        rr[A["node_slot"]] = rows / np.linalg.norm(rows, axis=1, keepdims=True)
    k = 10
    ids, sc, found = oracle.hnsw_brute_force(A, qs, k, rr)
    # normalise once (l2_normalize_fp32), quantise, |code|^2 as f32
    once = oracle.l2_normalize_rows(qs)
    over = min(2 * k, n, 256) if rerank else min(k, 256)
    for t in range(len(qs)):
        qc = oracle.hnsw_query_codes(dict(A, metric=0), once[t:t + 1])[0]
        qn = np.float32((qc.astype(np.int32) ** 2).sum())
        si, sd = _loop(_slot_dists(A, qc, qn), over)
        if rerank:
            sd = np.array([_rerank_l2(qs[t], rr[s]) for s in si], np.float32)
        order = np.argsort(sd, kind="stable")[:k]
        assert found[t] == k
        assert np.array_equal(ids[t], slot_ext[si[order]])
        assert np.array_equal(sc[t].view(np.uint32), sd[order].view(np.uint32))
