"""The GPU brute-force slot scan against the oracle, bit for bit: the INT8 L2 of every
slot (src/ffi/metal_compute.metal:19-78) through pion_metal_search_topk_w's
worst-replace loop (src/ffi/metal_wrap.m:495-580), entries in the loop's order; and
search_gpu_brute_force (src/vector/hnsw.mojo:3916-3992) with and without FP32 rerank
rows.  Covers several scan stages, ties at every distance, the clamps on k and
num_vectors, lists that overflow into the exact CUDA-core scan, and device memory."""
import numpy as np
import pytest

from pion_b200.workloads import mixture_np

pytestmark = pytest.mark.gpu


def _graph(n, centres, seed, metric="cosine", nq=64):
    import pion_b200
    rows, qs = mixture_np(n, 1536, centres, seed=seed, n_queries=nq)
    g = pion_b200.HNSWGraph(rows, M=8, ef_construction=48, metric=metric, threads=8)
    return g, rows, qs


@pytest.fixture(scope="module")
def small(ctx):
    import pion_b200
    g, rows, qs = _graph(6000, 64, seed=31)
    return g, g.arrays(), pion_b200.HNSWIndex(ctx, g), rows, qs


@pytest.fixture(scope="module")
def large(ctx):
    """40000 slots = 157 tiles: stages [0, 4), [4, 64), [64, 157)."""
    import pion_b200
    g, rows, qs = _graph(40000, 256, seed=37, nq=300)
    return g, g.arrays(), pion_b200.HNSWIndex(ctx, g), rows, qs


def _codes(oracle, A, qs):
    c = oracle.hnsw_query_codes(A, qs)
    return c, (c.astype(np.int32) ** 2).sum(1).astype(np.float32)


def _same(got, want):
    gs, gd = got
    ws, wd = want
    assert np.array_equal(gs, ws)
    assert np.array_equal(gd.view(np.uint32), wd.view(np.uint32))


# the exact prefix (dense rows) covers the first slots; a short prefix sends the rest
# through the candidate lists
PREFIXES = [None, "256", "1024"]


@pytest.fixture(params=PREFIXES, ids=["prefix-default", "prefix-256", "prefix-1024"])
def prefix(request, monkeypatch):
    if request.param is not None:
        monkeypatch.setenv("PION_B200_SLOT_PREFIX", request.param)
    return request.param


@pytest.mark.parametrize("k", [1, 10, 20, 64, 100, 256])
def test_slot_scan_matches_oracle(oracle, small, k, prefix):
    g, A, ix, rows, qs = small
    c, qn = _codes(oracle, A, qs)
    _same(ix.slot_scan_topk(c, k, qn), oracle.slot_scan_topk(A, c, qn, A["num_nodes"], k))


_LARGE_WANT = {}


@pytest.mark.parametrize("k", [10, 40, 200])
def test_slot_scan_stages(oracle, large, k, prefix):
    g, A, ix, rows, qs = large
    c, qn = _codes(oracle, A, qs)
    got = ix.slot_scan_topk(c, k)                      # q_norm computed on the GPU
    if k not in _LARGE_WANT:                           # the oracle's answer, once per k
        _LARGE_WANT[k] = oracle.slot_scan_topk(A, c, qn, A["num_nodes"], k)
    _same(got, _LARGE_WANT[k])
    if prefix is not None:
        assert ix.slot_stats()["replayed"] > 0         # the lists were used


def test_slot_scan_limits_and_device_memory(oracle, small):
    import torch
    g, A, ix, rows, qs = small
    c, qn = _codes(oracle, A, qs[:8])
    for nv, k in ((5, 9), (700, 64), (0, 3), (10 ** 9, 12)):
        want = oracle.slot_scan_topk(A, c, qn, nv, k)
        _same(ix.slot_scan_topk(c, k, qn, num_vectors=nv), want)
    ds, dd = ix.slot_scan_topk(torch.from_numpy(c).cuda(), 16, torch.from_numpy(qn).cuda())
    _same((ds.cpu().numpy(), dd.cpu().numpy()), oracle.slot_scan_topk(A, c, qn, A["num_nodes"], 16))


def test_slot_scan_ties(ctx, oracle, small, prefix):
    """Codes in {-1, 0, 1}: distances collide everywhere, so which tied slots survive
    and at which entry is decided by the loop's order alone."""
    import pion_b200
    g, A, ix, rows, qs = small
    A = dict(A)
    n, stride, hdr = A["num_nodes"], A["compact_stride"], A["compact_hdr"]
    rng = np.random.Generator(np.random.PCG64(8))
    buf = A["compact_buffer"].reshape(n, stride).copy()
    cc = rng.integers(-1, 2, size=(n, 1536)).astype(np.int8)
    buf[:, hdr:hdr + 1536] = cc
    buf[:, :4] = (cc.astype(np.int32) ** 2).sum(1).astype(np.float32)[:, None].view(np.uint8)
    A["compact_buffer"] = buf.reshape(-1)
    tix = pion_b200.HNSWIndex(ctx, A)
    qc = rng.integers(-1, 2, size=(40, 1536)).astype(np.int8)
    qn = (qc.astype(np.int32) ** 2).sum(1).astype(np.float32)
    for k in (7, 64, 256):
        _same(tix.slot_scan_topk(qc, k, qn), oracle.slot_scan_topk(A, qc, qn, n, k))


def test_slot_scan_overflow_and_exact_path(ctx, oracle, small, monkeypatch):
    """Zero codes and slot norms that fall with the slot index make every slot enter the
    loop, so the candidate lists overflow and the exact path takes over; the exact path
    is also forced for ordinary data."""
    import pion_b200
    g, A, ix, rows, qs = small
    c, qn = _codes(oracle, A, qs[:12])
    A2 = dict(A)
    n, stride, hdr = A["num_nodes"], A["compact_stride"], A["compact_hdr"]
    buf = A["compact_buffer"].reshape(n, stride).copy()
    buf[:, hdr:hdr + 1536] = 0
    buf[:, :4] = (4.0e6 - 64.0 * np.arange(n, dtype=np.float32))[:, None].view(np.uint8)
    A2["compact_buffer"] = buf.reshape(-1)
    oix = pion_b200.HNSWIndex(ctx, A2)
    monkeypatch.setenv("PION_B200_SLOT_PREFIX", "256")
    for k in (10, 20, 100):
        _same(oix.slot_scan_topk(c, k, qn), oracle.slot_scan_topk(A2, c, qn, n, k))
        if k == 10:  # lists of 512 slots, 256 kept: every query overflows
            assert oix.slot_stats()["exact_queries"] == len(c)
    monkeypatch.delenv("PION_B200_SLOT_PREFIX")
    _same(ix.slot_scan_topk(c, 30, qn), oracle.slot_scan_topk(A, c, qn, n, 30))
    st = ix.slot_stats()
    assert st["exact_queries"] == 0
    monkeypatch.setenv("PION_B200_SLOT_EXACT", "1")
    _same(ix.slot_scan_topk(c, 30, qn), oracle.slot_scan_topk(A, c, qn, n, 30))
    assert ix.slot_stats()["exact_queries"] == len(c)


@pytest.mark.parametrize("metric", ["cosine", "l2"])
def test_brute_force_matches_oracle(ctx, oracle, metric, prefix):
    import pion_b200
    g, rows, qs = _graph(9000, 64, seed=41, metric=metric, nq=200)
    A = g.arrays()
    ix = pion_b200.HNSWIndex(ctx, g)
    qs = qs * (1.0 if metric == "cosine" else 2.5)
    for k in (10, 150):
        ids, sc, found = ix.brute_force(qs, k)
        wi, ws, wf = oracle.hnsw_brute_force(A, qs, k)
        assert np.array_equal(found, wf) and np.array_equal(ids, wi)
        assert np.array_equal(sc.view(np.uint32), ws.view(np.uint32))
    rr = np.empty_like(rows)
    rr[A["node_slot"]] = rows
    ix.set_rerank_rows(rr)
    for k in (10, 100, 200):
        ids, sc, found = ix.brute_force(qs, k)
        wi, ws, wf = oracle.hnsw_brute_force(A, qs, k, rr)
        assert np.array_equal(found, wf) and np.array_equal(ids, wi)
        assert np.array_equal(sc.view(np.uint32), ws.view(np.uint32))
    ix.set_rerank_rows(None)
    ids, sc, found = ix.brute_force(qs[:5], 10)
    wi, ws, wf = oracle.hnsw_brute_force(A, qs[:5], 10)
    assert np.array_equal(ids, wi)


def test_brute_force_recall(ctx, oracle, small):
    """With rerank rows the brute-force scan is near exact: recall@10 against exact cosine
    top-10 of the rows."""
    g, A, ix, rows, qs = small
    rr = np.empty_like(rows)
    rn = rows / np.linalg.norm(rows, axis=1, keepdims=True)
    rr[A["node_slot"]] = rn
    ix.set_rerank_rows(rr)
    try:
        qn = qs / np.linalg.norm(qs, axis=1, keepdims=True)
        ids, sc, found = ix.brute_force(qn, 10)
    finally:
        ix.set_rerank_rows(None)
    truth = np.argsort(-(qn @ rn.T), axis=1, kind="stable")[:, :10]
    recall = np.mean([len(set(ids[i]) & set(truth[i])) / 10 for i in range(len(qs))])
    assert recall >= 0.97
