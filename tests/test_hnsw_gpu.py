"""HNSW INT8 search on the GPU against the oracle's restatement of the reference's
search_fp32_scored at dim 1536 (src/vector/hnsw.mojo:4136-4521): the same
host-built graph, the same queries.  The beam replays LinearPool
(src/common/heap.mojo:133-234) and the lane formulas of beam_search_1536_ref
(src/vector/reference/beam_1536.mojo:85-135) exactly, so the pools, and with them the
returned ids, distances and work counters, must be identical; recall@10 then matches
the reference's trivially (the parity bar is 0.5 points)."""
import numpy as np
import pytest

from pion_b200.workloads import mixture_np

pytestmark = pytest.mark.gpu


def _graph(n, centres, seed, threads=1, metric="cosine", M=16, efc=100, nq=64):
    import pion_b200
    rows, qs = mixture_np(n, 1536, centres, seed=seed, n_queries=nq)
    g = pion_b200.HNSWGraph(rows, M=M, ef_construction=efc, metric=metric, threads=threads)
    return g, rows, qs


def _same(oracle, A, ix, qs, k, ef):
    ids, dist = ix.search(qs, k, ef)
    st = ix.last_stats()
    oi, od, ost = oracle.hnsw_search(A, qs, k, ef)
    assert np.array_equal(ids, oi), f"ids differ at ef={ef}"
    assert np.array_equal(dist.view(np.uint32), od.view(np.uint32)), f"dists differ at ef={ef}"
    assert st == ost, (st, ost)
    return ids, dist


@pytest.fixture(scope="module")
def small(ctx):
    import pion_b200
    g, rows, qs = _graph(6000, 64, seed=3)
    return g, g.arrays(), pion_b200.HNSWIndex(ctx, g), rows, qs


@pytest.mark.parametrize("ef", [1, 4, 10, 16, 64, 128, 256, 1024])
def test_beam_matches_oracle(oracle, small, ef):
    g, A, ix, rows, qs = small
    _same(oracle, A, ix, qs, 10, ef)


def test_k_beyond_pool_and_device_memory(oracle, small):
    import torch
    g, A, ix, rows, qs = small
    ids, dist = _same(oracle, A, ix, qs, 40, 12)
    assert (ids[:, 12:] == -1).all() and np.isinf(dist[:, 12:]).all()
    qd = torch.from_numpy(qs).cuda()
    di, dd = ix.search(qd, 10, 64)
    hi, hd = ix.search(qs, 10, 64)
    assert np.array_equal(di.cpu().numpy(), hi) and np.array_equal(dd.cpu().numpy(), hd)


def test_parallel_build_large_batch(ctx, oracle):
    """A graph from the parallel link lanes; a batch larger than the resident warps."""
    import pion_b200
    g, rows, qs = _graph(40000, 256, seed=11, threads=8, nq=5000)
    A = g.arrays()
    ix = pion_b200.HNSWIndex(ctx, g)
    for ef in (64, 200):
        _same(oracle, A, ix, qs, 10, ef)


def test_l2_metric_and_deleted_nodes(ctx, oracle):
    import pion_b200
    g, rows, qs = _graph(5000, 32, seed=5, metric="l2")
    A = dict(g.arrays())
    dele = np.zeros((A["num_nodes"] + 7) // 8, np.uint8)
    gone = np.arange(7, A["num_nodes"], 13)
    gone = gone[gone != A["entry_point"]]
    np.bitwise_or.at(dele, gone >> 3, (1 << (gone & 7)).astype(np.uint8))
    A["deleted"] = dele
    ix = pion_b200.HNSWIndex(ctx, A)
    ids, _ = _same(oracle, A, ix, qs * 3.0, 10, 64)
    assert not np.isin(ids, gone).any()


def test_recall_smoke(ctx, oracle):
    """The reference's recall smoke test at dim 1536 (tests/test_vector_recall_smoke.py):
    150 planted clusters of 10 vectors, 60 queries near cluster centres, k = 10; recall
    against exact cosine top-10 >= 0.90."""
    import pion_b200
    rng = np.random.Generator(np.random.PCG64(150))
    centres = rng.standard_normal((150, 1536)).astype(np.float32)
    rows = (np.repeat(centres, 10, axis=0) +
            0.05 * rng.standard_normal((1500, 1536)).astype(np.float32))
    pick = rng.choice(150, 60, replace=False)
    qs = centres[pick] + 0.05 * rng.standard_normal((60, 1536)).astype(np.float32)
    g = pion_b200.HNSWGraph(rows, M=16, ef_construction=200, threads=1)
    ix = pion_b200.HNSWIndex(ctx, g)
    ids, dist = _same(oracle, g.arrays(), ix, qs, 10, 64)
    rn = rows / np.linalg.norm(rows, axis=1, keepdims=True)
    qn = qs / np.linalg.norm(qs, axis=1, keepdims=True)
    truth = np.argsort(-(qn @ rn.T), axis=1, kind="stable")[:, :10]
    recall = np.mean([len(set(ids[i]) & set(truth[i])) / 10 for i in range(60)])
    assert recall >= 0.90


def test_register_rejects_bad_layouts(ctx, small):
    import pion_b200
    g, A, ix, rows, qs = small
    bad = dict(A)
    l0 = A["l0_slots"].copy()
    l0[5, 1] = A["num_nodes"] + 3
    bad["l0_slots"] = l0
    with pytest.raises(pion_b200.PionError):
        pion_b200.HNSWIndex(ctx, bad)
    bad = dict(A)
    bad["dim"] = 768
    with pytest.raises(pion_b200.PionError):
        pion_b200.HNSWIndex(ctx, bad)
    with pytest.raises(pion_b200.PionError):
        ix.search(qs, 10, 2000)


def test_reference_beam_symbol(oracle, small):
    """pion_v_beam_1536 (the engine's own symbol, src/vector/vector_abi.mojo:31-36) with a
    BeamView1536 seeded the way search_fp32_scored seeds it (src/vector/hnsw.mojo:
    4351-4367: one pool entry for the start node, marked visited at the current epoch):
    the pool it leaves equals the restated beam_search_1536_ref's entry for entry."""
    import ctypes

    import pion_b200
    from pion_b200 import _lib
    g, A, ix, rows, qs = small
    lib = pion_b200.load()
    codes = oracle.hnsw_query_codes(A, qs[:6])
    comp = A["compact_buffer"]
    n = A["num_nodes"]
    rng = np.random.Generator(np.random.PCG64(4))
    for t in range(6):
        for ef in (10, 64, 200):
            start = int(A["entry_point"]) if t % 2 == 0 else int(rng.integers(n))
            qc = np.ascontiguousarray(codes[t])
            v = comp[A["node_slot"][start], 8:8 + 1536].astype(np.int32)
            d0 = np.float32(((v - qc.astype(np.int32)) ** 2).sum())
            qn = np.float32((qc.astype(np.int32) ** 2).sum())
            entries = np.zeros(ef, dtype=[("d", "<f4"), ("id", "<u4")])
            entries[0] = (d0, start)
            pool = _lib.LinearPool(entries.ctypes.data, ef, 1, 0, ef)
            visited = np.zeros(n, np.uint16)
            visited[start] = 7
            view = _lib.BeamView1536(ctypes.pointer(pool), ef, float(qn), 0.0, qc.ctypes.data,
                                     A["l0_compact"].ctypes.data, A["l0_slots"].ctypes.data, n,
                                     None, visited.ctypes.data, 7, comp.ctypes.data,
                                     A["compact_stride"], A["compact_hdr"], None)
            assert lib.pion_v_beam_1536(ctypes.byref(view)) == 0
            od, oi = oracle.hnsw_beam_pool(A, qc, qn, ef, [d0], [start], 0)
            assert pool.size == len(od) and pool.cursor == pool.size
            got = entries[:pool.size]
            assert np.array_equal(got["id"], oi)
            assert np.array_equal(got["d"].view(np.uint32), od.view(np.uint32))
    assert lib.pion_v_quant_beam_1536(None) == -1
    assert lib.pion_v_b200_beam_forget(None) == 0


def test_beam_symbol_sees_a_new_graph_at_the_same_addresses(oracle, small):
    """The device copy pion_v_beam_1536 keeps is keyed by the view's host pointers and
    sizes and by a fingerprint of sampled rows: another graph written into the same
    buffers is served as itself, without pion_v_b200_beam_forget."""
    import ctypes

    import pion_b200
    from pion_b200 import _lib
    _, A, _, _, qs = small
    B = _graph(6000, 64, seed=9)[0].arrays()
    assert B["num_nodes"] == A["num_nodes"] and B["compact_stride"] == A["compact_stride"]
    lib = pion_b200.load()
    bufs = {x: np.array(A[x], copy=True) for x in ("l0_compact", "l0_slots", "compact_buffer")}
    n = A["num_nodes"]
    for G in (A, B, A):
        for x in bufs:
            np.copyto(bufs[x], G[x])
        qc = np.ascontiguousarray(oracle.hnsw_query_codes(G, qs[:1])[0])
        start, ef = int(G["entry_point"]), 64
        v = G["compact_buffer"][G["node_slot"][start], 8:8 + 1536].astype(np.int32)
        d0 = np.float32(((v - qc.astype(np.int32)) ** 2).sum())
        qn = np.float32((qc.astype(np.int32) ** 2).sum())
        entries = np.zeros(ef, dtype=[("d", "<f4"), ("id", "<u4")])
        entries[0] = (d0, start)
        pool = _lib.LinearPool(entries.ctypes.data, ef, 1, 0, ef)
        visited = np.zeros(n, np.uint16)
        view = _lib.BeamView1536(ctypes.pointer(pool), ef, float(qn), 0.0, qc.ctypes.data,
                                 bufs["l0_compact"].ctypes.data, bufs["l0_slots"].ctypes.data,
                                 n, None, visited.ctypes.data, 7,
                                 bufs["compact_buffer"].ctypes.data, G["compact_stride"],
                                 G["compact_hdr"], None)
        assert lib.pion_v_beam_1536(ctypes.byref(view)) == 0
        od, oi = oracle.hnsw_beam_pool(G, qc, qn, ef, [d0], [start], 0)
        got = entries[:pool.size]
        assert np.array_equal(got["id"], oi)
        assert np.array_equal(got["d"].view(np.uint32), od.view(np.uint32))
    assert lib.pion_v_b200_beam_forget(None) == 0


def test_metric_scores(oracle, small, ctx):
    """metric_scores on the GPU == the restatement, bit for bit (COSINE: 1 - cos from the
    dequantised codes), and close to the exact fp32 cosine distance of the rows."""
    import pion_b200
    g, A, ix, rows, qs = small
    ids, dist = ix.search(qs, 10, 64)
    ids[3, 4] = -1                      # no node: keeps its score
    ids[5, 0] = A["num_nodes"] + 10
    got = ix.metric_scores(qs, ids, dist.copy())
    want = oracle.hnsw_metric_scores(A, qs, ids, dist)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert got[3, 4] == dist[3, 4] and got[5, 0] == dist[5, 0]
    rn = rows / np.linalg.norm(rows, axis=1, keepdims=True)
    qn = qs / np.linalg.norm(qs, axis=1, keepdims=True)
    ok = (ids >= 0) & (ids < A["num_nodes"])
    exact = 1.0 - np.einsum("qd,qkd->qk", qn, rn[np.where(ok, ids, 0)])
    assert np.abs(got - exact)[ok].max() < 0.02
    # L2 graph: squared L2 units, no halving
    g2, rows2, qs2 = _graph(3000, 16, seed=9, metric="l2", nq=16)
    ix2 = pion_b200.HNSWIndex(ctx, g2)
    i2, d2 = ix2.search(qs2 * 2.0, 10, 32)
    got2 = ix2.metric_scores(qs2 * 2.0, i2, d2.copy())
    want2 = oracle.hnsw_metric_scores(g2.arrays(), qs2 * 2.0, i2, d2)
    assert np.array_equal(got2.view(np.uint32), want2.view(np.uint32))


def test_beam_batch_matches_oracle(oracle, small):
    """pion_v_b200_hnsw_beam_batch over the registered graph: every query's pool, seeded
    as search_fp32_scored seeds it (the start node), comes back equal to the restated
    beam_search_1536_ref's entry for entry; pools with several seeded entries, expanded
    entries and a cursor too."""
    g, A, ix, rows, qs = small
    nq = 24
    codes = oracle.hnsw_query_codes(A, qs[:nq])
    comp = A["compact_buffer"]
    n = A["num_nodes"]
    rng = np.random.Generator(np.random.PCG64(12))
    qn = (codes.astype(np.int32) ** 2).sum(1).astype(np.float32)
    for ef in (16, 100):
        pools = np.zeros((nq, ef), dtype=[("d", "<f4"), ("id", "<u4")])
        sizes = np.zeros(nq, np.int32)
        cursors = np.zeros(nq, np.int32)
        seeds = []
        for t in range(nq):
            m = 1 if t % 3 else 3
            start = rng.choice(n, m, replace=False)
            d0 = []
            for s_ in start:
                v = comp[A["node_slot"][s_], 8:8 + 1536].astype(np.int32)
                d0.append(np.float32(((v - codes[t].astype(np.int32)) ** 2).sum()))
            order = np.argsort(np.array(d0), kind="stable")
            ds_, ids_ = np.array(d0, np.float32)[order], start[order].astype(np.uint32)
            pools["d"][t, :m] = ds_
            pools["id"][t, :m] = ids_
            sizes[t] = m
            seeds.append((ds_, ids_))
        ix.beam_batch(codes, qn, pools, sizes, cursors)
        for t in range(nq):
            od, oi = oracle.hnsw_beam_pool(A, codes[t], qn[t], ef, seeds[t][0], seeds[t][1], 0)
            assert sizes[t] == len(od)
            assert np.array_equal(pools["id"][t, :sizes[t]], oi)
            assert np.array_equal(pools["d"][t, :sizes[t]].view(np.uint32), od.view(np.uint32))


def test_index_file_serves_on_gpu(ctx, oracle, small, tmp_path):
    """A graph written as the reference's index file (pion.hnsw.0) and read back serves on
    the GPU with the same pools as the graph it came from."""
    import pion_b200
    g, A, ix, rows, qs = small
    p = str(tmp_path / "pion.hnsw.0")
    g.save(p)
    G = pion_b200.HNSWGraph.load(p)
    gix = pion_b200.HNSWIndex(ctx, G)
    i0, d0 = ix.search(qs, 10, 64)
    i1, d1 = gix.search(qs, 10, 64)
    assert np.array_equal(i0, i1) and np.array_equal(d0.view(np.uint32), d1.view(np.uint32))
    _same(oracle, G.arrays(), gix, qs, 10, 32)


def test_visited_words_cleared_between_queries(oracle, small, monkeypatch):
    """Each warp zeroes only the bitmap words its query touched; with a touched-word list
    too small for the query it zeroes the whole bitmap.  Both leave the bitmaps clean:
    many queries per warp, either way, give the oracle's pools."""
    g, A, ix, rows, qs = small
    many = np.concatenate([qs] * 40)  # more queries than resident warps
    monkeypatch.setenv("PION_B200_TOUCH_CAP", "32")
    _same(oracle, A, ix, many, 10, 256)
    monkeypatch.delenv("PION_B200_TOUCH_CAP")
    _same(oracle, A, ix, many, 10, 64)
    _same(oracle, A, ix, qs, 10, 1024)


@pytest.mark.parametrize("metric,M,efc,n", [("cosine", 16, 100, 20000), ("l2", 8, 64, 12000),
                                            ("cosine", 16, 200, 60000)])
def test_gpu_planned_build_equals_host_batched_build(ctx, metric, M, efc, n):
    """pion_v_b200_hnsw_build_gpu plans every batch of >= 64 nodes on the GPU (greedy
    descent, _search_layer_mt, _prune_neighbors) and links on the host: the graph must be
    the host batched build's, array for array."""
    import pion_b200
    rows, _ = mixture_np(n, 1536, 64, seed=n + M, n_queries=0)
    host = pion_b200.HNSWGraph(rows, M=M, ef_construction=efc, metric=metric, batch=1024,
                               threads=8)
    gpu = pion_b200.HNSWGraph(rows, M=M, ef_construction=efc, metric=metric, batch=1024,
                              threads=8, gpu=ctx)
    st = gpu.stats()
    assert st["gpu_planned"] > n // 2, st
    A, B = host.arrays(), gpu.arrays()
    for name in ("compact_buffer", "l0_compact", "l0_slots", "node_slot", "node_ids",
                 "node_level", "upper_offset", "upper_links"):
        assert np.array_equal(A[name], B[name]), name
    for name in ("entry_point", "max_level", "global_min", "global_max"):
        assert A[name] == B[name], name
