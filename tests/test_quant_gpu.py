"""The block-quantised HNSW search on the GPU against the oracle, bit for bit: the
block-quant branches of search_fp32_scored (src/vector/hnsw.mojo:4136-4330) for PolarQuant
INT4, NanoQuant INT2 and TurboQuant INT3 + QJL, the beam over MinHeap / MaxHeap
(src/vector/reference/quant_beams_1536.mojo:20-81, src/common/heap.mojo) and the FP32
rerank tail (hnsw.mojo:4052-4134).  Covers both metrics, ef below / equal to / above k,
ef = 1, no rerank rows, deleted nodes, candidate heaps that outgrow their first-pass
room (the re-run launch), several queries per warp, device memory, and a graph served from
the reference's index file in a block format."""
import numpy as np
import pytest

from pion_b200.workloads import mixture_np

pytestmark = pytest.mark.gpu

KINDS = ["polar", "nano", "turbo"]


@pytest.fixture(scope="module")
def graphs():
    import pion_b200
    out = {}
    for metric, seed in (("cosine", 51), ("l2", 53)):
        rows, qs = mixture_np(5000, 1536, 48, seed=seed, n_queries=96)
        g = pion_b200.HNSWGraph(rows, M=8, ef_construction=48, metric=metric, threads=8)
        out[metric] = (g, g.arrays(), rows, qs)
    return out


def _same(got, want):
    gi, gs, gn = got
    wi, ws, wn = want
    assert np.array_equal(np.asarray(gn), wn)
    assert np.array_equal(np.asarray(gi), wi)
    assert np.array_equal(np.asarray(gs).view(np.uint32), ws.view(np.uint32))


@pytest.mark.parametrize("metric", ["cosine", "l2"])
@pytest.mark.parametrize("kind", KINDS)
def test_quant_search_matches_oracle(ctx, oracle, graphs, kind, metric):
    import pion_b200
    g, A, rows, qs = graphs[metric]
    qz = pion_b200.HNSWQuant(g, rows, kind)
    Q = qz.arrays()
    ix = pion_b200.HNSWQuantIndex(ctx, g, qz)
    for k, ef in ((10, 64), (10, 10), (1, 1), (25, 16), (10, 200)):
        _same(ix.search(qs, k, ef), oracle.quant_search(A, Q, qs, k, ef))
    st = ix.last_stats()
    assert st["evals"] > 0 and st["expansions"] > 0 and st["reruns"] == 0
    ix.free()


@pytest.mark.parametrize("kind", KINDS)
def test_quant_search_without_rerank(ctx, oracle, graphs, kind):
    import pion_b200
    g, A, rows, qs = graphs["cosine"]
    qz = pion_b200.HNSWQuant(g, rows, kind)
    Q = dict(qz.arrays())
    ix = pion_b200.HNSWQuantIndex(ctx, g, qz, rerank=False)
    Q["rerank"] = None
    _same(ix.search(qs, 10, 48), oracle.quant_search(A, Q, qs, 10, 48))
    ix.free()


@pytest.mark.parametrize("kind", KINDS)
def test_quant_search_deleted_nodes(ctx, oracle, graphs, kind):
    """Deleted nodes are skipped by the beam (and by NanoQuant's greedy), never marked
    visited; the graph is registered from its arrays with a deletion bitmap."""
    import pion_b200
    g, A, rows, qs = graphs["l2"]
    n = A["num_nodes"]
    gen = np.random.Generator(np.random.PCG64(77))
    dead = gen.choice(n, n // 12, replace=False)
    bits = np.zeros((n + 7) // 8, np.uint8)
    for i in dead:
        bits[i >> 3] |= np.uint8(1 << (i & 7))
    A2 = dict(A)
    A2["deleted"] = bits
    qz = pion_b200.HNSWQuant(g, rows, kind)
    Q = qz.arrays()
    ix = pion_b200.HNSWQuantIndex(ctx, A2, Q)
    _same(ix.search(qs, 10, 40), oracle.quant_search(A2, Q, qs, 10, 40))
    ix.free()


def test_quant_search_heap_rerun(ctx, oracle, graphs, monkeypatch):
    """With the first pass's candidate heap capped at 40 entries every query outgrows it
    and is re-run with room for every node; the answers do not change."""
    import pion_b200
    g, A, rows, qs = graphs["cosine"]
    qz = pion_b200.HNSWQuant(g, rows, "turbo")
    Q = qz.arrays()
    ix = pion_b200.HNSWQuantIndex(ctx, g, qz)
    monkeypatch.setenv("PION_B200_QUANT_HEAP_CAP", "40")
    got = ix.search(qs, 10, 64)
    st = ix.last_stats()
    monkeypatch.delenv("PION_B200_QUANT_HEAP_CAP")
    assert st["reruns"] > 0
    _same(got, oracle.quant_search(A, Q, qs, 10, 64))
    ix.free()


def test_quant_search_many_queries_per_warp(ctx, oracle, graphs):
    """More queries than resident warps: each warp runs several in turn."""
    import pion_b200
    g, A, rows, _ = graphs["cosine"]
    _, qs = mixture_np(10, 1536, 48, seed=51, n_queries=6000)
    qz = pion_b200.HNSWQuant(g, rows, "polar")
    Q = qz.arrays()
    ix = pion_b200.HNSWQuantIndex(ctx, g, qz)
    _same(ix.search(qs, 10, 24), oracle.quant_search(A, Q, qs, 10, 24))
    ix.free()


def test_quant_search_device_memory(ctx, oracle, graphs):
    import torch

    import pion_b200
    g, A, rows, qs = graphs["l2"]
    qz = pion_b200.HNSWQuant(g, rows, "nano")
    Q = qz.arrays()
    ix = pion_b200.HNSWQuantIndex(ctx, g, qz)
    ids, sc, found = ix.search(torch.from_numpy(qs).cuda(), 10, 32)
    assert ids.is_cuda and sc.is_cuda and found.is_cuda
    _same((ids.cpu().numpy(), sc.cpu().numpy(), found.cpu().numpy()),
          oracle.quant_search(A, Q, qs, 10, 32))
    ix.free()


def test_quant_search_refuses(ctx, graphs):
    import pion_b200
    g, A, rows, qs = graphs["cosine"]
    qz = pion_b200.HNSWQuant(g, rows, "polar")
    ix = pion_b200.HNSWQuantIndex(ctx, g, qz)
    for ef in (0, 1025):
        with pytest.raises(pion_b200.PionError) as e:
            ix.search(qs[:2], 10, ef)
        assert e.value.code == -3
    hx = pion_b200.HNSWIndex(ctx, g)
    with pytest.raises(pion_b200.PionError):  # not a quantised index
        pion_b200.HNSWQuantIndex.search(hx, qs[:2], 10, 10)
    Q = dict(qz.arrays())
    Q["stride"] = 100
    with pytest.raises(pion_b200.PionError):
        pion_b200.HNSWQuantIndex(ctx, g, Q)
    hx.free()
    ix.free()


@pytest.mark.parametrize("kind", ["nano", "turbo"])
def test_quant_search_from_index_file(ctx, oracle, graphs, kind, tmp_path):
    """A block-quantised index file (pion.hnsw.0 with its rerank and QJL sections) loads
    and serves on the GPU with the oracle's answers."""
    import pion_b200
    g, A, rows, qs = graphs["cosine"]
    qz = pion_b200.HNSWQuant(g, rows, kind)
    p = str(tmp_path / "pion.hnsw.0")
    g.save(p, quant=qz)
    G2, q2 = pion_b200.HNSWGraph.load_quant(p)
    ix = pion_b200.HNSWQuantIndex(ctx, G2, q2)
    _same(ix.search(qs, 10, 64), oracle.quant_search(G2.arrays(), q2.arrays(), qs, 10, 64))
    ix.free()


NODE = np.dtype([("d", "<f4"), ("pad", "<i4"), ("id", "<i8")])


@pytest.mark.parametrize("kind,cap", [("polar", None), ("nano", None), ("turbo", None),
                                      ("turbo", 12)])
def test_quant_beam_symbol(ctx, oracle, graphs, kind, cap):
    """The reference's per-query symbol pion_v_quant_beam_1536 on a QuantBeamView1536
    seeded as search_fp32_scored seeds it (the start node in both heaps, the List reserves
    of ef + 32): the heaps come back array for array as the oracle's beam leaves them, the
    candidates cut at the List's capacity."""
    import ctypes

    import pion_b200
    from pion_b200 import _lib
    g, A, rows, qs = graphs["cosine"]
    qz = pion_b200.HNSWQuant(g, rows, kind)
    Q = qz.arrays()
    comp = Q["compact"].reshape(A["num_nodes"], Q["stride"])
    lib = pion_b200.load()
    n, ef = A["num_nodes"], 48
    visited = np.zeros(n, np.uint16)
    l0c = np.ascontiguousarray(A["l0_compact"])
    l0s = np.ascontiguousarray(A["l0_slots"])
    for t in range(6):
        q = oracle.l2_normalize_rows(qs[t][None])[0]
        qc, qsc, qn = oracle.query_block_int8(q)
        qsig, qres = None, np.float32(0.0)
        if kind == "turbo":
            resid = np.array([q[i] - np.float32(qc[i]) * qsc[i // 32] for i in range(1536)],
                             np.float32)
            qsig, qres = oracle.qjl_signs(resid, Q["qjl_random_signs"])
        start = (int(A["entry_point"]) + 97 * t) % n
        v = comp[A["node_slot"][start]]
        d0 = (qn + np.frombuffer(v[:4].tobytes(), np.float32)[0]) - \
            np.float32(2.0) * np.float32(oracle.quant_dot(kind, qc, qsc, v))
        ccap = cap or ef + 32
        cn = np.zeros(ccap, NODE)
        rn = np.zeros(ef + 32, NODE)
        cn[0] = (d0, 0, start)
        rn[0] = (d0, 0, start)
        minh = _lib.MinHeap(_lib.HeapList(cn.ctypes.data, 1, ccap))
        maxh = _lib.MaxHeap(_lib.HeapList(rn.ctypes.data, 1, ef + 32), float(d0), 0)
        keep = [np.ascontiguousarray(qc), np.ascontiguousarray(qsc)]
        sig = None if qsig is None else np.ascontiguousarray(qsig, np.uint64)
        view = _lib.QuantBeamView1536(
            kind=pion_b200.search.QUANT_KINDS[kind], ef=ef, candidates=ctypes.pointer(minh),
            results=ctypes.pointer(maxh), query_block_int8=keep[0].ctypes.data,
            query_block_scales=keep[1].ctypes.data, query_block_norm=float(qn),
            l0_compact=l0c.ctypes.data, l0_slots=l0s.ctypes.data, num_nodes=n, deleted=None,
            visited=visited.ctypes.data, cur_epoch=1, compact_buffer=comp.ctypes.data,
            compact_stride=Q["stride"], compact_hdr=0, nodes=None,
            qjl_buffer=Q["qjl"].ctypes.data if kind == "turbo" else None,
            qjl_res_norms=Q["qjl_res_norms"].ctypes.data if kind == "turbo" else None,
            qjl_query_signs=None if sig is None else sig.ctypes.data,
            qjl_query_res_norm=float(qres), qjl_lambda=1.0)
        assert lib.pion_v_quant_beam_1536(ctypes.byref(view)) == 0
        want_c, total, want_r, worst = oracle.quant_beam_heaps(
            A, Q, qc, qsc, qn, qsig, qres, ef, [(d0, start)], [(d0, start)], d0, cand_cap=ccap)
        assert minh.data.len == len(want_c) and maxh.data.len == len(want_r)
        got_c = [(np.float32(e["d"]).view(np.uint32), int(e["id"])) for e in cn[:minh.data.len]]
        got_r = [(np.float32(e["d"]).view(np.uint32), int(e["id"])) for e in rn[:maxh.data.len]]
        assert got_c == [(np.float32(d).view(np.uint32), i) for d, i in want_c]
        assert got_r == [(np.float32(d).view(np.uint32), i) for d, i in want_r]
        assert np.float32(maxh.cached_worst) == worst
        if cap is not None:
            assert total > cap  # the whole heap did not fit the List: cut at its capacity
    lib.pion_v_b200_beam_forget(None)


def test_quant_metric_scores(ctx, oracle, graphs):
    """metric_scores on a block-quantised graph reads its FP32 copy (hnsw.mojo:4586-4600):
    bit for bit the oracle's; without the copy the scores stay."""
    import pion_b200
    for metric in ("cosine", "l2"):
        g, A, rows, qs = graphs[metric]
        qz = pion_b200.HNSWQuant(g, rows, "turbo")
        Q = qz.arrays()
        ix = pion_b200.HNSWQuantIndex(ctx, g, qz)
        ids, sc, found = ix.search(qs, 10, 40)
        ids = np.array(ids)
        ids[0, 3] = 999999  # names no node: keeps its score
        got = np.array(sc, np.float32)
        assert ix.metric_scores(qs, ids, got) is True
        want = oracle.metric_scores_f32(A, Q["rerank"], qs, ids, sc)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        assert got[0, 3] == sc[0, 3]
        ix.free()
        bare = pion_b200.HNSWQuantIndex(ctx, g, qz, rerank=False)
        kept = np.array(sc, np.float32)
        assert bare.metric_scores(qs, ids, kept) is False
        assert np.array_equal(kept, sc)
        bare.free()
