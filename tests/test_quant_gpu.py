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
