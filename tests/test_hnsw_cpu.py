"""The host HNSW builder (pion_v_b200_hnsw_build, CPU code in the library) and the
oracle's search, on CPU.  The builder restates the reference's FT.OPTIMIZE build
(src/vector/hnsw.mojo:2540-2620); these tests check the structure it hands to the
beam: the compact layout of compact_vectors / _build_l0_slots (:2761-2990), list
capacities, the level formula of _level_of (:563-576), and reachability after
_repair_l0 (:2345-2536)."""
import math

import numpy as np
import pytest

from pion_b200.workloads import mixture_np


def _level_of(i, M):
    """_level_of restated in Python (SplitMix64, ml = 1/ln(M), cap 6)."""
    mask = (1 << 64) - 1
    z = (0x50494F4E + (i + 1) * 0x9E3779B97F4A7C15) & mask
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & mask
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & mask
    z = z ^ (z >> 31)
    r = np.float32((z >> 11) * (1.0 / 9007199254740992.0))
    if r <= 0:
        r = np.float32(1e-7)
    ml = np.float32(1.0) / np.float32(math.log(np.float32(M)))
    return min(int(-np.log(r) * ml), 6)


@pytest.fixture(scope="module")
def built():
    import pion_b200
    rows, qs = mixture_np(3000, 1536, 32, seed=17, n_queries=40)
    g = pion_b200.HNSWGraph(rows, M=8, ef_construction=64, threads=1)
    return g, g.arrays(), rows, qs


def test_layout_structure(built):
    g, A, rows, qs = built
    n, M = A["num_nodes"], A["M"]
    assert n == 3000 and A["dim"] == 1536 and A["compact_stride"] == 1600
    assert A["compact_hdr"] == 8
    slots = A["node_slot"].astype(np.int64)
    assert np.array_equal(np.sort(slots), np.arange(n))          # a permutation
    assert slots[A["entry_point"]] == 0                           # BFS starts at the entry
    cnt = A["l0_compact"][:, 0]
    assert cnt.max() <= 2 * M and (A["l0_slots"][:, 0] == cnt).all()
    for i in range(0, n, 97):
        nb = A["l0_compact"][i, 1:1 + cnt[i]]
        assert (nb < n).all()
        assert np.array_equal(A["l0_slots"][i, 1:1 + cnt[i]], A["node_slot"][nb])
    lv = A["node_level"]
    assert lv[A["entry_point"]] == A["max_level"] == lv.max()
    assert int(np.argmax(lv == lv.max())) == A["entry_point"]    # first node of the top level
    for i in range(0, n, 211):
        assert lv[i] == _level_of(i, M)
    off, up = A["upper_offset"], A["upper_links"]
    assert ((off >= 0) == (lv > 0)).all()
    assert up[:, 0].max() <= M


def test_slot_headers_and_codes(built):
    g, A, rows, qs = built
    comp = A["compact_buffer"]
    gmin, gmax = np.float32(A["global_min"]), np.float32(A["global_max"])
    rn = rows / np.linalg.norm(rows, axis=1, keepdims=True)
    # calibration: mean +- 8 sigma of the (normalised) rows
    assert abs(gmax - (rn.mean() + 8 * rn.std())) < 1e-4
    assert abs(gmin - (rn.mean() - 8 * rn.std())) < 1e-4
    rng_ = np.float32(gmax - gmin)
    for i in range(0, A["num_nodes"], 101):
        s = A["node_slot"][i]
        codes = comp[s, 8:8 + 1536].astype(np.int32)
        hdr = comp[s, :8].view(np.float32)
        assert hdr[0] == np.float32((codes * codes).sum())
        assert hdr[1] == np.float32((codes[:256] * codes[:256]).sum())
        # stored code = trunc(clamp((x - gmin) / range, 0, 1) * 254) - 127, allowing
        # one step where float normalisation rounding lands on a boundary
        x = rn[i].astype(np.float32)
        want = (np.clip((x - gmin) / rng_, 0, 1) * np.float32(254)).astype(np.int32) - 127
        assert np.abs(codes - want).max() <= 1
        assert (codes != want).mean() < 0.01


def test_level0_reachable_from_entry(built):
    g, A, rows, qs = built
    n = A["num_nodes"]
    seen = np.zeros(n, bool)
    seen[A["entry_point"]] = True
    frontier = [A["entry_point"]]
    l0 = A["l0_compact"]
    while frontier:
        nxt = []
        for x in frontier:
            for nb in l0[x, 1:1 + l0[x, 0]]:
                if not seen[nb]:
                    seen[nb] = True
                    nxt.append(nb)
        frontier = nxt
    assert seen.all()


def test_single_lane_build_is_deterministic(built):
    import pion_b200
    g, A, rows, qs = built
    g2 = pion_b200.HNSWGraph(rows, M=8, ef_construction=64, threads=1)
    B = g2.arrays()
    for key in ("compact_buffer", "l0_compact", "l0_slots", "upper_links", "node_slot"):
        assert np.array_equal(A[key], B[key]), key


def test_oracle_search_recall_and_order(oracle, built):
    g, A, rows, qs = built
    ids, dist, st = oracle.hnsw_search(A, qs, 10, 64)
    assert (np.diff(dist, axis=1) >= 0).all()
    assert st["expansions"] >= 64 * len(qs)
    rn = rows / np.linalg.norm(rows, axis=1, keepdims=True)
    qn = qs / np.linalg.norm(qs, axis=1, keepdims=True)
    truth = np.argsort(-(qn @ rn.T), axis=1)[:, :10]
    recall = np.mean([len(set(ids[i]) & set(truth[i])) / 10 for i in range(len(qs))])
    assert recall >= 0.6
    # the pool distances are exact squared L2 in code space
    codes = oracle.hnsw_query_codes(A, qs)
    comp = A["compact_buffer"]
    for t in range(0, len(qs), 7):
        v = comp[A["node_slot"][ids[t]], 8:8 + 1536].astype(np.int32)
        l2 = ((v - codes[t].astype(np.int32)) ** 2).sum(axis=1)
        assert np.array_equal(l2.astype(np.float32), dist[t])


def test_build_rejects_bad_arguments():
    import pion_b200
    with pytest.raises(pion_b200.PionError):
        pion_b200.HNSWGraph(np.zeros((10, 1536), np.float32), M=40)


KEYS = ("compact_buffer", "l0_compact", "l0_slots", "upper_links", "node_slot", "node_level")


def test_batched_build_of_one_is_the_one_lane_build(built):
    """Batched insertion with batches of one node is the one-lane build, array for array
    (the search half of an insertion never reads what its own links change)."""
    import pion_b200
    g, A, rows, qs = built
    gb = pion_b200.HNSWGraph(rows, M=8, ef_construction=64, threads=4, batch=1)
    B = gb.arrays()  # views of gb's buffers: gb stays alive while they are read
    for key in KEYS:
        assert np.array_equal(A[key], B[key]), key


def test_batched_build_is_deterministic_and_sound(oracle, built):
    """Batches of up to 128 nodes planned on 1 or 3 threads give the same graph, with the
    structure the beam needs and the recall of the one-lane build."""
    import pion_b200
    g, A, rows, qs = built
    g1 = pion_b200.HNSWGraph(rows, M=8, ef_construction=64, threads=1, batch=128)
    g3 = pion_b200.HNSWGraph(rows, M=8, ef_construction=64, threads=3, batch=128)
    B, C = g1.arrays(), g3.arrays()
    for key in KEYS:
        assert np.array_equal(B[key], C[key]), key
    assert g1.stats()["lanes"] < -1  # the batch count
    n, M = B["num_nodes"], B["M"]
    cnt = B["l0_compact"][:, 0]
    assert cnt.max() <= 2 * M and (cnt > 0).all()
    for i in range(n):  # no self links, every neighbour a node
        nb = B["l0_compact"][i, 1:1 + cnt[i]]
        assert (nb < n).all() and (nb != i).all()
    seen = np.zeros(n, bool)
    seen[B["entry_point"]] = True
    frontier = [B["entry_point"]]
    while frontier:
        nxt = []
        for x in frontier:
            for nb in B["l0_compact"][x, 1:1 + B["l0_compact"][x, 0]]:
                if not seen[nb]:
                    seen[nb] = True
                    nxt.append(nb)
        frontier = nxt
    assert seen.all()
    rn = rows / np.linalg.norm(rows, axis=1, keepdims=True)
    qn = qs / np.linalg.norm(qs, axis=1, keepdims=True)
    truth = np.argsort(-(qn @ rn.T), axis=1)[:, :10]

    def recall(G):
        ids, _, _ = oracle.hnsw_search(G, qs, 10, 64)
        return np.mean([len(set(ids[i]) & set(truth[i])) / 10 for i in range(len(qs))])
    assert recall(B) >= recall(A) - 0.02


def test_ft_search_start_node_composition(oracle, built):
    """FT.SEARCH takes its start node from _upper_level_greedy on the raw query (codes of the
    once-normalised query, src/commands/vector.mojo:4514-4518) and then runs
    search_fp32_scored from it, whose beam quantises the twice-normalised query.  The two
    greedy code sets differ only where the second normalisation moves a value across a
    rounding boundary, so the composition answers as the direct search does here, query
    for query."""
    g, A, rows, qs = built
    i0, d0, s0 = oracle.hnsw_search(A, qs, 10, 32)
    i1, d1, s1 = oracle.hnsw_search(A, qs, 10, 32, ft=True)
    same = (i0 == i1).all(1) & (d0.view(np.uint32) == d1.view(np.uint32)).all(1)
    assert same.all(), np.nonzero(~same)[0]
    assert s1["expansions"] > 0


def test_rescore_knn_sorts_like_the_reference():
    """rescore_knn's re-sort is _rescore_knn's insertion sort (src/commands/vector.mojo:
    1100-1105): ascending, equal scores keep their order; an index with no metric source
    leaves both arrays."""
    import pion_b200

    class Fake:
        def __init__(self, new, ok=True):
            self.new, self.ok = new, ok

        def metric_scores(self, q, ids, scores, ctx=None):
            if not self.ok:
                return False
            scores[...] = self.new
            return True

    gen = np.random.default_rng(4)
    ids = np.arange(40, dtype=np.int32).reshape(4, 10)
    new = gen.integers(0, 5, (4, 10)).astype(np.float32)  # many ties
    got_i, got_s = pion_b200.rescore_knn(Fake(new), None, ids.copy(), np.zeros((4, 10), np.float32))
    for t in range(4):
        si, ss = list(ids[t]), list(new[t])
        for a in range(1, 10):
            b = a
            while b > 0 and ss[b] < ss[b - 1]:
                ss[b], ss[b - 1] = ss[b - 1], ss[b]
                si[b], si[b - 1] = si[b - 1], si[b]
                b -= 1
        assert list(got_i[t]) == si and list(got_s[t]) == ss
    keep_i, keep_s = ids.copy(), new.copy()
    pion_b200.rescore_knn(Fake(None, ok=False), None, keep_i, keep_s)
    assert np.array_equal(keep_i, ids) and np.array_equal(keep_s, new)


def test_rescore_knn_nan_rows_and_types():
    """A NaN blocks the insertion sort where `<` fails against it, exactly as in the
    reference's loop; device tensors are refused (host arrays only)."""
    import pion_b200

    class Fake:
        def __init__(self, new):
            self.new = new

        def metric_scores(self, q, ids, scores, ctx=None):
            scores[...] = self.new
            return True

    new = np.array([[3.0, np.nan, 1.0, 0.5, 2.0],
                    [2.0, 1.0, 3.0, 0.0, 1.0]], np.float32)
    ids = np.arange(10, dtype=np.int32).reshape(2, 5)
    got_i, got_s = pion_b200.rescore_knn(Fake(new), None, ids.copy(), np.zeros_like(new))
    for t in range(2):
        si, ss = list(ids[t]), list(new[t])
        for a in range(1, 5):
            b = a
            while b > 0 and ss[b] < ss[b - 1]:
                ss[b], ss[b - 1] = ss[b - 1], ss[b]
                si[b], si[b - 1] = si[b - 1], si[b]
                b -= 1
        assert list(got_i[t]) == si
        assert np.array_equal(got_s[t], np.array(ss, np.float32), equal_nan=True)
    import torch
    with pytest.raises(TypeError):
        pion_b200.rescore_knn(Fake(new), None, torch.from_numpy(ids), np.zeros_like(new))
