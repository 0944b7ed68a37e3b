"""FLAT FP32 cosine (exact_knn under COSINE) on the GPU against the CPU oracle.

Distances are 1 - dot_f32_4chain(q^, row) (src/commands/vector.mojo:1228-1365,
src/vector/fp32_scan.mojo:17-38); the GPU rescoring uses the same operation order, so
the distances must be bit-identical to the oracle's (the parity contract only asks
for 1e-4 relative).  Ids must match after ordering by (distance, id), except among
rows tied at the k-th distance, where the reference's heap decides."""
import os

import numpy as np
import pytest

from pion_b200.workloads import mixture_np

pytestmark = pytest.mark.gpu


def assert_f32_matches(oracle, rows_n, queries, k, ids, dist):
    oi, od = oracle.exact_knn(rows_n, queries, k)
    n = rows_n.shape[0]
    kk = min(k, n)
    for t in range(queries.shape[0]):
        o = np.lexsort((oi[t, :kk], od[t, :kk]))
        ref_i, ref_d = oi[t, :kk][o], od[t, :kk][o]
        assert np.all(np.abs(dist[t, :kk] - ref_d) <= 1e-4 * (1 + np.abs(ref_d))), f"query {t}"
        assert np.array_equal(dist[t, :kk].view(np.uint32), ref_d.view(np.uint32)), f"query {t}"
        if not np.array_equal(ids[t, :kk], ref_i):
            # only rows tied at the k-th distance may differ
            kth = ref_d[-1]
            ours = dict(zip(ids[t, :kk].tolist(), dist[t, :kk].tolist()))
            theirs = dict(zip(ref_i.tolist(), ref_d.tolist()))
            for i in set(ours) ^ set(theirs):
                assert ours.get(i, theirs.get(i)) == kth, f"query {t}: id {i}"
        assert (ids[t, kk:] == -1).all() and np.isposinf(dist[t, kk:]).all()
        assert np.all(np.diff(dist[t, :kk]) >= 0)


@pytest.fixture
def env_guard():
    saved = {v: os.environ.get(v) for v in ("PION_B200_F32_PREPASS", "PION_B200_F32_EXACT")}
    yield
    for v, old in saved.items():
        if old is None:
            os.environ.pop(v, None)
        else:
            os.environ[v] = old


def test_l2_normalize_rows_bit_exact(ctx, oracle, rng):
    import pion_b200
    x = rng.standard_normal((2000, 1536)).astype(np.float32)
    x[0] = 0.0
    x[1] *= 1e-20
    x[2] *= 1e20
    for dim in (1536, 37, 4):
        a = pion_b200.l2_normalize_rows(ctx, np.ascontiguousarray(x[:, :dim]))
        b = oracle.l2_normalize_rows(x[:, :dim])
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), dim


@pytest.mark.parametrize("n,dim,nq,k,centres", [
    (100000, 1536, 1000, 10, 256),   # the FLAT FP32 benchmark configuration
    (20000, 1536, 130, 10, 64),
    (5000, 448, 37, 1, 32),
    (3000, 1536, 7, 64, 16),
    (777, 256, 129, 16, 8),
    (50, 1536, 3, 64, 4),
])
def test_flat_f32_knn_matches_oracle(ctx, oracle, n, dim, nq, k, centres):
    import pion_b200
    rows, qs = mixture_np(n, dim, centres, seed=n + k, n_queries=nq)
    qs *= 3.0  # exact_knn normalises the query itself
    ix = pion_b200.FlatF32Index(ctx, rows)
    ids, dist = ix.search(qs, k)
    assert_f32_matches(oracle, oracle.l2_normalize_rows(rows), qs, k, ids, dist)


def test_forced_prepass_and_exact_fallback(ctx, oracle, env_guard):
    import pion_b200
    rows, qs = mixture_np(100000, 1536, 256, seed=0, n_queries=64)
    ix = pion_b200.FlatF32Index(ctx, rows)
    rn = oracle.l2_normalize_rows(rows)
    os.environ["PION_B200_F32_PREPASS"] = "1"
    ids, dist = ix.search(qs, 10)
    assert_f32_matches(oracle, rn, qs, 10, ids, dist)
    os.environ["PION_B200_F32_PREPASS"] = "0"
    os.environ["PION_B200_F32_EXACT"] = "1"
    ids2, dist2 = ix.search(qs, 10)
    assert np.array_equal(ids2, ids) and np.array_equal(dist2, dist)


def test_duplicate_rows_tie_by_id(ctx, oracle):
    import pion_b200
    rows, qs = mixture_np(8000, 256, 16, seed=5, n_queries=4)
    rows[7000] = rows[10]
    rows[7500] = rows[10]
    qs[0] = rows[10]
    ix = pion_b200.FlatF32Index(ctx, rows)
    ids, dist = ix.search(qs, 5)
    assert ids[0, :3].tolist() == [10, 7000, 7500] and dist[0, 0] == dist[0, 1] == dist[0, 2]
    assert_f32_matches(oracle, oracle.l2_normalize_rows(rows), qs, 5, ids, dist)


def test_device_tensors_and_empty_index(ctx, oracle):
    import torch
    import pion_b200
    rows, qs = mixture_np(10000, 1536, 32, seed=8, n_queries=200)
    ix_h = pion_b200.FlatF32Index(ctx, rows)
    ids_h, d_h = ix_h.search(qs, 10)
    ix_d = pion_b200.FlatF32Index(ctx, torch.from_numpy(rows).cuda(), id_base=100)
    ids_d, d_d = ix_d.search(torch.from_numpy(qs).cuda(), 10)
    torch.cuda.synchronize()
    assert np.array_equal(ids_d.cpu().numpy(), ids_h + 100)
    assert np.array_equal(d_d.cpu().numpy(), d_h)
    empty = pion_b200.FlatF32Index(ctx, np.zeros((0, 64), np.float32))
    ids, d = empty.search(np.ones((2, 64), np.float32), 3)
    assert (ids == -1).all() and np.isposinf(d).all()


@pytest.mark.parametrize("cosine", [True, False])
def test_merge_delta_matches_oracle(ctx, oracle, cosine):
    """merge_delta (src/commands/vector.mojo:1368-1456): the graph's results rescored
    exactly from the FP32 rows and merged with the exact scan of the rows ingested since
    the build, identical to the restated composition."""
    import pion_b200
    n, built, nq, kg, k = 6000, 4500, 40, 16, 10
    rows, qs = mixture_np(n, 1536, 32, seed=21, n_queries=nq)
    if not cosine:
        rows = rows * 3.0
        qs = qs * 3.0
    stored = oracle.l2_normalize_rows(rows) if cosine else rows
    ix = pion_b200.FlatF32Index(ctx, rows, normalize=cosine)
    rng = np.random.Generator(np.random.PCG64(6))
    ids = np.full((nq, kg), -1, np.int32)
    for t in range(nq):  # a graph answer: slots below built, some lists short
        m = kg if t % 4 else kg // 2
        ids[t, :m] = rng.choice(built, m, replace=False)
    scores = rng.random((nq, kg)).astype(np.float32)
    ids[3, 2] = built + 7                 # a slot past the graph keeps its score
    want = oracle.merge_delta(stored, built, cosine, qs, ids, scores, k)
    gi, gs = ids.copy(), scores.copy()
    oi, osc = ix.merge_delta(qs, built, gi, gs, k, cosine=cosine)
    assert np.array_equal(gi, want[0]) and np.array_equal(gs.view(np.uint32), want[1].view(np.uint32))
    assert np.array_equal(oi, want[2])
    assert np.array_equal(osc.view(np.uint32), want[3].view(np.uint32))
    # nothing ingested since the build: the rescored graph list alone
    oi2, os2 = ix.merge_delta(qs, n, ids.copy(), scores.copy(), k, cosine=cosine)
    w2 = oracle.merge_delta(stored, n, cosine, qs, ids, scores, k)
    assert np.array_equal(oi2, w2[2]) and np.array_equal(os2, w2[3])


@pytest.mark.parametrize("n,dim,k,centres", [
    (100000, 1536, 10, 256),   # the FLAT FP32 configuration, one query at a time
    (30011, 1536, 64, 64),     # ragged last CTA, the 64-entry lists
    (4099, 512, 33, 16),
    (100, 1536, 10, 4),        # fewer rows than one CTA's rows in flight
    (7, 1536, 10, 2),          # fewer rows than k
])
def test_one_query_stream_matches_oracle(ctx, oracle, n, dim, k, centres):
    """nq = 1 takes the exact HBM stream (4 lanes per row, the 4-chain order restated
    across the group): distances bit-identical, ids as exact_knn's."""
    import pion_b200
    rows, qs = mixture_np(n, dim, centres, seed=n + 3 * k, n_queries=4)
    rows[n // 2] = rows[n // 3]        # duplicate rows: ties broken by id
    qs[1] = rows[n // 3] * 7.0
    ix = pion_b200.FlatF32Index(ctx, rows)
    rn = oracle.l2_normalize_rows(rows)
    for t in range(qs.shape[0]):
        ids, dist = ix.search(qs[t:t + 1] * 2.0, k)
        assert_f32_matches(oracle, rn, qs[t:t + 1] * 2.0, k, ids, dist)
    ix.free()


def test_one_query_stream_equals_tensor_path(ctx, oracle):
    """The stream forced for a whole batch returns what the tensor-core shortlist plus
    certified rescore returns, bit for bit, ids included (both order by (distance, id))."""
    import pion_b200
    rows, qs = mixture_np(60000, 1536, 128, seed=41, n_queries=96)
    ix = pion_b200.FlatF32Index(ctx, rows)
    want_i, want_d = ix.search(qs, 10)
    os.environ["PION_B200_F32_PATH"] = "1"
    try:
        got_i, got_d = ix.search(qs, 10)
    finally:
        os.environ.pop("PION_B200_F32_PATH", None)
    assert np.array_equal(got_i, want_i)
    assert np.array_equal(got_d.view(np.uint32), want_d.view(np.uint32))
    ix.free()
