"""Binary-quantised FLAT with FP32 rerank on the GPU against the oracle's composed
pipeline: sign codes (bit b of word w = x[64w+b] > 0, src/vector/kernels.mojo:1711-1720),
Hamming = popcount of XOR (src/vector/reference/quant_dots.mojo:95-100), the shortlist
of the S smallest distances by (distance, id), then exact cosine rerank with the stable
insertion sort of _exact_rescore (src/commands/vector.mojo:1413-1456).  Integer work and
ids must be bit-exact; scores bit-identical (same 4-chain order)."""
import os

import numpy as np
import pytest

from pion_b200.workloads import mixture_np

pytestmark = pytest.mark.gpu


def check(oracle, rows, qs, S, k, ids, sc):
    rn = oracle.l2_normalize_rows(rows)
    codes = oracle.bq_pack_signs(rn)
    oi, os_, _, _ = oracle.bq_knn(codes, rn, qs, S, k)
    assert np.array_equal(ids, oi.astype(np.int32))
    assert np.array_equal(sc.view(np.uint32), os_.view(np.uint32))


@pytest.mark.parametrize("n,dim,nq,S,k,centres", [
    (200000, 1536, 64, 100, 10, 256),   # three stages: 16 + 240 sample tiles, then the rest
    (20000, 1536, 130, 100, 10, 64),    # two stages
    (3000, 256, 7, 100, 10, 16),        # one stage
    (50, 1536, 3, 100, 10, 4),          # fewer rows than the shortlist
    (20000, 512, 40, 256, 1, 32),
    (20000, 512, 40, 10, 10, 32),
])
def test_bq_rerank_matches_oracle(ctx, oracle, n, dim, nq, S, k, centres):
    import pion_b200
    rows, qs = mixture_np(n, dim, centres, seed=n + S, n_queries=nq)
    ix = pion_b200.BQIndex(ctx, rows)
    ids, sc = ix.search(qs * 2.0, k, shortlist=S)
    check(oracle, rows, qs * 2.0, S, k, ids, sc)


def test_bq_exact_fallback_and_duplicates(ctx, oracle):
    import pion_b200
    rows, qs = mixture_np(30000, 1536, 64, seed=3, n_queries=20)
    rows[20000] = rows[5]    # identical codes and vectors: ties in both stages
    rows[29999] = rows[5]
    qs[0] = rows[5]
    ix = pion_b200.BQIndex(ctx, rows)
    ids, sc = ix.search(qs, 10)
    check(oracle, rows, qs, 100, 10, ids, sc)
    os.environ["PION_B200_BQ_EXACT"] = "1"
    try:
        ids2, sc2 = ix.search(qs, 10)
    finally:
        os.environ.pop("PION_B200_BQ_EXACT", None)
    assert np.array_equal(ids2, ids) and np.array_equal(sc2, sc)
    assert ids[0, :3].tolist() == [5, 20000, 29999]


@pytest.mark.parametrize("n,dim,S,k,centres", [
    (200000, 1536, 100, 10, 256),
    (20000, 512, 256, 1, 32),
    (3000, 1536, 100, 64, 16),
    (50, 1536, 100, 10, 4),          # fewer rows than the shortlist
])
def test_one_query_popcount_stream(ctx, oracle, n, dim, S, k, centres):
    """nq = 1 takes the popcount stream over the packed codes (histogram threshold,
    ties at the S-th distance by row id): shortlist and rerank equal the oracle's."""
    import pion_b200
    rows, qs = mixture_np(n, dim, centres, seed=n + S + 1, n_queries=3)
    ix = pion_b200.BQIndex(ctx, rows)
    for t in range(qs.shape[0]):
        ids, sc = ix.search(qs[t:t + 1], k, shortlist=S)
        check(oracle, rows, qs[t:t + 1], S, k, ids, sc)
    ix.free()


def test_one_query_stream_massive_ties(ctx, oracle):
    """Most rows share one code, so the S-th distance ties across more rows than the
    shared-memory sort holds: the ordered scan takes the first ones by id."""
    import pion_b200
    rows, qs = mixture_np(30000, 1536, 8, seed=12, n_queries=2)
    rows[5:25000] = rows[3]
    rows[25000:25010] *= -1.0
    ix = pion_b200.BQIndex(ctx, rows)
    for t in range(2):
        ids, sc = ix.search(qs[t:t + 1], 10, shortlist=100)
        check(oracle, rows, qs[t:t + 1], 100, 10, ids, sc)
    ids, sc = ix.search(rows[3:4], 10, shortlist=100)
    check(oracle, rows, rows[3:4], 100, 10, ids, sc)
    ix.free()


def test_one_query_stream_equals_tensor_path(ctx, oracle):
    import pion_b200
    rows, qs = mixture_np(60000, 1536, 64, seed=8, n_queries=70)
    ix = pion_b200.BQIndex(ctx, rows)
    want_i, want_s = ix.search(qs, 10)
    os.environ["PION_B200_BQ_PATH"] = "1"
    try:
        got_i, got_s = ix.search(qs, 10)
    finally:
        os.environ.pop("PION_B200_BQ_PATH", None)
    assert np.array_equal(got_i, want_i)
    assert np.array_equal(got_s.view(np.uint32), want_s.view(np.uint32))
    ix.free()


def test_one_query_staged_rerank_equals_spread_rerank(ctx, oracle):
    """The one-query rerank with the shortlist rows bulk-copied into shared memory (and the
    pick by each query's last CTA) equals the spread-rows kernel pair, for one query and
    for many (PION_B200_BQ_PATH=1 sends a batch down the popcount stream too)."""
    import pion_b200
    rows, qs = mixture_np(40000, 1536, 32, seed=31, n_queries=9)
    ix = pion_b200.BQIndex(ctx, rows)
    os.environ["PION_B200_BQ_PATH"] = "1"
    try:
        for S, k in ((100, 10), (256, 64), (7, 7)):
            a = ix.search(qs, k, shortlist=S)
            os.environ["PION_B200_BQ_RERANK"] = "1"
            try:
                b = ix.search(qs, k, shortlist=S)
            finally:
                os.environ.pop("PION_B200_BQ_RERANK", None)
            assert np.array_equal(a[0], b[0])
            assert np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32))
            check(oracle, rows, qs, S, k, a[0], a[1])
    finally:
        os.environ.pop("PION_B200_BQ_PATH", None)
    ix.free()


@pytest.mark.parametrize("n,dim", [(300000, 1536), (5000, 3072), (70001, 128)])
def test_one_query_staged_stream_equals_register_stream(ctx, oracle, n, dim):
    """The one-query first pass through shared memory (bulk copies of 128-row stages,
    ragged last stages) equals the register pass (PION_B200_BQ_STREAM=1) and the oracle."""
    import pion_b200
    rows, qs = mixture_np(n, dim, 64, seed=n + dim, n_queries=3)
    ix = pion_b200.BQIndex(ctx, rows)
    for t in range(qs.shape[0]):
        a = ix.search(qs[t:t + 1], 10, shortlist=100)
        os.environ["PION_B200_BQ_STREAM"] = "1"
        try:
            b = ix.search(qs[t:t + 1], 10, shortlist=100)
        finally:
            os.environ.pop("PION_B200_BQ_STREAM", None)
        assert np.array_equal(a[0], b[0])
        assert np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32))
        if n <= 100000:
            check(oracle, rows, qs[t:t + 1], 100, 10, a[0], a[1])
    ix.free()
