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
