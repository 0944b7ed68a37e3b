"""The reference-compatible pion_v_pkm_* symbols on the GPU against the oracle.

Structure of tests/test_vector_differential.mojo:283-351 in the reference (S=1000,
half-dim 448, NQ=8, K=32, seed 146): INT8 scores and top-k / combine / sort results
bit-identical, ids and order included; FP32 scores within 1e-4 (1 + |s|) (here they are
bit-identical too: the same 8-lane summation order)."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def P(a):
    return a.ctypes.data_as(ctypes.c_void_p)


@pytest.fixture(scope="module")
def L():
    from pion_b200 import _lib
    return _lib.load()


def pkm_case():
    rng = np.random.Generator(np.random.PCG64(146))
    S, HALF, NQ = 1000, 448, 8
    d_pad = ((HALF + 63) // 64) * 64
    keys = np.zeros((S, d_pad), np.float32)
    keys[:, :HALF] = rng.uniform(-1, 1, (S, HALF))
    q = np.zeros((NQ, d_pad), np.float32)
    q[:, :HALF] = rng.uniform(-1, 1, (NQ, HALF))
    return keys, q, HALF, rng


def test_pkm_differential(L, oracle):
    keys, q, HALF, rng = pkm_case()
    S, d_pad = keys.shape
    NQ, K = q.shape[0], 32
    a = np.empty((NQ, S), np.float32)
    L.pion_v_pkm_scores_f32(P(keys), S, d_pad, P(q), NQ, P(a))
    b = oracle.pkm_scores_f32(keys, q)
    assert np.all(np.abs(a - b) <= 1e-4 * (1 + np.abs(a)))
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))

    idx = rng.integers(0, S, 64).astype(np.int32)
    r = np.empty(64, np.float32)
    L.pion_v_pkm_rescore_f32(P(keys), d_pad, P(q[0].copy()), P(idx), 64, P(r))
    assert np.array_equal(r.view(np.uint32), oracle.pkm_rescore_f32(keys, q[0], idx).view(np.uint32))

    ki, ks = oracle.pkm_quantize_rows_i8(keys, d=HALF)
    qi, qsc = oracle.pkm_quantize_rows_i8(q, d=HALF)
    si = np.empty((NQ, S), np.float32)
    L.pion_v_pkm_scores_i8(P(ki), S, d_pad, P(ks), P(qi), P(qsc), NQ, P(si))
    ref = oracle.pkm_scores_i8(ki, ks, qi, qsc)
    assert np.array_equal(si.view(np.uint32), ref.view(np.uint32))

    tops = []
    for h in range(2):
        ti = np.empty(K, np.int32)
        tv = np.empty(K, np.float32)
        n = L.pion_v_pkm_topk_max(P(si[h].copy()), S, K, P(ti), P(tv))
        ri, rv = oracle.pkm_topk_max(si[h], K)
        assert n == len(ri) == K
        assert np.array_equal(ti, ri) and np.array_equal(tv.view(np.uint32), rv.view(np.uint32))
        tops.append((ti, tv))
    ci = np.empty(K, np.int32)
    cv = np.empty(K, np.float32)
    n = L.pion_v_pkm_combine_topk(P(tops[0][1]), P(tops[0][0]), K, P(tops[1][1]), P(tops[1][0]),
                                  K, S, K, P(ci), P(cv))
    ri, rv = oracle.pkm_combine_topk(tops[0][1], tops[0][0], tops[1][1], tops[1][0], S, K)
    assert n == len(ri) and np.array_equal(ci, ri) and np.array_equal(cv, rv)

    v0 = rng.uniform(-1, 1, 500).astype(np.float32)
    v0[::7] = v0[0]  # equal values: their order comes from the heapsort itself
    rv, ri = oracle.pkm_sort_desc(v0, np.arange(500, dtype=np.int32))
    v1 = v0.copy()
    i1 = np.arange(500, dtype=np.int32)
    L.pion_v_pkm_sort_desc(P(v1), P(i1), 500)
    assert np.array_equal(v1, rv) and np.array_equal(i1, ri)


@pytest.mark.parametrize("n,k,kind", [
    (1_000_000, 32, "normal"),
    (1_000_000, 100, "ties"),
    (300_000, 256, "normal"),
    (200_000, 16, "ascending"),   # every element is admitted: the replay sees all of them
    (5000, 7, "ties"),
    (3, 10, "normal"),            # n < k
])
def test_topk_max_exact_reference_order(L, oracle, n, k, kind):
    rng = np.random.Generator(np.random.PCG64(n + k))
    if kind == "normal":
        s = rng.standard_normal(n).astype(np.float32)
    elif kind == "ties":
        s = rng.integers(0, 50, n).astype(np.float32)
    else:
        s = np.arange(n, dtype=np.float32)
    kk = min(k, n)
    ti = np.empty(kk, np.int32)
    tv = np.empty(kk, np.float32)
    got = L.pion_v_pkm_topk_max(P(s), n, k, P(ti), P(tv))
    ri, rv = oracle.pkm_topk_max(s, k)
    assert got == kk
    assert np.array_equal(ti, ri) and np.array_equal(tv, rv)


def test_abi_version_and_isa(L):
    assert L.pion_v_abi_version() == 1 and L.pion_v_isa() == 100
