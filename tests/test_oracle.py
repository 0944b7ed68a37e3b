"""The CPU oracle against independent numpy / pure-Python restatements of the same
reference routines, hand-derived known answers, and the reference tests'
invariants.  CPU only."""
import math

import numpy as np
import pytest


# ------------------------------------------------------------------ helpers --

def np_quantize_rows_i8(src: np.ndarray, d: int):
    """Independent numpy restatement of pkm_quantize_rows_i8
    (src/vector/pkm_kernels.mojo:152-191)."""
    x = src[:, :d].astype(np.float32)
    m = np.abs(x).max(axis=1).astype(np.float32) if d else np.zeros(len(x), np.float32)
    scale = (m / np.float32(127.0)).astype(np.float32)
    scale[m == 0] = np.float32(1.0)
    inv = (np.float32(1.0) / scale).astype(np.float32)
    qv = (x * inv[:, None]).astype(np.float32)
    up = np.trunc((qv + np.float32(0.5)).astype(np.float32))
    dn = np.trunc((qv - np.float32(0.5)).astype(np.float32))
    qi = np.where(qv >= 0, up, dn)
    qi = np.clip(qi, -127, 127).astype(np.int8)
    out = np.zeros(src.shape, np.int8)
    out[:, :d] = qi
    return out, scale


def np_scores_i8(keys, rs, q, qs):
    dot = q.astype(np.int64) @ keys.astype(np.int64).T
    s = dot.astype(np.float32) * rs[None, :].astype(np.float32)
    return (s.astype(np.float32) * qs[:, None].astype(np.float32)).astype(np.float32)


def py_topk_max(scores, k):
    """Pure-Python restatement of ref_pkm_topk_max (src/vector/reference/pkm_ref.mojo:110-130)."""
    n = len(scores)
    kk = min(k, n)
    if kk <= 0:
        return [], []
    val = [float(np.float32(s)) for s in scores[:kk]]
    idx = list(range(kk))

    def sift(start, size):
        root = start
        while True:
            c = 2 * root + 1
            if c >= size:
                return
            if c + 1 < size and val[c + 1] < val[c]:
                c += 1
            if val[c] < val[root]:
                val[root], val[c] = val[c], val[root]
                idx[root], idx[c] = idx[c], idx[root]
                root = c
            else:
                return

    for s in range(kk // 2 - 1, -1, -1):
        sift(s, kk)
    for i in range(kk, n):
        sv = float(scores[i])
        if sv > val[0]:
            val[0] = sv
            idx[0] = i
            sift(0, kk)
    # heapsort descending
    for s in range(kk // 2 - 1, -1, -1):
        sift(s, kk)
    for e in range(kk - 1, 0, -1):
        val[0], val[e] = val[e], val[0]
        idx[0], idx[e] = idx[e], idx[0]
        sift(0, e)
    return idx, val


# ---------------------------------------------------------- known answers --

def test_quantize_known_answers(oracle):
    # Hand-derived from src/vector/pkm_kernels.mojo:152-191: max|x| = 1 -> scale
    # 1/127, inv = 127 (f32: 1/(1/127) rounds to 127.0); 1.0 -> 127; -0.5 -> -63.5
    # -0.5 = -64 -> trunc -64; 0.25 -> 31.75 + 0.5 = 32.25 -> 32; 0 -> 0; padding 0.
    src = np.zeros((2, 8), np.float32)
    src[0, :4] = [1.0, -0.5, 0.25, 0.0]
    q, s = oracle.pkm_quantize_rows_i8(src, d=4)
    assert q[0].tolist() == [127, -64, 32, 0, 0, 0, 0, 0]
    assert s[0] == np.float32(1.0) / np.float32(127.0)
    # an all-zero row keeps scale 1.0 and codes 0
    assert s[1] == 1.0 and not q[1].any()


def test_scores_i8_known_answer(oracle):
    keys = np.zeros((2, 64), np.int8)
    keys[0, :3] = [127, -127, 5]
    keys[1, :2] = [1, 1]
    q = np.zeros((1, 64), np.int8)
    q[0, :3] = [2, 3, -4]
    rs = np.array([0.5, 0.25], np.float32)
    qs = np.array([2.0], np.float32)
    d = oracle.pkm_scores_i8(keys, rs, q, qs)
    # dot0 = 254 - 381 - 20 = -147 -> (-147 * 0.5) * 2 = -147; dot1 = 5 -> 2.5
    assert d.tolist() == [[-147.0, 2.5]]


def test_topk_ties_known_answer(oracle):
    # Five equal scores, k = 3: the first three (ids 0, 1, 2) seed the heap and an
    # equal later score never displaces (strict `>`).
    idx, val = oracle.pkm_topk_max(np.ones(5, np.float32), 3)
    assert sorted(idx.tolist()) == [0, 1, 2] and val.tolist() == [1.0, 1.0, 1.0]


def test_hamming_and_sign_bits_known_answer(oracle):
    x = np.zeros((1, 128), np.float32)
    x[0, 0] = 1.0      # bit 0 of word 0
    x[0, 63] = 0.5     # bit 63 of word 0
    x[0, 64] = -1.0    # negative -> 0
    x[0, 65] = 2.0     # bit 1 of word 1
    c = oracle.bq_pack_signs(x)
    assert c[0].tolist() == [1 | (1 << 63), 2]
    assert oracle.hamming(c[0], np.zeros(2, np.uint64)) == 3


# ------------------------------------------- the reference PKM differential --

def test_pkm_differential_structure(oracle):
    """tests/test_vector_differential.mojo:283-351 shape: S=1000, half-dim 448
    (d_pad 448), NQ=8, K=32; INT8 scores and top-k bit-exact between two
    restatements, FP32 within 1e-4 (1 + |s|)."""
    rng = np.random.Generator(np.random.PCG64(146))
    S, HALF, NQ, K = 1000, 448, 8, 32
    d_pad = ((HALF + 63) // 64) * 64
    keys = np.zeros((S, d_pad), np.float32)
    keys[:, :HALF] = rng.uniform(-1, 1, (S, HALF))
    q = np.zeros((NQ, d_pad), np.float32)
    q[:, :HALF] = rng.uniform(-1, 1, (NQ, HALF))

    a = oracle.pkm_scores_f32(keys, q)
    b = (q.astype(np.float64) @ keys.astype(np.float64).T)
    assert np.all(np.abs(a - b) <= 1e-4 * (1 + np.abs(b)))

    idx = rng.integers(0, S, 64).astype(np.int32)
    r = oracle.pkm_rescore_f32(keys, q[0], idx)
    assert np.allclose(r, b[0, idx], rtol=1e-4, atol=1e-4)

    ki, ks = oracle.pkm_quantize_rows_i8(keys, d=HALF)
    ki2, ks2 = np_quantize_rows_i8(keys, HALF)
    assert np.array_equal(ki, ki2) and np.array_equal(ks.view(np.uint32), ks2.view(np.uint32))
    qi, qsc = oracle.pkm_quantize_rows_i8(q, d=HALF)
    sa = oracle.pkm_scores_i8(ki, ks, qi, qsc)
    sb = np_scores_i8(ki, ks, qi, qsc)
    assert np.array_equal(sa.view(np.uint32), sb.view(np.uint32))

    for h in range(2):
        oi, ov = oracle.pkm_topk_max(sa[h], K)
        pi, pv = py_topk_max(sa[h], K)
        assert oi.tolist() == pi and ov.tolist() == [float(np.float32(v)) for v in pv]
    t0i, t0v = oracle.pkm_topk_max(sa[0], K)
    t1i, t1v = oracle.pkm_topk_max(sa[1], K)
    ci, cv = oracle.pkm_combine_topk(t0v, t0i, t1v, t1i, S, K)
    # every combined score is a pair sum; the list is the K largest sums, descending
    sums = (t0v[:, None].astype(np.float32) + t1v[None, :].astype(np.float32)).ravel()
    assert np.array_equal(np.sort(cv)[::-1], np.sort(sums)[::-1][:K])
    assert all(cv[i] >= cv[i + 1] for i in range(len(cv) - 1))

    v = rng.uniform(-1, 1, 500).astype(np.float32)
    sv, si = oracle.pkm_sort_desc(v, np.arange(500, dtype=np.int32))
    assert np.array_equal(sv, np.sort(v)[::-1]) and np.array_equal(v[si], sv)


def test_topk_heap_order_with_many_ties(oracle):
    rng = np.random.Generator(np.random.PCG64(7))
    s = rng.integers(0, 6, 3000).astype(np.float32)
    for k in (1, 5, 32, 100):
        oi, ov = oracle.pkm_topk_max(s, k)
        pi, pv = py_topk_max(s, k)
        assert oi.tolist() == pi and ov.tolist() == pv


def test_flat_i8_knn_equals_scores_plus_topk(oracle):
    rng = np.random.Generator(np.random.PCG64(11))
    n, dim, nq, k = 3000, 192, 5, 10
    keys, ks = oracle.pkm_quantize_rows_i8(rng.standard_normal((n, dim)).astype(np.float32))
    q, qs = oracle.pkm_quantize_rows_i8(rng.standard_normal((nq, dim)).astype(np.float32))
    ids, vals = oracle.flat_i8_knn(keys, ks, q, qs, k, nthreads=3)
    full = oracle.pkm_scores_i8(keys, ks, q, qs)
    for t in range(nq):
        ti, tv = oracle.pkm_topk_max(full[t], k)
        assert ids[t].tolist() == ti.tolist() and vals[t].tolist() == tv.tolist()
    # fewer rows than k pads with -1 / -inf
    ids2, vals2 = oracle.flat_i8_knn(keys[:3], ks[:3], q, qs, 5)
    assert (ids2[:, 3:] == -1).all() and np.isneginf(vals2[:, 3:]).all()


# ----------------------------------------------------------- exact FP32 rows --

def test_dot_4chain_and_normalise(oracle, rng):
    for dim in (1536, 448, 37, 3):
        a = rng.standard_normal(dim).astype(np.float32)
        b = rng.standard_normal(dim).astype(np.float32)
        ref = float(a.astype(np.float64) @ b.astype(np.float64))
        assert abs(oracle.dot_f32_4chain(a, b) - ref) <= 1e-4 * (1 + abs(ref))
        l2 = float(((a.astype(np.float64) - b) ** 2).sum())
        assert abs(oracle.l2sq_f32_4chain(a, b) - l2) <= 1e-4 * (1 + l2)
    x = rng.standard_normal((4, 1536)).astype(np.float32)
    x[3] = 0
    y = oracle.l2_normalize_rows(x)
    assert np.allclose(np.linalg.norm(y[:3], axis=1), 1.0, atol=1e-6)
    assert not y[3].any()  # a zero vector passes through


def test_exact_knn_cosine_order_and_ties(oracle, rng):
    n, dim, k = 2000, 256, 10
    rows = oracle.l2_normalize_rows(rng.standard_normal((n, dim)).astype(np.float32))
    rows[1500] = rows[10]   # exact duplicate -> tied score, earlier slot first
    qs = rng.standard_normal((4, dim)).astype(np.float32)
    qs[0] = rows[10] * 3.0
    ids, sc = oracle.exact_knn(rows, qs, k)
    for t in range(4):
        qn = oracle.exact_query_normalize(qs[t])
        ref = 1.0 - rows.astype(np.float64) @ qn.astype(np.float64)
        order = np.lexsort((np.arange(n), ref))
        # ranking agrees with float64 up to near-ties, scores within 1e-5
        assert np.all(np.abs(sc[t] - ref[ids[t]]) < 1e-5)
        assert np.all(np.diff(sc[t]) >= 0)
        assert set(ids[t]) <= set(order[:k + 5])
    # both copies are selected with identical scores; their order in the reply comes
    # from the heap's pop order (src/commands/vector.mojo:1335-1359), not from the slot
    assert set(ids[0, :2].tolist()) == {10, 1500} and sc[0, 0] == sc[0, 1]


# ---------------------------------------------------------------- BQ + rerank --

def test_bq_knn_matches_numpy(oracle, rng):
    n, dim, nq, sl, k = 3000, 256, 3, 50, 10
    rows = oracle.l2_normalize_rows(rng.standard_normal((n, dim)).astype(np.float32))
    codes = oracle.bq_pack_signs(rows)
    qs = rng.standard_normal((nq, dim)).astype(np.float32)
    ids, sc, sid, sd = oracle.bq_knn(codes, rows, qs, sl, k)
    for t in range(nq):
        qn = oracle.exact_query_normalize(qs[t])
        qb = rows > 0
        ham = (qb != (qn > 0)[None, :]).sum(axis=1)
        order = np.lexsort((np.arange(n), ham))[:sl]
        assert sid[t].tolist() == order.tolist()
        assert sd[t].tolist() == ham[order].tolist()
        resc = np.array([1.0 - oracle.dot_f32_4chain(qn, rows[i]) for i in order], np.float32)
        o2 = np.argsort(resc, kind="stable")[:k]
        assert ids[t].tolist() == order[o2].tolist()
        assert np.array_equal(sc[t], resc[o2])


def test_shard_merge_selection(oracle):
    ids = np.array([5, 1, 9, 2, 7], np.int64)
    sc = np.array([0.3, 0.1, 0.1, 0.5, 0.05], np.float32)
    oi, os_ = oracle.shard_merge_asc(ids, sc, 3)
    assert oi.tolist() == [7, 1, 9] and os_.tolist() == [np.float32(0.05), np.float32(0.1),
                                                          np.float32(0.1)]
