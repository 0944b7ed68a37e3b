"""FLAT INT8 inner product on the GPU against the CPU oracle.

Scores must be bit-identical to ref_pkm_scores_i8 (src/vector/reference/pkm_ref.mojo:
47-61) and ids identical to the (score desc, id asc) order; the reference's own
heap selection (ref_pkm_topk_max) may differ only among scores tied at the k-th
place, which is checked too."""
import os

import numpy as np
import pytest

from pion_b200.workloads import mixture_np

pytestmark = pytest.mark.gpu


def quantized_case(oracle, n, dim, nq, seed, centres=64):
    rows, qs = mixture_np(n, dim, centres, seed, nq)
    keys, ks = oracle.pkm_quantize_rows_i8(rows)
    q, qsc = oracle.pkm_quantize_rows_i8(qs)
    return keys, ks, q, qsc


def assert_matches_oracle(oracle, keys, ks, q, qsc, k, ids, sc):
    n = keys.shape[0]
    kk = min(k, n)
    full = oracle.pkm_scores_i8(keys, ks, q, qsc)
    ref_i, ref_v = oracle.flat_i8_knn(keys, ks, q, qsc, k)
    for t in range(q.shape[0]):
        order = np.lexsort((np.arange(n), -full[t]))[:kk]
        assert ids[t, :kk].tolist() == order.tolist(), f"query {t}"
        assert np.array_equal(sc[t, :kk].view(np.uint32), full[t][order].view(np.uint32))
        assert (ids[t, kk:] == -1).all() and np.isneginf(sc[t, kk:]).all()
        # the reference heap selects the same set unless scores tie at the k-th place
        a, b = set(order.tolist()), set(ref_i[t, :kk].tolist())
        if a != b:
            kth = full[t][order[-1]]
            assert all(full[t][i] == kth for i in a ^ b)
        assert np.array_equal(np.sort(ref_v[t, :kk]), np.sort(sc[t, :kk]))


@pytest.fixture
def path_env():
    old = os.environ.get("PION_B200_I8_PATH")
    yield
    if old is None:
        os.environ.pop("PION_B200_I8_PATH", None)
    else:
        os.environ["PION_B200_I8_PATH"] = old


def test_quantize_rows_bit_exact(ctx, oracle, rng):
    import pion_b200
    x = rng.standard_normal((3000, 1536)).astype(np.float32)
    x[0] = 0.0
    x[1, :4] = [1.0, -0.5, 0.25, 0.0]
    x[1, 4:] = 0.0
    x[2] *= 1e-30
    x[3] *= 1e30
    x[4] = np.float32(0.5) * np.sign(x[4])  # every element on a rounding boundary
    for d in (1536, 1000):
        a, s = pion_b200.quantize_rows_i8(ctx, x, d=d)
        b, t = oracle.pkm_quantize_rows_i8(x, d=d)
        assert np.array_equal(a, b)
        assert np.array_equal(s.view(np.uint32), t.view(np.uint32))


@pytest.mark.parametrize("n,dim,nq,k,path", [
    (20000, 1536, 1, 10, 0),
    (20000, 1536, 1, 10, 2),
    (20000, 1536, 3, 10, 1),
    (20000, 1536, 128, 10, 0),
    (20000, 1536, 300, 32, 0),
    (5000, 448, 77, 64, 0),
    (3000, 64, 5, 1, 0),
    (777, 1536, 130, 16, 0),
    (50, 1536, 2, 64, 0),
    (50, 1536, 2, 64, 1),
    (200000, 1536, 16, 10, 0),   # threshold pre-pass active
    (200000, 1536, 16, 64, 0),
])
def test_flat_i8_knn_matches_oracle(ctx, oracle, path_env, n, dim, nq, k, path):
    import pion_b200
    os.environ["PION_B200_I8_PATH"] = str(path)
    keys, ks, q, qsc = quantized_case(oracle, n, dim, nq, seed=n + nq)
    ix = pion_b200.FlatI8Index(ctx, keys, ks)
    ids, sc = ix.search(q, qsc, k)
    assert_matches_oracle(oracle, keys, ks, q, qsc, k, ids, sc)


@pytest.mark.parametrize("k", [1, 10, 32])
def test_forced_prepass_on_small_index(ctx, oracle, k):
    """The threshold pre-pass (first max(64, 8k) tiles) + main pass over the rest."""
    import pion_b200
    keys, ks, q, qsc = quantized_case(oracle, 80000, 1536, 130, seed=17)
    ix = pion_b200.FlatI8Index(ctx, keys, ks)
    os.environ["PION_B200_I8_PREPASS"] = "1"
    try:
        ids, sc = ix.search(q, qsc, k)
    finally:
        os.environ.pop("PION_B200_I8_PREPASS", None)
    assert_matches_oracle(oracle, keys, ks, q, qsc, k, ids, sc)


@pytest.mark.parametrize("path", [1, 2])
def test_ties_break_by_ascending_id(ctx, oracle, path_env, path):
    import pion_b200
    os.environ["PION_B200_I8_PATH"] = str(path)
    keys, ks, q, qsc = quantized_case(oracle, 4096, 256, 4, seed=5)
    # plant duplicates of the rows nearest to each query at later ids
    full = oracle.pkm_scores_i8(keys, ks, q, qsc)
    for t in range(4):
        best = int(np.argmax(full[t]))
        for j in range(3):
            keys[1000 + 700 * j + t] = keys[best]
            ks[1000 + 700 * j + t] = ks[best]
    ix = pion_b200.FlatI8Index(ctx, keys, ks)
    ids, sc = ix.search(q, qsc, 8)
    assert_matches_oracle(oracle, keys, ks, q, qsc, 8, ids, sc)


def test_device_memory_path_equals_host(ctx, oracle):
    import torch
    import pion_b200
    keys, ks, q, qsc = quantized_case(oracle, 10000, 1536, 200, seed=3)
    ix_h = pion_b200.FlatI8Index(ctx, keys, ks)
    ids_h, sc_h = ix_h.search(q, qsc, 10)
    dk, dks = torch.from_numpy(keys).cuda(), torch.from_numpy(ks).cuda()
    ix_d = pion_b200.FlatI8Index(ctx, dk, dks, id_base=5, borrow=True)
    ids_d, sc_d = ix_d.search(torch.from_numpy(q).cuda(), torch.from_numpy(qsc).cuda(), 10)
    torch.cuda.synchronize()
    ctx.sync()
    assert np.array_equal(ids_d.cpu().numpy(), ids_h + 5)
    assert np.array_equal(sc_d.cpu().numpy(), sc_h)


def test_register_index_descriptor(ctx, oracle):
    """pion_v_b200_register_index dispatches on the kind: a FLAT INT8 index registered
    through the descriptor answers like one registered directly; unknown kinds fail."""
    import ctypes

    import pion_b200
    from pion_b200 import _lib
    keys, ks, q, qsc = quantized_case(oracle, 5000, 1536, 64, seed=4)
    want_i, want_s = pion_b200.FlatI8Index(ctx, keys, ks).search(q, qsc, 10)
    d = _lib.IndexDesc(kind=1, mem=0, n_rows=keys.shape[0], dim=1536, id_base=0, normalize=0,
                       reserved=0, rows=keys.ctypes.data, row_scale=ks.ctypes.data, hnsw=None)
    h = ctypes.c_void_p()
    ctx.check(ctx.lib.pion_v_b200_register_index(ctx.h, ctypes.byref(d), ctypes.byref(h)))
    ids = np.empty((64, 10), np.int32)
    sc = np.empty((64, 10), np.float32)
    ctx.check(ctx.lib.pion_v_b200_flat_i8_knn(ctx.h, h, q.ctypes.data, qsc.ctypes.data, 64, 10,
                                              ids.ctypes.data, sc.ctypes.data, 0))
    ctx.lib.pion_v_b200_index_free(h)
    assert np.array_equal(ids, want_i) and np.array_equal(sc, want_s)
    d.kind = 9
    h2 = ctypes.c_void_p()
    assert ctx.lib.pion_v_b200_register_index(ctx.h, ctypes.byref(d), ctypes.byref(h2)) == -1
    assert not h2.value


def test_empty_index_and_bad_shapes(ctx, oracle):
    import pion_b200
    keys = np.zeros((0, 1536), np.int8)
    ix = pion_b200.FlatI8Index(ctx, keys, np.zeros(0, np.float32))
    ids, sc = ix.search(np.zeros((2, 1536), np.int8), np.ones(2, np.float32), 4)
    assert (ids == -1).all() and np.isneginf(sc).all()
    keys, ks, q, qsc = quantized_case(oracle, 100, 64, 2, seed=9)
    ix = pion_b200.FlatI8Index(ctx, keys, ks)
    with pytest.raises(pion_b200.PionError) as e:
        ix.search(q, qsc, 65)
    assert e.value.code == -3
    with pytest.raises(pion_b200.PionError):
        pion_b200.FlatI8Index(ctx, np.zeros((10, 24), np.int8), np.ones(10, np.float32))


def test_merge_topk_matches_numpy(ctx, rng):
    import pion_b200
    nq, L, k = 37, 19, 10
    v = np.sort(rng.integers(0, 50, (nq, L, k)).astype(np.float32), axis=2)[:, :, ::-1].copy()
    i = rng.integers(0, 10000, (nq, L, k)).astype(np.int32)
    # lists must be ordered (score desc, id asc)
    for a in range(nq):
        for b in range(L):
            o = np.lexsort((i[a, b], -v[a, b]))
            v[a, b], i[a, b] = v[a, b][o], i[a, b][o]
    ids, sc = pion_b200.merge_topk(ctx, v, i, k, descending=True)
    for a in range(nq):
        fv, fi = v[a].ravel(), i[a].ravel()
        o = np.lexsort((fi, -fv))[:k]
        assert ids[a].tolist() == fi[o].tolist() and sc[a].tolist() == fv[o].tolist()


def test_full_size_one_million_rows(ctx, oracle):
    """1M x 1536 (1024 centres), 1024 queries, k=10: tensor-core path vs the one-query
    scan on 16 queries, and vs the oracle on 3 queries."""
    import torch
    import pion_b200
    from pion_b200.workloads import mixture_torch
    rows, qf = mixture_torch(1_000_000, 1536, 1024, seed=1, n_queries=1024)
    keys, ks = pion_b200.quantize_rows_i8(ctx, rows)
    q, qsc = pion_b200.quantize_rows_i8(ctx, qf)
    del rows
    ix = pion_b200.FlatI8Index(ctx, keys, ks, borrow=True)
    try:
        ids, sc = ix.search(q, qsc, 10)
        os.environ["PION_B200_I8_PATH"] = "1"
        ids1, sc1 = ix.search(q[:16].contiguous(), qsc[:16].contiguous(), 10)
        torch.cuda.synchronize()
        ctx.sync()
    finally:
        os.environ.pop("PION_B200_I8_PATH", None)
    assert torch.equal(ids[:16], ids1) and torch.equal(sc[:16], sc1)
    hk, hks = keys.cpu().numpy(), ks.cpu().numpy()
    hq, hqs = q[:3].cpu().numpy(), qsc[:3].cpu().numpy()
    oi, ov = oracle.flat_i8_knn(hk, hks, hq, hqs, 10)
    got_i, got_v = ids[:3].cpu().numpy(), sc[:3].cpu().numpy()
    for t in range(3):
        assert np.array_equal(np.sort(ov[t]), np.sort(got_v[t]))
        assert set(oi[t].tolist()) == set(got_i[t].tolist())
    # sortedness and id validity over the whole batch
    s = sc.cpu().numpy()
    assert (np.diff(s, axis=1) <= 0).all()
    assert ((ids >= 0) & (ids < 1_000_000)).all()


@pytest.mark.parametrize("descending,lists_major", [(True, True), (False, True), (True, False)])
def test_merge_topk_pairs_matches_numpy(ctx, rng, descending, lists_major):
    """The all-gather layout: one buffer of interleaved (f32 score, i32 id) pairs,
    ties at every score, padding entries (id -1) at the ends of some lists."""
    import torch

    import pion_b200
    from pion_b200.sharded import pack_pairs
    L, nq, k = 8, 300, 10
    v = rng.integers(0, 6, (L, nq, k)).astype(np.float32)
    i = rng.integers(0, 100000, (L, nq, k)).astype(np.int32)
    sign = -1.0 if descending else 1.0
    pad = -np.inf if descending else np.inf
    v[0, :5, 7:] = pad
    i[0, :5, 7:] = -1
    for a in range(L):
        for b in range(nq):
            o = np.lexsort((np.where(i[a, b] < 0, 1 << 30, i[a, b]), sign * v[a, b]))
            v[a, b], i[a, b] = v[a, b][o], i[a, b][o]
    pairs = pack_pairs(torch.from_numpy(i), torch.from_numpy(v))  # [L, nq, k, 2]
    if not lists_major:
        pairs = pairs.permute(1, 0, 2, 3).contiguous()
    for dev in (False, True):
        p = pairs.cuda() if dev else pairs.numpy()
        ids, sc = pion_b200.merge_topk_pairs(ctx, p, k, descending=descending,
                                             lists_major=lists_major)
        if dev:
            ids, sc = ids.cpu().numpy(), sc.cpu().numpy()
        for b in range(nq):
            fv, fi = v[:, b].ravel(), i[:, b].ravel()
            o = np.lexsort((np.where(fi < 0, 1 << 30, fi), sign * fv))[:k]
            assert ids[b].tolist() == fi[o].tolist(), b
            assert sc[b].tolist() == fv[o].tolist(), b


def test_merge_topk_many_lists_unstaged(ctx, rng):
    """More lists x k than a warp stages in shared memory: the global-memory path."""
    import pion_b200
    nq, L, k = 9, 300, 16
    v = -np.sort(-rng.standard_normal((nq, L, k)).astype(np.float32), axis=2)
    i = rng.integers(0, 1 << 30, (nq, L, k)).astype(np.int32)
    ids, sc = pion_b200.merge_topk(ctx, v, i, k, descending=True)
    for a in range(nq):
        fv, fi = v[a].ravel(), i[a].ravel()
        o = np.lexsort((fi, -fv))[:k]
        assert ids[a].tolist() == fi[o].tolist()


def test_timing_phases(ctx, oracle):
    """The threshold and main passes are timed separately inside the scoring span."""
    import pion_b200
    keys, ks, q, qsc = quantized_case(oracle, 120000, 1536, 256, seed=77)
    ix = pion_b200.FlatI8Index(ctx, keys, ks)
    ctx.timing(True)
    try:
        for _ in range(3):
            ix.search(q, qsc, 10)
        tot, n = ctx.timing_read(0)
        thr, nt = ctx.timing_read(1)
        main, nm = ctx.timing_read(2)
    finally:
        ctx.timing(False)
    assert n == 3 and nt == 3 and nm == 3
    assert 0 < thr < tot and 0 < main < tot and thr + main <= tot * 1.001
    ix.free()


def test_second_device_in_one_process(oracle):
    """The kernels' shared-memory limit is raised on every device a process uses, not
    only on the first one that launched them."""
    import torch

    import pion_b200
    if torch.cuda.device_count() < 2:
        pytest.skip("one visible GPU")
    keys, ks, q, qsc = quantized_case(oracle, 20000, 1536, 130, seed=5)
    got = []
    for dev in (0, 1):
        with pion_b200.Context(dev) as c:
            ix = pion_b200.FlatI8Index(c, keys, ks)
            got.append(ix.search(q, qsc, 10))
            got.append(ix.search(q, qsc, 40))
            ix.free()
    assert all(np.array_equal(a[0], b[0]) for a, b in zip(got[:2], got[2:]))
    assert_matches_oracle(oracle, keys, ks, q, qsc, 10, *got[0])


def test_wait_that_runs_out(ctx, oracle, monkeypatch):
    """A device-side wait that runs out (one CTA's MMA warp waits on a barrier nothing
    arrives on, with a 1 ms budget) ends the kernel with PION_B200_ETIMEOUT: the copies
    and MMAs in flight drain, the tensor memory is freed, and the next call on the same
    context is correct.  Host-buffer calls report it themselves; device-buffer calls
    through pion_v_b200_sync, never as a later call's failure."""
    import torch

    import pion_b200
    from pion_b200 import _lib
    keys, ks, q, qsc = quantized_case(oracle, 20000, 1536, 300, seed=31)
    ix = pion_b200.FlatI8Index(ctx, keys, ks)
    want_i, want_v = ix.search(q, qsc, 10)
    dq, dqs = torch.from_numpy(q).cuda(), torch.from_numpy(qsc).cuda()
    ctx.set_wait_budget(1_000_000)
    monkeypatch.setenv("PION_B200_TEST_STALL", "1")
    try:
        with pytest.raises(pion_b200.PionError) as e:
            ix.search(q, qsc, 10)
        assert e.value.code == _lib.ETIMEOUT
        ix.search(dq, dqs, 10)            # device buffers: returns once queued
        monkeypatch.delenv("PION_B200_TEST_STALL")
        got_i, got_v = ix.search(q, qsc, 10)  # a host call after it is not blamed
        assert np.array_equal(got_i, want_i)
        with pytest.raises(pion_b200.PionError) as e:
            ctx.sync()
        assert e.value.code == _lib.ETIMEOUT
    finally:
        monkeypatch.delenv("PION_B200_TEST_STALL", raising=False)
        ctx.set_wait_budget(0)
    ctx.sync()
    got_i, got_v = ix.search(q, qsc, 10)
    assert np.array_equal(got_i, want_i) and np.array_equal(got_v, want_v)
    di, dv = ix.search(dq, dqs, 10)
    ctx.sync()
    assert np.array_equal(di.cpu().numpy(), want_i)
    ix.free()


@pytest.mark.parametrize("descending", [True, False])
def test_merge_many_lists_one_cta_per_query(ctx, rng, descending):
    """More than 128 lists per query (a one-query scan's per-CTA lists) take the CTA-per-
    query merge: host and device memory, the pair layout, lists-major."""
    import torch

    import pion_b200
    from pion_b200.sharded import pack_pairs
    L, nq, k = 600, 3, 10
    sign = -1.0 if descending else 1.0
    v = rng.integers(0, 40, (L, nq, k)).astype(np.float32)
    i = rng.integers(0, 1 << 20, (L, nq, k)).astype(np.int32)
    for a in range(L):
        for b in range(nq):
            o = np.lexsort((i[a, b], sign * v[a, b]))
            v[a, b], i[a, b] = v[a, b][o], i[a, b][o]
    want = []
    for b in range(nq):
        fv, fi = v[:, b].ravel(), i[:, b].ravel()
        o = np.lexsort((fi, sign * fv))[:k]
        want.append((fi[o], fv[o]))
    pairs = pack_pairs(torch.from_numpy(i), torch.from_numpy(v))
    for p in (pairs.numpy(), pairs.cuda()):
        ids, sc = pion_b200.merge_topk_pairs(ctx, p, k, descending=descending, lists_major=True)
        ids = ids if isinstance(ids, np.ndarray) else ids.cpu().numpy()
        sc = sc if isinstance(sc, np.ndarray) else sc.cpu().numpy()
        for b in range(nq):
            assert ids[b].tolist() == want[b][0].tolist()
            assert sc[b].tolist() == want[b][1].tolist()
    vq = np.ascontiguousarray(v.transpose(1, 0, 2))
    iq = np.ascontiguousarray(i.transpose(1, 0, 2))
    ids, sc = pion_b200.merge_topk(ctx, vq, iq, k, descending=descending)
    for b in range(nq):
        assert ids[b].tolist() == want[b][0].tolist()


def test_search_pairs_equals_search(ctx, oracle):
    """PION_B200_OUT_PAIRS: the final merge writes interleaved (score, id) pairs, equal to
    packing the two-array result; for the batched path, the one-query scan and an empty
    index."""
    import torch

    import pion_b200
    from pion_b200.sharded import pack_pairs
    keys, ks = oracle.pkm_quantize_rows_i8(mixture_np(30000, 1536, 64, 9, 0)[0])
    q, qsc = oracle.pkm_quantize_rows_i8(mixture_np(10, 1536, 64, 10, 200)[1])
    dk, dks = torch.from_numpy(keys).cuda(), torch.from_numpy(ks).cuda()
    dq, dqs = torch.from_numpy(q).cuda(), torch.from_numpy(qsc).cuda()
    ix = pion_b200.FlatI8Index(ctx, dk, dks, id_base=500)
    for b in (200, 1):
        ids, sc = ix.search(dq[:b].contiguous(), dqs[:b].contiguous(), 10)
        pairs = ix.search_pairs(dq[:b].contiguous(), dqs[:b].contiguous(), 10)
        torch.cuda.synchronize()
        assert torch.equal(pairs, pack_pairs(ids, sc))
    ix.free()
    empty = pion_b200.FlatI8Index(ctx, dk[:0], dks[:0])
    pairs = empty.search_pairs(dq[:3].contiguous(), dqs[:3].contiguous(), 4)
    torch.cuda.synchronize()
    assert (pairs[..., 1] == -1).all()
    assert torch.isneginf(pairs[..., 0].contiguous().view(torch.float32)).all()
    empty.free()


def test_ten_entry_lists_equal_sixteen_entry_lists(ctx, oracle, monkeypatch):
    """k = 10 runs the tensor-core kernel with ten-entry register lists (the k-th is the
    last entry); the sixteen-entry kernel (PION_B200_I8_KCAP16=1) gives the same scores
    and ids, and both equal the oracle -- with planted duplicate rows so that scores tie
    at the tenth place."""
    import pion_b200
    rows, qf = mixture_np(70000, 1536, 64, seed=14, n_queries=300)
    rows[1000:1040] = rows[5]          # forty copies of one row: ties at every rank
    keys, ks = oracle.pkm_quantize_rows_i8(rows)
    q, qs = oracle.pkm_quantize_rows_i8(qf)
    q[:3] = keys[5]
    qs[:3] = ks[5]
    ix = pion_b200.FlatI8Index(ctx, keys, ks)
    a = ix.search(q, qs, 10)
    monkeypatch.setenv("PION_B200_I8_KCAP16", "1")
    b = ix.search(q, qs, 10)
    monkeypatch.delenv("PION_B200_I8_KCAP16")
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32))
    oi, ov = oracle.flat_i8_knn(keys, ks, q, qs, 10)
    for t in range(q.shape[0]):
        o = np.lexsort((oi[t], -ov[t]))
        assert a[0][t].tolist() == oi[t][o].tolist(), t
        assert np.array_equal(a[1][t].view(np.uint32), ov[t][o].view(np.uint32)), t
    ix.free()
