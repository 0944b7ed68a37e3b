"""Every benchmarked configuration at its full size, on the GPU, against the CPU oracle.

* FLAT INT8 inner product, 1M x 1536 (1024 centres, seed 1), all 1024 queries of the
  batch, k = 10: scores bit-identical to ref_pkm_scores_i8 and ids identical to
  ref_pkm_topk_max's selection (src/vector/reference/pkm_ref.mojo:47-61, 110-130), whose
  strict `>` admission in ascending row order keeps the earliest row among equal scores,
  so the selected set is the top k by (score desc, id asc).
* Binary-quantised FLAT with FP32 rerank, 1M x 1536 (seed 2), 1024 queries, Hamming
  shortlist 100 then cosine rerank to 10 (src/vector/reference/quant_dots.mojo:95-100,
  src/commands/vector.mojo:1413-1456): ids and scores bit-identical.
* HNSW INT8, 1M x 1536 (seed 3), M 16, efConstruction 200, the 4096-query batch at ef
  64, 128 and 256 (src/vector/hnsw.mojo:4136-4521, beam_1536.mojo:85-135): ids, pool
  distances and work counters identical to the oracle beam on the same host-built
  graph, hence the same recall@10 against exact FLAT (reported).
* Sharded FLAT INT8, 10M x 1536 (4096 centres, seed 4) as 8 row shards merged by
  (score, id) (src/commands/vector.mojo:4394-4436), batches of 1, 64 and 4096: 64
  sampled queries against the oracle, the 8-shard merge equal to the single index for
  every query, and batch 1 (the one-query scan) equal to the batched path.

The inputs come from the same seeded device generator the benchmark uses.  These are
the slow tests of the GPU suite (minutes, most of it the oracle and the host graph
build)."""
import os

import numpy as np
import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def _i8_index(ctx, n, centres, seed, nq, chunk=1 << 20):
    """Quantised rows and queries on the device (pkm_quantize_rows_i8 on the GPU,
    checked bit-exact against the oracle elsewhere)."""
    import torch

    import pion_b200
    from pion_b200.workloads import mixture_torch
    keys = torch.empty((n, 1536), dtype=torch.int8, device="cuda")
    ks = torch.empty(n, dtype=torch.float32, device="cuda")
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        part, _ = mixture_torch(n, 1536, centres, seed, 0, row_range=(s, e))
        kq, sq = pion_b200.quantize_rows_i8(ctx, part)
        keys[s:e], ks[s:e] = kq, sq
        del part, kq, sq
    _, qf = mixture_torch(n, 1536, centres, seed, nq, row_range=(0, 0))
    q, qs = pion_b200.quantize_rows_i8(ctx, qf)
    torch.cuda.synchronize()
    return keys, ks, q, qs


def _assert_i8_equal(ids, sc, oi, ov):
    """GPU (score desc, id asc) lists == the oracle's selection re-sorted the same way."""
    for t in range(ids.shape[0]):
        o = np.lexsort((oi[t], -ov[t]))
        assert ids[t].tolist() == oi[t][o].tolist(), f"query {t}"
        assert np.array_equal(sc[t].view(np.uint32), ov[t][o].view(np.uint32)), f"query {t}"


def test_flat_i8_1m_full_batch(ctx, oracle):
    import pion_b200
    keys, ks, q, qs = _i8_index(ctx, 1_000_000, 1024, 1, 1024)
    ix = pion_b200.FlatI8Index(ctx, keys, ks, borrow=True)
    ids, sc = ix.search(q, qs, 10)
    ids1, sc1 = ix.search(q[:1].contiguous(), qs[:1].contiguous(), 10)  # one-query scan
    ctx.sync()
    hk, hks, hq, hqs = (x.cpu().numpy() for x in (keys, ks, q, qs))
    oi, ov = oracle.flat_i8_knn(hk, hks, hq, hqs, 10)
    _assert_i8_equal(ids.cpu().numpy(), sc.cpu().numpy(), oi, ov)
    assert np.array_equal(ids1.cpu().numpy()[0], ids.cpu().numpy()[0])
    ix.free()


def test_bq_1m_full_batch(ctx, oracle):
    import torch

    import pion_b200
    from pion_b200.workloads import mixture_torch
    rows, qf = mixture_torch(1_000_000, 1536, 1024, seed=2, n_queries=1024)
    ix = pion_b200.BQIndex(ctx, rows)
    ids, sc = ix.search(qf, 10, shortlist=100)
    ctx.sync()
    hr = rows.cpu().numpy()
    hq = qf.cpu().numpy()
    del rows
    ix.free()
    torch.cuda.empty_cache()
    rn = oracle.l2_normalize_rows(hr)
    del hr
    codes = oracle.bq_pack_signs(rn)
    oi, os_, _, _ = oracle.bq_knn(codes, rn, hq, 100, 10)
    assert np.array_equal(ids.cpu().numpy(), oi.astype(np.int32))
    assert np.array_equal(sc.cpu().numpy().view(np.uint32), os_.view(np.uint32))


@pytest.fixture(scope="module")
def hnsw_1m(ctx):
    """The 1M x 1536 graph of the HNSW benchmark (seed 3, M 16, efConstruction 200),
    built on the host by the library's builder (the reference's FT.OPTIMIZE build)."""
    import pion_b200
    from pion_b200.workloads import mixture_torch
    rows, qf = mixture_torch(1_000_000, 1536, 1024, seed=3, n_queries=4096)
    hr, hq = rows.cpu().numpy(), qf.cpu().numpy()
    del rows
    g = pion_b200.HNSWGraph(hr, M=16, ef_construction=200)
    ix = pion_b200.HNSWIndex(ctx, g)
    yield g, g.arrays(), ix, hr, hq
    ix.free()


@pytest.fixture(scope="module")
def hnsw_1m_truth(ctx, hnsw_1m):
    import torch

    import pion_b200
    _, _, _, hr, hq = hnsw_1m
    flat = pion_b200.FlatF32Index(ctx, torch.from_numpy(hr).cuda())
    truth, _ = flat.search(torch.from_numpy(hq).cuda(), 10)
    t = truth.cpu().numpy()
    flat.free()
    torch.cuda.empty_cache()
    return t


@pytest.mark.parametrize("ef", [64, 128, 256])
def test_hnsw_1m_full_batch(oracle, hnsw_1m, hnsw_1m_truth, ef):
    g, A, ix, hr, hq = hnsw_1m
    ids, dist = ix.search(hq, 10, ef)
    st = ix.last_stats()
    oi, od, ost = oracle.hnsw_search(A, hq, 10, ef)
    assert np.array_equal(ids, oi), f"ids differ at ef={ef}"
    assert np.array_equal(dist.view(np.uint32), od.view(np.uint32)), f"dists differ at ef={ef}"
    assert st == ost, (st, ost)
    t = hnsw_1m_truth
    rec = float(np.mean([len(set(ids[i]) & set(t[i])) / 10 for i in range(len(t))]))
    rec_o = float(np.mean([len(set(oi[i]) & set(t[i])) / 10 for i in range(len(t))]))
    print(f"HNSW 1M ef={ef}: recall@10 GPU {rec:.4f}, oracle {rec_o:.4f}")
    assert rec == rec_o


def test_sharded_flat_i8_10m(ctx, oracle):
    """Config 5 on one GPU: the 8 row shards as 8 indexes with global ids, each
    searched, the per-shard pairs merged lists-major (the layout of the all-gather)."""
    import torch

    import pion_b200
    from pion_b200.sharded import pack_pairs, shard_bounds
    n, shards = 10_000_000, 8
    keys, ks, q, qs = _i8_index(ctx, n, 4096, 4, 4096)
    full = pion_b200.FlatI8Index(ctx, keys, ks, borrow=True)
    parts = []
    for r in range(shards):
        lo, hi = shard_bounds(n, shards, r)
        parts.append(pion_b200.FlatI8Index(ctx, keys[lo:hi], ks[lo:hi], id_base=lo, borrow=True))
    for b in (4096, 64):
        qb, qsb = q[:b].contiguous(), qs[:b].contiguous()
        ids, sc = full.search(qb, qsb, 10)
        pairs = torch.stack([pack_pairs(*p.search(qb, qsb, 10)) for p in parts])
        mi, ms = pion_b200.merge_topk_pairs(ctx, pairs, 10, descending=True, lists_major=True)
        ctx.sync()
        assert torch.equal(mi, ids) and torch.equal(ms.view(torch.int32), sc.view(torch.int32))
        if b == 64:
            g_ids, g_sc = ids.cpu().numpy(), sc.cpu().numpy()
    ids1, sc1 = full.search(q[:1].contiguous(), qs[:1].contiguous(), 10)
    ctx.sync()
    assert np.array_equal(ids1.cpu().numpy()[0], g_ids[0])
    hk, hks = keys.cpu().numpy(), ks.cpu().numpy()
    oi, ov = oracle.flat_i8_knn(hk, hks, q[:64].cpu().numpy(), qs[:64].cpu().numpy(), 10)
    _assert_i8_equal(g_ids, g_sc, oi, ov)
    for p in parts:
        p.free()
    full.free()
