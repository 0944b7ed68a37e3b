"""The multi-GPU path's host logic (pion_b200.sharded) on CPU: world_size 2 over gloo.

Each rank scores its contiguous row shard with the oracle (standing in for the GPU
kernels, which a CPU box cannot run), the shard results are all-gathered through
ShardedSearch, and merged by (score, id).  Both ranks must return exactly the
single-index answer of the oracle (up to ties at the k-th place)."""
import os
import socket

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _merge(descending):
    """Test-side stand-in for the GPU merge kernel: (score, id) order over the lists."""
    import torch

    def merge(pairs):  # [W, B, k, 2] int32: (score bits, id)
        from pion_b200.sharded import unpack_pairs
        ids, scores = unpack_pairs(pairs)
        W, B, k = scores.shape
        s = scores.permute(1, 0, 2).reshape(B, W * k).numpy()
        i = ids.permute(1, 0, 2).reshape(B, W * k).numpy()
        out_i = np.empty((B, k), np.int32)
        out_s = np.empty((B, k), np.float32)
        for b in range(B):
            o = np.lexsort((i[b], -s[b] if descending else s[b]))[:k]
            out_i[b], out_s[b] = i[b][o], s[b][o]
        return torch.from_numpy(out_i), torch.from_numpy(out_s)

    return merge


def _rank_main(rank, world, port, mode, result_dir):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    import oracle
    from pion_b200.sharded import ShardedSearch, shard_bounds
    from pion_b200.workloads import mixture_np

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rows, qs = mixture_np(6000, 64, 16, seed=23, n_queries=20)
    k = 7
    lo, hi = shard_bounds(rows.shape[0], world, rank)
    if mode == "i8":
        keys, ks = oracle.pkm_quantize_rows_i8(rows)
        q, qsc = oracle.pkm_quantize_rows_i8(qs)

        def local(_):
            i, v = oracle.flat_i8_knn(keys[lo:hi], ks[lo:hi], q, qsc, k)
            i = np.where(i >= 0, i + lo, -1).astype(np.int32)
            return torch.from_numpy(i), torch.from_numpy(v)
        descending = True
    else:
        rn = oracle.l2_normalize_rows(rows)

        def local(_):
            i, v = oracle.exact_knn(rn[lo:hi], qs, k)
            i = np.where(i >= 0, i + lo, -1).astype(np.int32)
            return torch.from_numpy(i), torch.from_numpy(v)
        descending = False
    search = ShardedSearch(local, k, _merge(descending))
    ids, sc = search(None)
    np.save(os.path.join(result_dir, f"{mode}_{rank}_ids.npy"), ids.numpy())
    np.save(os.path.join(result_dir, f"{mode}_{rank}_sc.npy"), sc.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["i8", "f32"])
def test_two_rank_shards_equal_single_index(oracle, tmp_path, mode):
    import torch.multiprocessing as mp

    from pion_b200.workloads import mixture_np

    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), mode, str(tmp_path)), nprocs=world,
             join=True)
    rows, qs = mixture_np(6000, 64, 16, seed=23, n_queries=20)
    k = 7
    if mode == "i8":
        keys, ks = oracle.pkm_quantize_rows_i8(rows)
        q, qsc = oracle.pkm_quantize_rows_i8(qs)
        ref_i, ref_s = oracle.flat_i8_knn(keys, ks, q, qsc, k)
        full = oracle.pkm_scores_i8(keys, ks, q, qsc)
    else:
        rn = oracle.l2_normalize_rows(rows)
        ref_i, ref_s = oracle.exact_knn(rn, qs, k)
        full = None
    outs = [(np.load(tmp_path / f"{mode}_{r}_ids.npy"), np.load(tmp_path / f"{mode}_{r}_sc.npy"))
            for r in range(world)]
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])
    ids, sc = outs[0]
    for t in range(qs.shape[0]):
        assert np.array_equal(np.sort(sc[t]), np.sort(ref_s[t]))
        if set(ids[t].tolist()) != set(ref_i[t].tolist()):
            kth = sc[t][-1]
            for i in set(ids[t].tolist()) ^ set(ref_i[t].tolist()):
                val = full[t][i] if full is not None else None
                assert val is None or val == kth
