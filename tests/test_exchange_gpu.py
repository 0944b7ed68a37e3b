"""The NVLink peer-memory shard exchange on two GPUs (skipped with fewer): each rank holds
a row shard, pion_v_b200_flat_i8_knn_sharded shares the threshold sample, scores the shard
and exchanges the k-lists (or starts from its own sample share's bound and exchanges once);
every rank must return the single index's answer, step after step (the receive buffers
alternate by the step's parity).  The ranks are processes, one
per GPU, swapping the IPC handles over gloo."""
import os
import socket

import numpy as np
import pytest

from pion_b200.workloads import mixture_np

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# (batch, local bound) per step: the exchange's parities and regions in every order
CASES = ((300, 0), (1, 0), (130, 0), (300, 1), (7, 1), (130, 0), (64, 1))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    import oracle
    import pion_b200
    from pion_b200.sharded import PeerExchange, PeerShardedSearch, shard_bounds
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.set_device(rank)
    rows, qf = mixture_np(60000, 1536, 64, seed=5, n_queries=300)
    keys, ks = oracle.pkm_quantize_rows_i8(rows)
    q, qs = oracle.pkm_quantize_rows_i8(qf)
    lo, hi = shard_bounds(keys.shape[0], world, rank)
    with pion_b200.Context(rank) as ctx:
        ctx.set_wait_budget(5_000_000_000)
        ix = pion_b200.FlatI8Index(ctx, torch.from_numpy(keys[lo:hi]).cuda(),
                                   torch.from_numpy(ks[lo:hi]).cuda(), id_base=lo)
        ex = PeerExchange(ctx, 512, 10)
        steps = (PeerShardedSearch(ix, ex), PeerShardedSearch(ix, ex, local_bound=True))
        dq, dqs = torch.from_numpy(q).cuda(), torch.from_numpy(qs).cuda()
        for s, (b, local) in enumerate(CASES):  # both parities, both bounds
            ids, sc = steps[local]([dq[:b].contiguous(), dqs[:b].contiguous()])
            torch.cuda.synchronize()
            ctx.sync()
            np.save(os.path.join(out_dir, f"r{rank}_s{s}_ids.npy"), ids.cpu().numpy())
            np.save(os.path.join(out_dir, f"r{rank}_s{s}_sc.npy"), sc.cpu().numpy())
        torch.cuda.synchronize()
        dist.barrier()
        ex.close()
        ix.free()
    dist.barrier()
    dist.destroy_process_group()


def test_two_gpu_peer_exchange_equals_single_index(oracle, tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    rows, qf = mixture_np(60000, 1536, 64, seed=5, n_queries=300)
    keys, ks = oracle.pkm_quantize_rows_i8(rows)
    q, qs = oracle.pkm_quantize_rows_i8(qf)
    oi, ov = oracle.flat_i8_knn(keys, ks, q, qs, 10)
    for s, (b, _) in enumerate(CASES):
        for r in range(2):
            ids = np.load(tmp_path / f"r{r}_s{s}_ids.npy")
            sc = np.load(tmp_path / f"r{r}_s{s}_sc.npy")
            for t in range(b):
                o = np.lexsort((oi[t], -ov[t]))
                assert ids[t].tolist() == oi[t][o].tolist(), (s, r, t)
                assert np.array_equal(sc[t].view(np.uint32), ov[t][o].view(np.uint32))
