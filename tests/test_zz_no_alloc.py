"""The allocation-free FLAT INT8 entry point (pion_v_b200_flat_i8_knn_static).

Some engines cannot call cudaMalloc while serving a query (their device memory
is reserved up front by their own allocator, or the query thread must not take
cudaMalloc's device-wide synchronisation).  This entry point keeps its scratch in
a fixed static device array instead.  Here it is called through the C ABI with
device buffers and must return exactly what the regular entry point returns, on
two calls in a row (the second call reuses the array the first one left behind).
The file sorts last so that a stop-at-first-failure run has already run every
other test; it also passes alone in a fresh process."""
import numpy as np
import pytest

from pion_b200.workloads import mixture_np

pytestmark = pytest.mark.gpu


def _static_call(lib, dk, dks, dq, dqs, k, stream):
    import torch
    nq = dq.shape[0]
    oi = torch.full((nq, k), -7, dtype=torch.int32, device=dq.device)
    ov = torch.full((nq, k), float("nan"), dtype=torch.float32, device=dq.device)
    rc = lib.pion_v_b200_flat_i8_knn_static(dk.data_ptr(), dks.data_ptr(), dk.shape[0],
                                            dk.shape[1], dq.data_ptr(), dqs.data_ptr(), nq, k,
                                            oi.data_ptr(), ov.data_ptr(), stream)
    return rc, oi, ov


@pytest.mark.parametrize("k", [10, 32, 64])
def test_static_scratch_matches_regular_entry_point(oracle, k):
    """k = 10 takes the 8-epilogue-warp kernel with 16-entry lists; 32 and 64 the
    4-warp kernels with one list per split."""
    import torch
    import pion_b200
    from pion_b200 import _lib

    lib = _lib.load()
    rows, qf = mixture_np(20000, 1536, 64, seed=77, n_queries=300)
    keys, ks = oracle.pkm_quantize_rows_i8(rows)
    q, qs = oracle.pkm_quantize_rows_i8(qf)
    with pion_b200.Context(0) as ctx:
        ix = pion_b200.FlatI8Index(ctx, keys, ks)
        want_i, want_v = ix.search(q, qs, k)          # batch: tensor-core path
        want1_i, want1_v = ix.search(q[:1], qs[:1], k)  # one query: scan path
        ix.free()
    dk, dks = torch.from_numpy(keys).cuda(), torch.from_numpy(ks).cuda()
    dq, dqs = torch.from_numpy(q).cuda(), torch.from_numpy(qs).cuda()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        rc, oi, ov = _static_call(lib, dk, dks, dq, dqs, k, stream)
        assert rc == 0, f"call {call}: status {rc}"
        assert np.array_equal(oi.cpu().numpy(), want_i), f"call {call}: ids differ"
        assert np.array_equal(ov.cpu().numpy().view(np.uint32), want_v.view(np.uint32))
        rc, oi, ov = _static_call(lib, dk, dks, dq[:1].contiguous(), dqs[:1].contiguous(), k,
                                  stream)
        assert rc == 0
        assert np.array_equal(oi.cpu().numpy(), want1_i)
        assert np.array_equal(ov.cpu().numpy().view(np.uint32), want1_v.view(np.uint32))


def test_static_scratch_empty_index():
    """No rows: every result slot is padding (id -1, score -inf), on two calls."""
    import torch
    from pion_b200 import _lib

    lib = _lib.load()
    dk = torch.zeros((1, 1536), dtype=torch.int8, device="cuda")
    dks = torch.ones(1, dtype=torch.float32, device="cuda")
    dq = torch.ones((5, 1536), dtype=torch.int8, device="cuda")
    dqs = torch.ones(5, dtype=torch.float32, device="cuda")
    for _ in range(2):
        oi = torch.full((5, 10), 7, dtype=torch.int32, device="cuda")
        ov = torch.zeros((5, 10), dtype=torch.float32, device="cuda")
        rc = lib.pion_v_b200_flat_i8_knn_static(dk.data_ptr(), dks.data_ptr(), 0, 1536,
                                                dq.data_ptr(), dqs.data_ptr(), 5, 10,
                                                oi.data_ptr(), ov.data_ptr(),
                                                torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        assert (oi == -1).all() and torch.isneginf(ov).all()


def test_static_scratch_largest_batch_that_fits(oracle):
    """A batch at the edge of the static array -- it fits, one more query does not
    (found by bisection: a refused call returns before any launch) -- returns what the
    regular entry point does."""
    import torch
    import pion_b200
    from pion_b200 import _lib

    lib = _lib.load()
    rows, qf = mixture_np(60000, 1536, 64, seed=78, n_queries=4096)
    keys, ks = oracle.pkm_quantize_rows_i8(rows)
    q, qs = oracle.pkm_quantize_rows_i8(qf)
    dk, dks = torch.from_numpy(keys).cuda(), torch.from_numpy(ks).cuda()
    dq, dqs = torch.from_numpy(q).cuda(), torch.from_numpy(qs).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    lo, hi = 1, 4096  # lo fits, hi does not; keep it so until they are adjacent
    assert _static_call(lib, dk, dks, dq[:1], dqs[:1], 64, stream)[0] == 0
    assert _static_call(lib, dk, dks, dq, dqs, 64, stream)[0] == _lib.ESHAPE
    while hi - lo > 1:
        mid = (lo + hi) // 2
        rc = _static_call(lib, dk, dks, dq[:mid].contiguous(), dqs[:mid].contiguous(), 64,
                          stream)[0]
        assert rc in (0, _lib.ESHAPE)
        lo, hi = (mid, hi) if rc == 0 else (lo, mid)
    nq = lo
    with pion_b200.Context(0) as ctx:
        ix = pion_b200.FlatI8Index(ctx, keys, ks)
        want_i, want_v = ix.search(q[:nq], qs[:nq], 64)
        ix.free()
    for _ in range(2):
        rc, oi, ov = _static_call(lib, dk, dks, dq[:nq].contiguous(), dqs[:nq].contiguous(), 64,
                                  stream)
        assert rc == 0
        assert np.array_equal(oi.cpu().numpy(), want_i)
        assert np.array_equal(ov.cpu().numpy().view(np.uint32), want_v.view(np.uint32))


def test_static_scratch_rejects_oversized_calls():
    import torch
    from pion_b200 import _lib

    lib = _lib.load()
    dk = torch.zeros((100000, 64), dtype=torch.int8, device="cuda")
    dks = torch.ones(100000, dtype=torch.float32, device="cuda")
    dq = torch.zeros((8192, 64), dtype=torch.int8, device="cuda")
    dqs = torch.ones(8192, dtype=torch.float32, device="cuda")
    rc, _, _ = _static_call(lib, dk, dks, dq, dqs, 64, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.ESHAPE
