"""Seeded synthetic KNN workloads: L2-normalised Gaussian mixtures.

A point is ``centre[u] + sigma * N(0, I)`` with centres ~ N(0, I)^dim and u uniform
over the centres, then scaled to unit L2 length.  This stands in for the 1536-d
OpenAI-embedding dataset Pion's own benchmarks use (unit vectors, clustered).

``mixture_np`` draws on the host with numpy's PCG64 (small cases, CPU tests);
``mixture_torch`` draws on a CUDA device with torch's Philox generator (full-size
benchmarks; 1M x 1536 takes well under a second there).  Both are deterministic
for a given seed, but they are different random streams.
"""
from __future__ import annotations

import numpy as np

SIGMA = 0.3


def mixture_np(n: int, dim: int, n_centres: int, seed: int, n_queries: int = 0,
               sigma: float = SIGMA, chunk: int = 65536):
    """(rows float32[n, dim], queries float32[n_queries, dim]), unit rows."""
    rng = np.random.Generator(np.random.PCG64(seed))
    centres = rng.standard_normal((n_centres, dim), dtype=np.float32)

    def draw(m: int) -> np.ndarray:
        out = np.empty((m, dim), np.float32)
        for s in range(0, m, chunk):
            e = min(m, s + chunk)
            lab = rng.integers(0, n_centres, e - s)
            x = centres[lab] + np.float32(sigma) * rng.standard_normal((e - s, dim),
                                                                       dtype=np.float32)
            x /= np.linalg.norm(x, axis=1, keepdims=True).astype(np.float32)
            out[s:e] = x
        return out

    rows = draw(n)
    queries = draw(n_queries) if n_queries else np.empty((0, dim), np.float32)
    return rows, queries


CHUNK_ROWS = 131072


def mixture_torch(n: int, dim: int, n_centres: int, seed: int, n_queries: int = 0,
                  device="cuda", sigma: float = SIGMA, row_range=None):
    """Same distribution drawn on a CUDA device; returns (rows, queries) tensors.

    Rows come in fixed chunks of CHUNK_ROWS, each from its own generator seeded by
    (seed, chunk), so any row range [lo, hi) -- one shard of a row-sharded index --
    is generated identically whatever the number of shards.  Queries come from a
    separate generator; all draws share the same centres."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    centres = torch.randn(n_centres, dim, generator=g, device=device, dtype=torch.float32)

    def draw(gen, m):
        lab = torch.randint(0, n_centres, (m,), generator=gen, device=device)
        x = centres[lab] + sigma * torch.randn(m, dim, generator=gen, device=device)
        return x / x.norm(dim=1, keepdim=True)

    lo, hi = row_range if row_range is not None else (0, n)
    rows = torch.empty(max(0, hi - lo), dim, device=device, dtype=torch.float32)
    for c in range(lo // CHUNK_ROWS, (hi + CHUNK_ROWS - 1) // CHUNK_ROWS):
        cs, ce = c * CHUNK_ROWS, min(n, (c + 1) * CHUNK_ROWS)
        gc = torch.Generator(device=device)
        gc.manual_seed(seed * 1_000_003 + 7_919 * (c + 1))
        x = draw(gc, ce - cs)
        a, b = max(cs, lo), min(ce, hi)
        rows[a - lo:b - lo] = x[a - cs:b - cs]
        del x
    if n_queries:
        gq = torch.Generator(device=device)
        gq.manual_seed(seed * 1_000_003 + 1)
        queries = draw(gq, n_queries)
    else:
        queries = torch.empty(0, dim, device=device)
    return rows, queries
