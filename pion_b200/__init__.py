"""pion_b200 — B200-native FT.SEARCH KNN scoring and top-k for Pion.

The compute lives in ``libpion_vector_b200.so`` (hand-written sm_100a CUDA behind
the C ABI in ``include/pion_vector_b200.h``); this package holds its Python host
API (``search``), the build recipe (``build``) and the synthetic workload
generator (``workloads``).
"""
from ._lib import PionError, load  # noqa: F401
from .search import (  # noqa: F401
    BQIndex,
    Context,
    FlatF32Index,
    FlatI8Index,
    HNSWGraph,
    HNSWIndex,
    HNSWQuant,
    HNSWQuantIndex,
    l2_normalize_rows,
    merge_topk,
    merge_topk_pairs,
    quantize_rows_i8,
    rescore_knn,
)

__all__ = ["Context", "FlatI8Index", "FlatF32Index", "BQIndex", "HNSWGraph", "HNSWIndex",
           "HNSWQuant", "HNSWQuantIndex", "quantize_rows_i8",
           "l2_normalize_rows", "merge_topk", "merge_topk_pairs", "rescore_knn", "PionError", "load"]
