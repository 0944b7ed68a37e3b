"""ctypes binding of libpion_vector_b200.so (the C ABI in include/pion_vector_b200.h).

The library is the product: there is no Python or CPU fallback.  Loading fails
loudly when the shared library is missing or was built without a symbol.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libpion_vector_b200.so")

OK = 0
EINVAL = -1
ENOMEM = -2
ESHAPE = -3
ENODEV = -4
ECUDA = -10
ETIMEOUT = -11
EABI = -12

MEM_HOST = 0
MEM_DEVICE = 1
MEM_DEVICE_BORROW = 2
OUT_PAIRS = 0x100
SHARD_LOCAL_BOUND = 0x200

MERGE_DESC = 1
MERGE_LISTS_MAJOR = 2
MERGE_PAIRS = 4
IPC_HANDLE_BYTES = 64

ABI_VERSION = 1

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_PP = ctypes.POINTER(ctypes.c_void_p)

# name -> (restype, argtypes); every symbol include/pion_vector_b200.h declares.
SIGNATURES = {
    "pion_v_abi_version": (_I64, []),
    "pion_v_isa": (_I64, []),
    "pion_v_pkm_scores_f32": (None, [_P, _I64, _I64, _P, _I64, _P]),
    "pion_v_pkm_rescore_f32": (None, [_P, _I64, _P, _P, _I64, _P]),
    "pion_v_pkm_scores_i8": (None, [_P, _I64, _I64, _P, _P, _P, _I64, _P]),
    "pion_v_pkm_topk_max": (_I64, [_P, _I64, _I64, _P, _P]),
    "pion_v_pkm_sort_desc": (None, [_P, _P, _I64]),
    "pion_v_pkm_combine_topk": (_I64, [_P, _P, _I64, _P, _P, _I64, _I64, _I64, _P, _P]),
    "pion_v_b200_init": (_I, [_I, _I, _PP]),
    "pion_v_b200_shutdown": (_I, [_P]),
    "pion_v_b200_set_stream": (_I, [_P, _P]),
    "pion_v_b200_sync": (_I, [_P]),
    "pion_v_b200_set_wait_budget": (_I, [_P, _I64]),
    "pion_v_b200_last_error": (ctypes.c_char_p, [_P]),
    "pion_v_b200_reserve": (_I, [_P, _I64, _I64]),
    "pion_v_b200_launch_count": (_I64, [_P]),
    "pion_v_b200_timing_enable": (_I, [_P, _I]),
    "pion_v_b200_timing_read": (_I, [_P, ctypes.POINTER(ctypes.c_double),
                                     ctypes.POINTER(ctypes.c_int64)]),
    "pion_v_b200_timing_read_tag": (_I, [_P, _I, ctypes.POINTER(ctypes.c_double),
                                         ctypes.POINTER(ctypes.c_int64)]),
    "pion_v_b200_register_flat_i8": (_I, [_P, _P, _P, _I64, _I64, _I64, _I, _PP]),
    "pion_v_b200_flat_i8_knn": (_I, [_P, _P, _P, _P, _I64, _I64, _P, _P, _I]),
    "pion_v_b200_flat_i8_knn_static": (_I, [_P, _P, _I64, _I64, _P, _P, _I64, _I64, _P, _P,
                                            _P]),
    "pion_v_b200_register_flat_f32": (_I, [_P, _P, _I64, _I64, _I64, _I, _I, _PP]),
    "pion_v_b200_flat_f32_knn": (_I, [_P, _P, _P, _I64, _I64, _P, _P, _I]),
    "pion_v_b200_register_bq": (_I, [_P, _P, _I64, _I64, _I64, _I, _I, _PP]),
    "pion_v_b200_bq_rerank_knn": (_I, [_P, _P, _P, _I64, _I64, _I64, _P, _P, _I]),
    "pion_v_b200_index_free": (_I, [_P]),
    "pion_v_b200_index_rows": (_I64, [_P]),
    "pion_v_b200_quantize_rows_i8": (_I, [_P, _P, _I64, _I64, _I64, _P, _P, _I]),
    "pion_v_b200_l2_normalize_rows": (_I, [_P, _P, _I64, _I64, _P, _I]),
    "pion_v_b200_merge_topk": (_I, [_P, _P, _P, _I64, _I64, _I64, _I, _P, _P, _I]),
    "pion_v_b200_exchange_create": (_I, [_P, _I, _I, _I, _I64, _I64, _PP]),
    "pion_v_b200_exchange_handle": (_I, [_P, _P]),
    "pion_v_b200_exchange_connect": (_I, [_P, _P]),
    "pion_v_b200_exchange_world": (_I, [_P]),
    "pion_v_b200_exchange_free": (_I, [_P]),
    "pion_v_b200_exchange_merge": (_I, [_P, _P, _P, _I64, _I64, ctypes.c_uint32, _I, _P, _P]),
    "pion_v_b200_flat_i8_knn_sharded": (_I, [_P, _P, _P, _P, _P, _I64, _I64, ctypes.c_uint32,
                                             _I, _P, _P]),
    "pion_v_b200_hnsw_build": (_I, [_P, _I64, _I64, _I64, _I64, _I, _I64, _I, _PP]),
    "pion_v_b200_hnsw_build_batched": (_I, [_P, _I64, _I64, _I64, _I64, _I, _I64, _I, _I64,
                                            _PP]),
    "pion_v_b200_hnsw_graph_layout": (_I, [_P, _P]),
    "pion_v_b200_hnsw_graph_stats": (_I, [_P, _P]),
    "pion_v_b200_hnsw_graph_stats6": (_I, [_P, _P]),
    "pion_v_b200_hnsw_build_gpu": (_I, [_P, _P, _I64, _I64, _I64, _I64, _I, _I64, _I, _I64,
                                        _PP]),
    "pion_v_b200_hnsw_graph_free": (_I, [_P]),
    "pion_v_b200_register_hnsw": (_I, [_P, _P, _PP]),
    "pion_v_b200_hnsw_search": (_I, [_P, _P, _P, _I64, _I64, _I64, _P, _P, _I]),
    "pion_v_b200_hnsw_last_stats": (_I, [_P, _P]),
    "pion_v_b200_hnsw_metric_scores": (_I, [_P, _P, _P, _I64, _I64, _P, _P, _I]),
    "pion_v_b200_register_index": (_I, [_P, _P, _P]),
    "pion_v_b200_merge_delta": (_I, [_P, _P, _I64, _I, _P, _I64, _I64, _P, _P, _I64, _P, _P, _I]),
    "pion_v_b200_hnsw_load": (_I, [ctypes.c_char_p, _P]),
    "pion_v_b200_hnsw_save": (_I, [_P, ctypes.c_char_p, _I64]),
    "pion_v_b200_hnsw_beam_batch": (_I, [_P, _P, _P, _P, _I64, _I64, _P, _P, _P, _I]),
    "pion_v_b200_slot_scan_topk": (_I, [_P, _P, _P, _P, _I64, _I64, _I64, _P, _P, _I]),
    "pion_v_b200_hnsw_set_rerank_rows": (_I, [_P, _P, _P, _I64, _I64, _I]),
    "pion_v_b200_slot_last_stats": (_I, [_P, _P]),
    "pion_v_b200_hnsw_brute_force": (_I, [_P, _P, _P, _I64, _I64, _P, _P, _P, _I]),
    "pion_v_beam_1536": (_I64, [_P]),
    "pion_v_quant_beam_1536": (_I64, [_P]),
    "pion_v_b200_hnsw_quantize": (_I, [_P, _P, _I64, _I, _PP]),
    "pion_v_b200_hnsw_quant_layout": (_I, [_P, _P]),
    "pion_v_b200_hnsw_quant_free": (_I, [_P]),
    "pion_v_b200_register_hnsw_quant": (_I, [_P, _P, _P, _PP]),
    "pion_v_b200_hnsw_load_quant": (_I, [ctypes.c_char_p, _P, _P]),
    "pion_v_b200_hnsw_save_quant": (_I, [_P, _P, ctypes.c_char_p, _I64]),
    "pion_v_b200_hnsw_quant_search": (_I, [_P, _P, _P, _I64, _I64, _I64, _P, _P, _P, _I]),
    "pion_v_b200_beam_forget": (_I, [_P]),
}


class IndexDesc(ctypes.Structure):
    """pion_b200_index_desc (include/pion_vector_b200.h)."""
    _fields_ = [("kind", ctypes.c_int32), ("mem", ctypes.c_int32), ("n_rows", ctypes.c_int64),
                ("dim", ctypes.c_int64), ("id_base", ctypes.c_int64),
                ("normalize", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("rows", ctypes.c_void_p), ("row_scale", ctypes.c_void_p),
                ("hnsw", ctypes.c_void_p), ("quant", ctypes.c_void_p)]


class HnswQuantLayout(ctypes.Structure):
    """pion_b200_hnsw_quant_layout (include/pion_vector_b200.h)."""
    _fields_ = [("kind", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("num_nodes", ctypes.c_int64), ("compact", ctypes.c_void_p),
                ("stride", ctypes.c_int64), ("qjl", ctypes.c_void_p),
                ("qjl_res_norms", ctypes.c_void_p), ("qjl_random_signs", ctypes.c_void_p),
                ("qjl_lambda", ctypes.c_float), ("reserved2", ctypes.c_int32),
                ("rerank", ctypes.c_void_p)]


class LinearPool(ctypes.Structure):
    """pion_linear_pool (include/pion_vector_b200.h): LinearPool's fields in order."""
    _fields_ = [("entries", ctypes.c_void_p), ("capacity", ctypes.c_int64),
                ("size", ctypes.c_int64), ("cursor", ctypes.c_int64), ("ef", ctypes.c_int64)]


class BeamView1536(ctypes.Structure):
    """pion_beam_view_1536 (include/pion_vector_b200.h): BeamView1536's fields in order."""
    _fields_ = [("pool", ctypes.POINTER(LinearPool)), ("ef", ctypes.c_int64),
                ("query_norm_sq", ctypes.c_float), ("query_prefix_norm_sq", ctypes.c_float),
                ("query_int8", ctypes.c_void_p), ("l0_compact", ctypes.c_void_p),
                ("l0_slots", ctypes.c_void_p), ("num_nodes", ctypes.c_int64),
                ("deleted", ctypes.c_void_p), ("visited", ctypes.c_void_p),
                ("cur_epoch", ctypes.c_uint16), ("compact_buffer", ctypes.c_void_p),
                ("compact_stride", ctypes.c_int64), ("compact_hdr", ctypes.c_int64),
                ("nodes", ctypes.c_void_p)]


class HeapNode(ctypes.Structure):
    """pion_heap_node (include/pion_vector_b200.h): HeapNode's layout."""
    _fields_ = [("distance", ctypes.c_float), ("pad", ctypes.c_int32), ("id", ctypes.c_int64)]


class HeapList(ctypes.Structure):
    """pion_heap_list: the List[HeapNode] of MinHeap / MaxHeap (data, length, capacity)."""
    _fields_ = [("data", ctypes.c_void_p), ("len", ctypes.c_int64), ("capacity", ctypes.c_int64)]


class MinHeap(ctypes.Structure):
    _fields_ = [("data", HeapList)]


class MaxHeap(ctypes.Structure):
    _fields_ = [("data", HeapList), ("cached_worst", ctypes.c_float), ("pad", ctypes.c_int32)]


class QuantBeamView1536(ctypes.Structure):
    """pion_quant_beam_view_1536 (include/pion_vector_b200.h): QuantBeamView1536's fields
    in order."""
    _fields_ = [("kind", ctypes.c_int64), ("ef", ctypes.c_int64),
                ("candidates", ctypes.POINTER(MinHeap)), ("results", ctypes.POINTER(MaxHeap)),
                ("query_block_int8", ctypes.c_void_p), ("query_block_scales", ctypes.c_void_p),
                ("query_block_norm", ctypes.c_float), ("l0_compact", ctypes.c_void_p),
                ("l0_slots", ctypes.c_void_p), ("num_nodes", ctypes.c_int64),
                ("deleted", ctypes.c_void_p), ("visited", ctypes.c_void_p),
                ("cur_epoch", ctypes.c_uint16), ("compact_buffer", ctypes.c_void_p),
                ("compact_stride", ctypes.c_int64), ("compact_hdr", ctypes.c_int64),
                ("nodes", ctypes.c_void_p), ("qjl_buffer", ctypes.c_void_p),
                ("qjl_res_norms", ctypes.c_void_p), ("qjl_query_signs", ctypes.c_void_p),
                ("qjl_query_res_norm", ctypes.c_float), ("qjl_lambda", ctypes.c_float)]


class HnswLayout(ctypes.Structure):
    """pion_b200_hnsw_layout (include/pion_vector_b200.h)."""
    _fields_ = [
        ("num_nodes", ctypes.c_int64), ("dim", ctypes.c_int64), ("M", ctypes.c_int64),
        ("entry_point", ctypes.c_int64), ("max_level", ctypes.c_int64),
        ("global_min", ctypes.c_float), ("global_max", ctypes.c_float),
        ("metric", ctypes.c_int32), ("reserved", ctypes.c_int32),
        ("compact_buffer", ctypes.c_void_p), ("compact_stride", ctypes.c_int64),
        ("compact_hdr", ctypes.c_int64), ("l0_compact", ctypes.c_void_p),
        ("l0_slots", ctypes.c_void_p), ("node_slot", ctypes.c_void_p),
        ("node_ids", ctypes.c_void_p), ("deleted", ctypes.c_void_p),
        ("node_level", ctypes.c_void_p), ("upper_offset", ctypes.c_void_p),
        ("upper_links", ctypes.c_void_p), ("upper_rows", ctypes.c_int64),
    ]

_lock = threading.Lock()
_lib = None


class PionError(RuntimeError):
    """A negative status from the library, with its message."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"pion_vector_b200 error {code}: {msg}")
        self.code = code


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the shared library and bind every declared symbol (raises if absent)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise ImportError(
                f"{path} is missing: build it with `python -m pion_b200.build` "
                "(the CUDA library is required; there is no CPU fallback)")
        lib = ctypes.CDLL(path)
        missing = []
        for name, (res, args) in SIGNATURES.items():
            try:
                fn = getattr(lib, name)
            except AttributeError:
                missing.append(name)
                continue
            fn.restype = res
            fn.argtypes = args
        if missing:
            raise ImportError(f"{path} lacks symbols: {', '.join(missing)}")
        _lib = lib
        return lib
