"""The reference's index file pion.hnsw.0 (src/vector/hnsw.mojo:1209-1700) read and written
by the library's host code, on CPU.  A second writer restated here in Python from
_save_body (hnsw.mojo:1209-1440) produces files the library has not written itself
(versions 3 and 4, an index name, a larger capacity, key records), so the loader is
checked against the format rather than against its own writer."""
import os
import struct

import numpy as np
import pytest

from pion_b200.workloads import mixture_np

MAGIC = 0x574E534E4F494E50


@pytest.fixture(scope="module")
def built():
    import pion_b200
    rows, qs = mixture_np(2500, 1536, 24, seed=29, n_queries=32)
    g = pion_b200.HNSWGraph(rows, M=8, ef_construction=48, threads=1)
    return g, g.arrays(), rows, qs


def _blocks(A):
    """Per node the reference's neighbour block: level 0 at [0, 2M), level l at
    [2M + (l-1) M, +M), counts at [8M, 8M + 7)."""
    n, M = A["num_nodes"], A["M"]
    per = 8 * M + 7
    blk = np.zeros((n, per), np.uint32)
    l0 = A["l0_compact"]
    for i in range(n):
        c = int(l0[i, 0])
        blk[i, :c] = l0[i, 1:1 + c]
        blk[i, 8 * M] = c
        for lv in range(1, int(A["node_level"][i]) + 1):
            row = A["upper_links"][A["upper_offset"][i] + lv - 1]
            c = int(row[0])
            blk[i, 2 * M + (lv - 1) * M:2 * M + (lv - 1) * M + c] = row[1:1 + c]
            blk[i, 8 * M + lv] = c
    return blk


def write_reference_file(path, A, version=5, max_elements=None, name=b"idx", groups=0,
                         fmt=0, magic=MAGIC, truncate=None):
    """_save_body's byte layout (hnsw.mojo:1209-1440), restated."""
    n, M, stride = A["num_nodes"], A["M"], A["compact_stride"]
    ids = A["node_ids"].astype(np.int64)
    max_el = max_elements or int(ids.max()) + 1
    h = np.zeros(32, np.uint64)
    h[0], h[1], h[2], h[3], h[4], h[5] = magic, version, n, A["dim"], M, 48
    h[6], h[7] = A["entry_point"], A["max_level"]
    h[9], h[10], h[11] = 8 * M + 7, max_el, len(name)
    h[20], h[21], h[22], h[23], h[24] = stride, A["compact_hdr"], fmt, groups, A["metric"]
    hb = bytearray(h.tobytes())
    hb[64:72] = struct.pack("<ff", A["global_min"], A["global_max"])
    hb[96:96 + len(name)] = name
    out = bytearray(hb)
    out += np.ascontiguousarray(A["compact_buffer"]).tobytes()
    node_map = np.full(max_el if version < 4 else int(ids.max()) + 1, -1, np.int64)
    node_map[ids] = np.arange(n)
    if version >= 4:
        out += struct.pack("<Q", len(node_map))
    out += node_map.tobytes()
    out += np.ascontiguousarray(A["l0_compact"]).tobytes()
    blk = _blocks(A)
    if version < 4:  # v3: every element's block
        blk = np.concatenate([blk, np.zeros((max_el - n, blk.shape[1]), np.uint32)])
    out += blk.tobytes()
    idl = np.stack([ids, A["node_level"].astype(np.int64)], axis=1)
    out += idl.tobytes()
    out += np.ascontiguousarray(A["node_slot"]).tobytes()
    comp = A["compact_buffer"].reshape(n, stride)
    norms = comp[A["node_slot"], :8].copy().view(np.float32)
    out += np.ascontiguousarray(norms[:, 0]).tobytes() + np.ascontiguousarray(norms[:, 1]).tobytes()
    if groups:
        out += np.zeros(2 * groups, np.float32).tobytes()
    keys = np.zeros((n, 32), np.uint8)
    keys[:, 0] = 3
    keys[:, 1:4] = np.frombuffer(b"doc", np.uint8)
    out += keys.tobytes()
    if truncate:
        out = out[:truncate]
    with open(path, "wb") as f:
        f.write(out)


def _same_graph(A, B):
    for k in ("num_nodes", "dim", "M", "entry_point", "max_level", "compact_stride",
              "compact_hdr", "metric", "upper_rows"):
        assert A[k] == B[k], k
    assert np.float32(A["global_min"]) == np.float32(B["global_min"])
    assert np.float32(A["global_max"]) == np.float32(B["global_max"])
    for k in ("compact_buffer", "l0_compact", "l0_slots", "node_slot", "node_ids", "node_level",
              "upper_offset", "upper_links"):
        assert np.array_equal(A[k], B[k]), k


def test_save_load_round_trip(built, tmp_path):
    import pion_b200
    g, A, rows, qs = built
    p = str(tmp_path / "pion.hnsw.0")
    g.save(p)
    G = pion_b200.HNSWGraph.load(p)
    _same_graph(A, G.arrays())
    with open(p, "rb") as f:  # the v5 header the engine checks
        h = np.frombuffer(f.read(256), np.uint64)
    assert h[0] == MAGIC and h[1] == 5 and h[9] == 8 * A["M"] + 7 and h[22] == 0


@pytest.mark.parametrize("version", [3, 4, 5])
def test_load_reference_layout(built, tmp_path, version, oracle):
    """Files in the reference's layout written by the restated _save_body load into the
    same graph, and the restated beam answers the same on both."""
    import pion_b200
    g, A, rows, qs = built
    p = str(tmp_path / f"v{version}.hnsw")
    write_reference_file(p, A, version=version, max_elements=4000)
    G = pion_b200.HNSWGraph.load(p)
    B = G.arrays()
    _same_graph(A, B)
    i0, d0, _ = oracle.hnsw_search(A, qs, 10, 32)
    i1, d1, _ = oracle.hnsw_search(B, qs, 10, 32)
    assert np.array_equal(i0, i1) and np.array_equal(d0, d1)


@pytest.mark.parametrize("bad", ["magic", "version2", "quant", "groups", "truncated"])
def test_load_refuses(built, tmp_path, bad):
    import pion_b200
    g, A, rows, qs = built
    p = str(tmp_path / "bad.hnsw")
    kw = {"magic": dict(magic=0x1234), "version2": dict(version=2), "quant": dict(fmt=1),
          "groups": dict(groups=48), "truncated": dict(truncate=300000)}[bad]
    write_reference_file(p, A, **kw)
    with pytest.raises(pion_b200.PionError) as e:
        pion_b200.HNSWGraph.load(p)
    assert e.value.code in (-1, -3)
    with pytest.raises(pion_b200.PionError):
        pion_b200.HNSWGraph.load(str(tmp_path / "missing.hnsw"))
    assert not os.path.exists(str(tmp_path / "missing.hnsw"))
