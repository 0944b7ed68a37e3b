"""The reference's index file pion.hnsw.0 (src/vector/hnsw.mojo:1209-1700) read and written
by the library's host code, on CPU.  A second writer restated here in Python from
_save_body (hnsw.mojo:1209-1440) produces files the library has not written itself
(versions 3 and 4, an index name, a larger capacity, key records, the block-quantised
formats with their rerank and QJL sections), so the loader is checked against the format
rather than against its own writer."""
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


QFMT = {"polar": 1, "turbo": 2, "nano": 4}


def write_reference_file(path, A, version=5, max_elements=None, name=b"idx", groups=0,
                         fmt=0, magic=MAGIC, truncate=None, quant=None, stride=None):
    """_save_body's byte layout (hnsw.mojo:1209-1440), restated; with `quant` (arrays of a
    block format) the slots are the block slots (header 0), the node norms zeros, and the
    rerank / QJL sections flagged in word 25 follow the key records (:1271-1284,
    1421-1430)."""
    n, M = A["num_nodes"], A["M"]
    stride = stride or (quant["stride"] if quant is not None else A["compact_stride"])
    ids = A["node_ids"].astype(np.int64)
    max_el = max_elements or int(ids.max()) + 1
    h = np.zeros(32, np.uint64)
    h[0], h[1], h[2], h[3], h[4], h[5] = magic, version, n, A["dim"], M, 48
    h[6], h[7] = A["entry_point"], A["max_level"]
    h[9], h[10], h[11] = 8 * M + 7, max_el, len(name)
    if quant is not None:
        fmt = fmt or QFMT[quant["kind"]]
        h[25] = (1 if quant.get("rerank") is not None else 0) | \
            (2 if quant.get("qjl") is not None else 0)
    h[20], h[21], h[22], h[23], h[24] = stride, 0 if quant is not None else A["compact_hdr"], \
        fmt, groups, A["metric"]
    hb = bytearray(h.tobytes())
    hb[64:72] = struct.pack("<ff", A["global_min"], A["global_max"])
    hb[96:96 + len(name)] = name
    out = bytearray(hb)
    out += np.ascontiguousarray(quant["compact"] if quant is not None
                                else A["compact_buffer"]).tobytes()
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
    if quant is not None:
        out += np.zeros(2 * n, np.float32).tobytes()
    else:
        comp = A["compact_buffer"].reshape(n, stride)
        norms = comp[A["node_slot"], :8].copy().view(np.float32)
        out += np.ascontiguousarray(norms[:, 0]).tobytes() + \
            np.ascontiguousarray(norms[:, 1]).tobytes()
    if groups:
        out += np.zeros(2 * groups, np.float32).tobytes()
    keys = np.zeros((n, 32), np.uint8)
    keys[:, 0] = 3
    keys[:, 1:4] = np.frombuffer(b"doc", np.uint8)
    out += keys.tobytes()
    if quant is not None:
        if quant.get("rerank") is not None:
            out += np.ascontiguousarray(quant["rerank"], np.float32).tobytes()
        if quant.get("qjl") is not None:
            out += np.ascontiguousarray(quant["qjl"], np.uint64).tobytes()
            out += np.ascontiguousarray(quant["qjl_res_norms"], np.float32).tobytes()
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


# ------------------------------------------------------- block-quantised files --

def _same_quant(G, Q, B, P):
    """Graph arrays (the INT8 slot keys aside) and quant arrays equal."""
    for k in ("num_nodes", "dim", "M", "entry_point", "max_level", "metric", "upper_rows"):
        assert G[k] == B[k], k
    for k in ("l0_compact", "l0_slots", "node_slot", "node_ids", "node_level", "upper_offset",
              "upper_links"):
        assert np.array_equal(G[k], B[k]), k
    assert Q["kind"] == P["kind"] and Q["stride"] == P["stride"]
    assert np.array_equal(Q["compact"], P["compact"])
    assert np.array_equal(Q["rerank"].view(np.uint32), P["rerank"].view(np.uint32))
    for k in ("qjl", "qjl_random_signs"):
        assert (k in Q) == (k in P)
        if k in Q:
            assert np.array_equal(Q[k], P[k]), k
    if "qjl_res_norms" in Q:
        assert np.array_equal(Q["qjl_res_norms"].view(np.uint32),
                              P["qjl_res_norms"].view(np.uint32))


@pytest.mark.parametrize("kind", ["polar", "nano", "turbo"])
def test_quant_file_round_trip(built, tmp_path, kind, oracle):
    """A graph saved with its block slots loads back into the same graph and buffers, and
    the restated quant search answers the same on both."""
    import pion_b200
    g, A, rows, qs = built
    qz = pion_b200.HNSWQuant(g, rows, kind)
    Q = qz.arrays()
    p = str(tmp_path / f"{kind}.hnsw")
    g.save(p, quant=qz)
    with open(p, "rb") as f:
        h = np.frombuffer(f.read(256), np.uint64)
    assert h[22] == QFMT[kind] and h[21] == 0 and h[20] == Q["stride"]
    assert h[25] == (3 if kind == "turbo" else 1)
    G2, q2 = pion_b200.HNSWGraph.load_quant(p)
    B, P = G2.arrays(), q2.arrays()
    _same_quant(A, Q, B, P)
    i0, s0, n0 = oracle.quant_search(A, Q, qs, 10, 32)
    i1, s1, n1 = oracle.quant_search(B, P, qs, 10, 32)
    assert np.array_equal(i0, i1) and np.array_equal(s0.view(np.uint32), s1.view(np.uint32))
    with pytest.raises(pion_b200.PionError) as e:  # the INT8 loader refuses it
        pion_b200.HNSWGraph.load(p)
    assert e.value.code == -3


@pytest.mark.parametrize("kind", ["polar", "turbo"])
def test_quant_file_reference_layout(built, tmp_path, kind):
    """Files in the reference's layout with block slots (restated writer) load into the
    library's graph and buffers; without sections the buffers stay empty."""
    import pion_b200
    g, A, rows, qs = built
    qz = pion_b200.HNSWQuant(g, rows, kind)
    Q = qz.arrays()
    p = str(tmp_path / f"ref_{kind}.hnsw")
    write_reference_file(p, A, quant=Q, max_elements=4000)
    G2, q2 = pion_b200.HNSWGraph.load_quant(p)
    _same_quant(A, Q, G2.arrays(), q2.arrays())
    bare = {"kind": kind, "stride": Q["stride"], "compact": Q["compact"]}
    write_reference_file(p, A, quant=bare, version=4)
    G3, q3 = pion_b200.HNSWGraph.load_quant(p)
    P3 = q3.arrays()
    assert P3["rerank"] is None and "qjl" not in P3
    assert np.array_equal(P3["compact"], Q["compact"])
    # a plain INT8 file through the same call: no quant buffers
    write_reference_file(p, A)
    G5, q5 = pion_b200.HNSWGraph.load_quant(p)
    assert q5 is None
    _same_graph(A, G5.arrays())


@pytest.mark.parametrize("bad", ["two_formats", "stride", "truncated_qjl", "truncated_rerank"])
def test_quant_file_refuses(built, tmp_path, bad):
    import pion_b200
    g, A, rows, qs = built
    qz = pion_b200.HNSWQuant(g, rows, "turbo")
    Q = qz.arrays()
    p = str(tmp_path / "bad.hnsw")
    n = A["num_nodes"]
    kw = {"two_formats": dict(fmt=3), "stride": dict(stride=868),
          "truncated_qjl": dict(truncate=-(n * 4 + 100)),  # inside the QJL rows
          "truncated_rerank": dict(truncate=-(n * 196 + 100))}[bad]
    if "truncate" in kw:
        write_reference_file(p, A, quant=Q)
        with open(p, "rb") as f:
            data = f.read()
        with open(p, "wb") as f:
            f.write(data[:len(data) + kw["truncate"]])
    else:
        write_reference_file(p, A, quant=Q, **kw)
    with pytest.raises(pion_b200.PionError) as e:
        pion_b200.HNSWGraph.load_quant(p)
    assert e.value.code in (-1, -3)
