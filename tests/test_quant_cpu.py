"""The oracle's restatement of the three block-quantised HNSW searches (PolarQuant INT4,
NanoQuant INT2, TurboQuant INT3 + QJL), checked on CPU against a second restatement
written here in numpy / plain Python from the same reference code:
quantize_fp32_to_block_int4/_int3/_int2 and _int8 (src/vector/kernels.mojo:1116-1842),
ref_int4/3/2_dot (src/vector/reference/quant_dots.mojo:45-102), qjl_compute_signs and the
1536-dim WHT (kernels.mojo:981-1019, 1685-1714), the LCG of the QJL signs
(src/vector/hnsw.mojo:497-509), MinHeap / MaxHeap (src/common/heap.mojo), the beam
(src/vector/reference/quant_beams_1536.mojo:20-81) and search_fp32_scored's block-quant
branches with the shared FP32 rerank (src/vector/hnsw.mojo:4052-4330)."""
import numpy as np
import pytest

from pion_b200.workloads import mixture_np

F = np.float32
BLOCK_BYTES = {"polar": 18, "nano": 10, "turbo": 14}


def round_away(q_f):
    return int(q_f + F(0.5)) if q_f >= 0 else int(q_f - F(0.5))


def py_block(kind, x):
    x = x.astype(F)
    out = bytearray(4)
    recon = F(0.0)
    qmax = {"polar": F(7.0), "nano": F(1.5), "turbo": F(3.0)}[kind]
    for b in range(48):
        blk = x[32 * b:32 * b + 32]
        absmax = F(0.0)
        for v in blk:
            av = v if v >= 0 else -v
            if av > absmax:
                absmax = av
        scale = absmax / qmax if absmax > 0 else F(1.0)
        inv = F(1.0) / scale
        if kind == "nano":
            stored = scale * F(0.5)
            out += np.float16(stored).tobytes()
            q = []
            for v in blk:
                t = min(3, max(0, round_away(v * inv + F(1.5))))
                q.append(t)
                r = F(t * 2 - 3) * stored
                recon = recon + r * r
            for g in range(8):
                out.append(q[4 * g] | q[4 * g + 1] << 2 | q[4 * g + 2] << 4 | q[4 * g + 3] << 6)
        else:
            out += np.float16(scale).tobytes()
            lo, hi = (-8, 7) if kind == "polar" else (-4, 3)
            q = []
            for v in blk:
                t = min(hi, max(lo, round_away(v * inv)))
                q.append(t)
                r = F(t) * scale
                recon = recon + r * r
            if kind == "polar":
                for i in range(16):
                    out.append(((q[i + 16] + 8) << 4) | (q[i] + 8))
            else:
                for g in range(4):
                    v = [q[8 * g + i] + 4 for i in range(8)]
                    out.append((v[0] | v[1] << 3 | (v[2] & 3) << 6) & 0xFF)
                    out.append((v[2] >> 2 | v[3] << 1 | v[4] << 4 | (v[5] & 1) << 7) & 0xFF)
                    out.append((v[5] >> 1 | v[6] << 2 | v[7] << 5) & 0xFF)
    out[0:4] = np.array([recon], F).tobytes()
    return np.frombuffer(bytes(out), np.int8)


def py_codes(kind, slot, b):
    d = slot.view(np.uint8)[4 + BLOCK_BYTES[kind] * b + 2:]
    if kind == "polar":
        return [int(d[i] & 15) - 8 for i in range(16)] + [int(d[i] >> 4) - 8 for i in range(16)]
    if kind == "nano":
        out = []
        for h in range(2):
            p = int(d[4 * h]) | int(d[4 * h + 1]) << 8 | int(d[4 * h + 2]) << 16 | int(d[4 * h + 3]) << 24
            out += [((p >> (2 * k)) & 3) * 2 - 3 for k in range(16)]
        return out
    out = []
    for g in range(4):
        u = int(d[3 * g]) | int(d[3 * g + 1]) << 8 | int(d[3 * g + 2]) << 16
        out += [((u >> (3 * k)) & 7) - 4 for k in range(8)]
    return out


def py_dot(kind, qc, qs, slot):
    total = F(0.0)
    for b in range(48):
        off = 4 + BLOCK_BYTES[kind] * b
        combined = qs[b] * F(np.frombuffer(slot[off:off + 2].tobytes(), np.float16)[0])
        acc = int(np.dot(qc[32 * b:32 * b + 32].astype(np.int64), np.array(py_codes(kind, slot, b))))
        total = total + F(acc) * combined
    return total


def py_query_block(q):
    codes = np.zeros(1536, np.int8)
    scales = np.zeros(48, F)
    recon = F(0.0)
    for b in range(48):
        blk = q[32 * b:32 * b + 32]
        absmax = F(0.0)
        for v in blk:
            av = v if v >= 0 else -v
            if av > absmax:
                absmax = av
        scale = absmax / F(127.0) if absmax > 0 else F(1.0)
        inv = F(1.0) / scale
        scales[b] = scale
        for i, v in enumerate(blk):
            t = min(127, max(-127, round_away(v * inv)))
            codes[32 * b + i] = t
            r = F(t) * scale
            recon = recon + r * r
    return codes, scales, recon


def py_random_signs():
    s, out, m = 42, [], (1 << 64) - 1
    for _ in range(24):
        bits = 0
        for b in range(64):
            s = (s * 6364136223846793005 + 1442695040888963407) & m
            if (s >> 33) & 1:
                bits |= 1 << b
        out.append(bits)
    return np.array(out, np.uint64)


def py_qjl(res, rs):
    t = np.zeros(1536, F)
    n2 = F(0.0)
    for i in range(1536):
        sv = F(1.0) if (int(rs[i >> 6]) >> (i & 63)) & 1 else F(-1.0)
        t[i] = res[i] * sv
        n2 = n2 + res[i] * res[i]
    for base in (0, 512, 1024):
        d = t[base:base + 512]
        h = 1
        while h < 512:
            for i in range(0, 512, 2 * h):
                x = d[i:i + h].copy()
                y = d[i + h:i + 2 * h].copy()
                d[i:i + h] = x + y
                d[i + h:i + 2 * h] = x - y
            h *= 2
        d *= F(0.044194173824159216)
    bits = []
    for w in range(24):
        v = 0
        for b in range(64):
            if t[w * 64 + b] > 0:
                v |= 1 << b
        bits.append(v)
    return np.array(bits, np.uint64), n2


def test_f16_rounding(oracle):
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.standard_normal(3000).astype(F) * F(1e-3),
                        rng.standard_normal(3000).astype(F) * F(40.0),
                        (rng.random(2000) * F(6e-8)).astype(F),      # subnormal halves
                        np.array([65504, 65520, 1e6, 0, -0.0, 2.0 ** -24, 3 * 2.0 ** -25], F)])
    # ties: values exactly halfway between two halves
    h = rng.integers(1, 0x7bff, 500).astype(np.uint16)
    lo = h.view(np.float16).astype(F)
    hi = (h + 1).view(np.float16).astype(F)
    x = np.concatenate([x, ((lo.astype(np.float64) + hi) / 2).astype(F)])
    with np.errstate(over="ignore"):  # 1e6 and 65520 round to +inf in float16
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(oracle.f32_to_f16_bits(x), want)


@pytest.mark.parametrize("kind", ["polar", "nano", "turbo"])
def test_blocks_and_dots(oracle, kind):
    rng = np.random.default_rng(11)
    for t in range(4):
        x = (rng.standard_normal(1536) * (0.02 if t else 3.0)).astype(F)
        x[rng.integers(0, 1536, 40)] = 0.0
        slot = oracle.quant_block(kind, x)
        assert np.array_equal(slot, py_block(kind, x))
        q = (rng.standard_normal(1536) * 0.03).astype(F)
        qc, qs, qn = oracle.query_block_int8(q)
        pc, ps, pn = py_query_block(q)
        assert np.array_equal(qc, pc) and np.array_equal(qs, ps) and qn == pn
        assert oracle.quant_dot(kind, qc, qs, slot) == py_dot(kind, qc, qs, slot)


def test_qjl_signs(oracle):
    rs = oracle.qjl_random_signs()
    assert np.array_equal(rs, py_random_signs())
    rng = np.random.default_rng(5)
    for _ in range(3):
        r = (rng.standard_normal(1536) * 0.01).astype(F)
        bits, n2 = oracle.qjl_signs(r, rs)
        pb, pn = py_qjl(r, rs)
        assert np.array_equal(bits, pb) and n2 == pn


# ------------------------------------------------------------- the search --

class PyMin:
    def __init__(self):
        self.a = []

    def push(self, d, i):
        a = self.a
        a.append([d, i])
        c = len(a) - 1
        while c > 0:
            p = (c - 1) // 2
            if a[c][0] < a[p][0]:
                a[c], a[p] = a[p], a[c]
                c = p
            else:
                break

    def pop(self):
        a = self.a
        root = a[0]
        if len(a) > 1:
            a[0] = a.pop()
            c, n = 0, len(a)
            while True:
                l, r, s = 2 * c + 1, 2 * c + 2, c
                if l < n and a[l][0] < a[s][0]:
                    s = l
                if r < n and a[r][0] < a[s][0]:
                    s = r
                if s == c:
                    break
                a[c], a[s] = a[s], a[c]
                c = s
        else:
            a.pop()
        return root


class PyMax:
    def __init__(self):
        self.a, self.worst = [], F(-1e30)

    def _up(self, c):
        a = self.a
        while c > 0:
            p = (c - 1) // 2
            if a[c][0] > a[p][0]:
                a[c], a[p] = a[p], a[c]
                c = p
            else:
                break

    def _down(self, c):
        a, n = self.a, len(self.a)
        while True:
            l, r, s = 2 * c + 1, 2 * c + 2, c
            if l < n and a[l][0] > a[s][0]:
                s = l
            if r < n and a[r][0] > a[s][0]:
                s = r
            if s == c:
                break
            a[c], a[s] = a[s], a[c]
            c = s

    def push(self, d, i):
        if d > self.worst:
            self.worst = d
        self.a.append([d, i])
        self._up(len(self.a) - 1)

    def push_bounded(self, d, i, ef):
        if len(self.a) < ef:
            self.a.append([d, i])
            self._up(len(self.a) - 1)
            if d > self.worst:
                self.worst = d
        elif d < self.worst:
            self.a[0] = [d, i]
            self._down(0)
            self.worst = self.a[0][0]

    def pop(self):
        a = self.a
        root = a[0]
        if len(a) > 1:
            a[0] = a.pop()
            self._down(0)
            self.worst = a[0][0]
        else:
            a.pop()
            self.worst = F(-1e30)
        return root


def is_del(A, i):
    d = A.get("deleted")
    return d is not None and (int(d[i >> 3]) >> (i & 7)) & 1 == 1


def py_beam(A, dist, ef, cand, res, seen):
    """quant_beam_search_1536_ref's loop over seeded heaps: deleted nodes are skipped before
    the visited test and never marked."""
    while cand.a:
        c = cand.pop()
        if c[0] > res.worst and len(res.a) >= ef:
            break
        row, srow = A["l0_compact"][c[1]], A["l0_slots"][c[1]]
        for i in range(int(row[0])):
            nidx = int(row[1 + i])
            if nidx >= A["num_nodes"] or is_del(A, nidx) or nidx in seen:
                continue
            seen.add(nidx)
            d = dist(nidx, int(srow[1 + i]))
            cand.push(d, nidx)
            res.push_bounded(d, nidx, ef)


def py_search(A, Q, kind, q, k, ef):
    comp = Q["compact"].reshape(A["num_nodes"], Q["stride"])
    slot_of = A["node_slot"]
    if A["metric"] == 1:
        import oracle
        q = oracle.l2_normalize_rows(q[None])[0]
    qc, qs, qn = py_query_block(q)
    qsig, qres = None, F(0.0)
    if kind == "turbo":
        res = np.array([q[i] - F(qc[i]) * qs[i // 32] for i in range(1536)], F)
        qsig, qres = py_qjl(res, Q["qjl_random_signs"])

    def dist(node, slot_row=None, qjl=True):
        # the greedy scores without the QJL term (hnsw.mojo:4224-4246), the beam with it
        v = comp[slot_of[node]] if slot_row is None else comp[slot_row]
        norm_v = np.frombuffer(v[:4].tobytes(), F)[0]
        dot = py_dot(kind, qc, qs, v)
        if kind != "turbo" or not qjl:
            return (qn + norm_v) - F(2.0) * dot
        ham = sum(bin(int(a) ^ int(b)).count("1") for a, b in zip(qsig, Q["qjl"][node]))
        cos_est = (F(1536) - F(2) * F(ham)) * (F(1.0) / F(1536))
        qjl_c = F(Q["qjl_lambda"]) * cos_est * (qres * Q["qjl_res_norms"][node])
        return ((qn + norm_v) - F(2.0) * dot) - F(2.0) * qjl_c

    M = A["M"]
    cur = A["entry_point"]
    cd = dist(cur, qjl=False)
    for lv in range(A["max_level"], 0, -1):
        changed = True
        while changed:
            changed = False
            nc = int(A["upper_links"][A["upper_offset"][cur] + lv - 1][0])
            for i in range(nc):
                row = A["upper_links"][A["upper_offset"][cur] + lv - 1]
                nidx = int(row[1 + i])
                if nidx >= A["num_nodes"]:
                    continue
                if kind == "nano" and is_del(A, nidx):  # NanoQuant's greedy skips them
                    continue
                d = dist(nidx, qjl=False)
                if d < cd:
                    cd, cur, changed = d, nidx, True
    cand, res, seen = PyMin(), PyMax(), {cur}
    cand.push(cd, cur)
    res.push(cd, cur)
    py_beam(A, dist, ef, cand, res, seen)
    ids, ds = [], []
    while res.a:
        r = res.pop()
        ids.append(r[1])
        ds.append(r[0])
    ids.reverse()
    ds.reverse()
    rr = Q["rerank"]
    for i, node in enumerate(ids):
        a = np.zeros(8, F)
        b = np.zeros(8, F)
        for d0 in range(0, 1536, 16):
            da = q[d0:d0 + 8] - rr[node][d0:d0 + 8]
            a = a + da * da
            db = q[d0 + 8:d0 + 16] - rr[node][d0 + 8:d0 + 16]
            b = b + db * db
        s = a + b
        while len(s) > 1:
            s = s[:len(s) // 2] + s[len(s) // 2:]
        ds[i] = s[0]
    for i in range(1, len(ds)):
        j = i
        while j > 0 and ds[j] < ds[j - 1]:
            ds[j], ds[j - 1] = ds[j - 1], ds[j]
            ids[j], ids[j - 1] = ids[j - 1], ids[j]
            j -= 1
    return [int(A["node_ids"][i]) for i in ids[:k]], [F(d) for d in ds[:k]]


@pytest.fixture(scope="module")
def qgraph():
    import pion_b200
    rows, qs = mixture_np(1500, 1536, 12, seed=41, n_queries=4)
    g = pion_b200.HNSWGraph(rows, M=8, ef_construction=40, threads=1)
    return g, g.arrays(), rows, qs


@pytest.mark.parametrize("kind", ["polar", "nano", "turbo"])
def test_quant_search_matches_python(oracle, qgraph, kind):
    g, A, rows, qs = qgraph
    Q = oracle.quant_graph(A, rows, kind)
    ids, sc, cnt = oracle.quant_search(A, Q, qs, 10, 24)
    for t in range(len(qs)):
        pi, ps = py_search(A, Q, kind, qs[t], 10, 24)
        assert cnt[t] == len(pi)
        assert list(ids[t, :cnt[t]]) == pi
        assert np.array_equal(sc[t, :cnt[t]].view(np.uint32), np.array(ps, F).view(np.uint32))


@pytest.mark.parametrize("metric", ["cosine", "l2"])
@pytest.mark.parametrize("kind", ["polar", "nano", "turbo"])
def test_library_quantizer_matches_oracle(oracle, kind, metric):
    """pion_v_b200_hnsw_quantize (host C++) writes the oracle's compact buffer, QJL rows,
    residual norms and rerank rows bit for bit."""
    import pion_b200
    rows, _ = mixture_np(700, 1536, 9, seed=43 if metric == "cosine" else 47, n_queries=1)
    rows[5] = 0.0  # a zero row passes through the normalisation
    rows[6, :32] = 0.0  # an all-zero block takes scale 1
    g = pion_b200.HNSWGraph(rows, M=6, ef_construction=32, metric=metric, threads=1)
    A = g.arrays()
    want = oracle.quant_graph(A, rows, kind)
    qz = pion_b200.HNSWQuant(g, rows, kind)
    got = qz.arrays()
    assert got["stride"] == want["stride"]
    assert np.array_equal(got["compact"], want["compact"])
    assert np.array_equal(got["rerank"].view(np.uint32), want["rerank"].view(np.uint32))
    if kind == "turbo":
        assert np.array_equal(got["qjl"], want["qjl"])
        assert np.array_equal(got["qjl_res_norms"].view(np.uint32),
                              want["qjl_res_norms"].view(np.uint32))
        assert np.array_equal(got["qjl_random_signs"], want["qjl_random_signs"])
    else:
        assert "qjl" not in got


def test_library_quantizer_refuses(qgraph):
    import pion_b200
    g, A, rows, qs = qgraph
    with pytest.raises(ValueError):
        pion_b200.HNSWQuant(g, rows, "int5")
    with pytest.raises(pion_b200.PionError):
        pion_b200.HNSWQuant(g, rows[:-1], "polar")


@pytest.mark.parametrize("kind", ["polar", "turbo"])
def test_beam_from_heaps_matches_python(oracle, qgraph, kind):
    """The oracle's beam on a view's state (orc_quant_beam_heaps: the query given as codes,
    heaps given as arrays) leaves the heaps array for array as the Python loop does, and
    cuts the candidates at a capacity."""
    g, A, rows, qs = qgraph
    Q = oracle.quant_graph(A, rows, kind)
    comp = Q["compact"].reshape(A["num_nodes"], Q["stride"])
    q = oracle.l2_normalize_rows(qs[1][None])[0] if A["metric"] == 1 else qs[1]
    qc, qsc, qn = oracle.query_block_int8(q)
    qsig, qres = None, F(0.0)
    if kind == "turbo":
        resid = np.array([q[i] - F(qc[i]) * qsc[i // 32] for i in range(1536)], F)
        qsig, qres = oracle.qjl_signs(resid, Q["qjl_random_signs"])

    def dist(node, slot_row=None, qjl=True):
        v = comp[A["node_slot"][node]] if slot_row is None else comp[slot_row]
        nv = np.frombuffer(v[:4].tobytes(), F)[0]
        d = (qn + nv) - F(2.0) * F(oracle.quant_dot(kind, qc, qsc, v))
        if kind != "turbo" or not qjl:
            return d
        ham = sum(bin(int(a) ^ int(b)).count("1") for a, b in zip(qsig, Q["qjl"][node]))
        cos_est = (F(1536) - F(2) * F(ham)) * (F(1.0) / F(1536))
        return d - F(2.0) * (F(Q["qjl_lambda"]) * cos_est * (qres * Q["qjl_res_norms"][node]))

    start = int(A["entry_point"])
    d0 = dist(start, qjl=False)
    cand, res = PyMin(), PyMax()
    cand.push(d0, start)
    res.push(d0, start)
    py_beam(A, dist, 20, cand, res, {start})
    got_c, total, got_r, worst = oracle.quant_beam_heaps(A, Q, qc, qsc, qn, qsig, qres, 20,
                                                         [(d0, start)], [(d0, start)], d0)
    assert total == len(cand.a) == len(got_c)
    assert [(np.float32(d).view(np.uint32), i) for d, i in got_c] == \
        [(np.float32(d).view(np.uint32), i) for d, i in cand.a]
    assert [(np.float32(d).view(np.uint32), i) for d, i in got_r] == \
        [(np.float32(d).view(np.uint32), i) for d, i in res.a]
    assert worst == res.worst
    cut, total2, _, _ = oracle.quant_beam_heaps(A, Q, qc, qsc, qn, qsig, qres, 20,
                                                [(d0, start)], [(d0, start)], d0, cand_cap=5)
    assert total2 == total and cut == got_c[:5]


@pytest.mark.parametrize("kind", ["polar", "nano"])
def test_quant_search_deleted_matches_python(oracle, qgraph, kind):
    """With a deletion bitmap: the beam skips deleted nodes (all kinds), NanoQuant's
    greedy skips them too (hnsw.mojo:4179), the others' greedy does not."""
    g, A, rows, qs = qgraph
    n = A["num_nodes"]
    gen = np.random.default_rng(5)
    dead = gen.choice(n, n // 6, replace=False)
    bits = np.zeros((n + 7) // 8, np.uint8)
    for i in dead:
        bits[i >> 3] |= np.uint8(1 << (i & 7))
    A2 = dict(A)
    A2["deleted"] = bits
    Q = oracle.quant_graph(A, rows, kind)
    ids, sc, cnt = oracle.quant_search(A2, Q, qs, 10, 24)
    for t in range(len(qs)):
        pi, ps = py_search(A2, Q, kind, qs[t], 10, 24)
        assert cnt[t] == len(pi)
        assert list(ids[t, :cnt[t]]) == pi
        assert np.array_equal(sc[t, :cnt[t]].view(np.uint32), np.array(ps, F).view(np.uint32))


@pytest.mark.parametrize("seed", [3, 11])
def test_quant_search_randomised_against_python(oracle, seed):
    """Small random graphs (M, ef, k, metric and kind drawn per case) with duplicated rows
    (ties in every distance): the oracle and the statement-by-statement Python restatement
    agree on ids and score bits."""
    import pion_b200
    gen = np.random.default_rng(seed)
    n = int(gen.integers(300, 700))
    rows, qs = mixture_np(n, 1536, int(gen.integers(4, 16)), seed=seed, n_queries=3)
    rows[n // 2:n // 2 + 20] = rows[:20]  # exact duplicates: equal distances
    metric = ["cosine", "l2"][seed % 2]
    g = pion_b200.HNSWGraph(rows, M=int(gen.integers(4, 9)), ef_construction=32,
                           metric=metric, threads=1)
    A = g.arrays()
    for kind in ("polar", "nano", "turbo"):
        Q = oracle.quant_graph(A, rows, kind)
        k, ef = int(gen.integers(1, 12)), int(gen.integers(1, 40))
        ids, sc, cnt = oracle.quant_search(A, Q, qs, k, ef)
        for t in range(len(qs)):
            pi, ps = py_search(A, Q, kind, qs[t], k, ef)
            assert cnt[t] == len(pi)
            assert list(ids[t, :cnt[t]]) == pi
            assert np.array_equal(sc[t, :cnt[t]].view(np.uint32),
                                  np.array(ps, F).view(np.uint32))
