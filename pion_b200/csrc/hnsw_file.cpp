// The reference's HNSW index file (pion.hnsw.0), read into and written from the host
// Graph.  Format v3 to v5 as HNSWGraph._save_body writes it and _load_body reads it
// (src/vector/hnsw.mojo:1209-1440 and 1485-1700):
//
//   header, 32 little-endian u64 (256 bytes):
//     [0] magic "PIONHNSW"  [1] version  [2] num_nodes  [3] dim  [4] M  [5] ef_construction
//     [6] entry point  [7] max level  bytes 64/68: f32 global_min / global_max
//     [9] neighbour block u32s per node (8 M + 7)  [10] max_elements  [11] name length
//     bytes 96-159: index name  [20] slot stride  [21] slot header bytes
//     [22] compact format (0 = INT8 + header)  [23] calibration groups  [24] metric
//     [25] optional sections  [26] vector field name length, bytes 216-247: the name
//     [31] build id
//   compact buffer       num_nodes x stride
//   node map             v4+: u64 count, then count x i64 (external id -> node, -1 none);
//                        v3: max_elements x i64
//   l0_compact           num_nodes x 33 u32 (count, level-0 neighbour nodes)
//   neighbour blocks     v4+: num_nodes, v3: max_elements blocks of 8 M + 7 u32:
//                        level 0 at [0, 2M), level l >= 1 at [2M + (l-1) M, +M),
//                        per-level counts at [8M, 8M + 7)
//   id + level           num_nodes x 2 i64 (external id, max level)
//   slot                 num_nodes x u32 (compact slot of each node)
//   node norms, prefix norms   num_nodes x f32 each
//   calibration groups   (only when [23] > 0) qmins and scales, f32 each
//   key records          num_nodes x 32 bytes
//   further sections flagged in [25] (FP32 rerank rows of the quantised formats, QJL,
//   prefixes, schema, long keys)
//
// The block-quantised formats ([22] = 1 INT4, 2 INT3, 4 INT2; slot header 0, stride
// 868 / 676 / 484) keep their slots in the compact buffer, write zero norms, and append
// after the key records the sections flagged in [25]: bit 0 the FP32 rerank rows
// (num_nodes x dim f32, by node), bit 1 the QJL sign rows (num_nodes x 24 u64, by node)
// then the residual norms (num_nodes x f32) (hnsw.mojo:1271-1284, 1421-1430, 1694-1712).
//
// The loader keeps what the GPU search needs (the compact slots, level-0 lists, slots,
// ids, levels and upper-level lists; for the quantised formats their sections) and
// derives l0_slots as _build_l0_slots does (hnsw.mojo:2761-2786).  Per-group calibration
// is refused: the GPU beam quantises queries with the global range.
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "hnsw_host.h"

namespace pion {
namespace hnsw {

namespace {

constexpr uint64_t kMagic = 0x574E534E4F494E50ull;  // "PIONHNSW"
constexpr int kDim = 1536;

struct File {
    FILE* f = nullptr;
    ~File() {
        if (f) fclose(f);
    }
};

bool read_all(FILE* f, void* dst, size_t bytes) {
    return bytes == 0 || fread(dst, 1, bytes, f) == bytes;
}

bool skip(FILE* f, uint64_t bytes) {
    // in steps that fit a long
    while (bytes > 0) {
        const uint64_t step = bytes > (1ull << 30) ? (1ull << 30) : bytes;
        if (fseek(f, (long)step, SEEK_CUR) != 0) return false;
        bytes -= step;
    }
    return true;
}

bool write_all(FILE* f, const void* src, size_t bytes) {
    return bytes == 0 || fwrite(src, 1, bytes, f) == bytes;
}

}  // namespace

int load_file(const char* path, Graph& g, QuantBuffers* q, std::string& why) {
    File fh;
    fh.f = fopen(path, "rb");
    if (!fh.f) {
        why = "cannot open the file";
        return -1;
    }
    FILE* f = fh.f;
    uint64_t h[32];
    if (!read_all(f, h, sizeof(h))) {
        why = "short header";
        return -3;
    }
    if (h[0] != kMagic) {
        why = "not a pion.hnsw file (magic)";
        return -1;
    }
    const uint64_t version = h[1];
    if (version < 3 || version > 5) {
        why = "format version " + std::to_string(version) + " (want 3 to 5)";
        return -3;
    }
    const int64_t n = (int64_t)h[2], dim = (int64_t)h[3], M = (int64_t)h[4];
    const int64_t entry = (int64_t)h[6], max_level = (int64_t)h[7];
    const int64_t pool_per = (int64_t)h[9], max_elem = (int64_t)h[10];
    const int64_t stride = (int64_t)h[20], slot_hdr = (int64_t)h[21];
    int qkind = -1;  // the block format of the slots, -1 = plain INT8
    if (h[22] == 1)
        qkind = kQuantPolar;
    else if (h[22] == 2)
        qkind = kQuantTurbo;
    else if (h[22] == 4)
        qkind = kQuantNano;
    else if (h[22] != 0) {
        why = "unknown compact format " + std::to_string(h[22]);
        return -3;
    }
    if (qkind >= 0 && !q) {
        why = "a block-quantised index (INT4 / INT3 / INT2): load it with its quant sections";
        return -3;
    }
    if (h[23] != 0) {
        why = "per-group calibration is not supported (the beam quantises with the global range)";
        return -3;
    }
    if (dim != kDim) {
        why = "dim " + std::to_string(dim) + " (the beam is the 1536-dim routine)";
        return -3;
    }
    if (n <= 0 || n > max_elem || n >= (int64_t)0xffffffffll) {
        why = "bad node count";
        return -1;
    }
    if (M < 1 || 2 * M > 32 || pool_per != 8 * M + 7) {
        why = "bad M or neighbour block size";
        return -3;
    }
    if (qkind < 0 && (slot_hdr != 8 || stride < slot_hdr + dim || stride % 16 != 0)) {
        why = "bad slot stride or header";
        return -3;
    }
    if (qkind >= 0 && (slot_hdr != 0 || stride != quant_stride(qkind))) {
        why = "slot stride or header does not match the block format";
        return -3;
    }
    if (entry < 0 || entry >= n || max_level < 0 || max_level > 6) {
        why = "bad entry point or level";
        return -1;
    }
    float gminmax[2];
    memcpy(gminmax, reinterpret_cast<const char*>(h) + 64, 8);

    g = Graph{};
    g.n = n;
    g.dim = dim;
    g.M = M;
    g.efc = (int64_t)h[5];
    g.id_base = 0;
    g.metric = h[24] <= 1 ? (int)h[24] : 0;
    g.gmin = gminmax[0];
    g.gmax = gminmax[1];
    g.entry = entry;
    g.max_level = (int)max_level;
    g.stride = stride;
    g.hdr = slot_hdr;
    if (q) *q = QuantBuffers{};
    std::vector<int8_t>& slots = qkind >= 0 ? q->compact : g.compact;
    slots.resize((size_t)n * stride);
    if (!read_all(f, slots.data(), slots.size())) {
        why = "short compact buffer";
        return -1;
    }
    uint64_t map_ids = (uint64_t)max_elem;
    if (version >= 4 && !read_all(f, &map_ids, 8)) {
        why = "short node map";
        return -1;
    }
    if (map_ids > (uint64_t)max_elem || !skip(f, map_ids * 8)) {
        why = "bad node map";
        return -1;
    }
    g.l0_compact.resize((size_t)n * 33);
    if (!read_all(f, g.l0_compact.data(), g.l0_compact.size() * 4)) {
        why = "short l0_compact";
        return -1;
    }
    const int64_t blocks = version < 4 ? max_elem : n;
    std::vector<uint32_t> pool((size_t)n * pool_per);
    if (!read_all(f, pool.data(), pool.size() * 4) ||
        !skip(f, (uint64_t)(blocks - n) * pool_per * 4)) {
        why = "short neighbour blocks";
        return -1;
    }
    std::vector<int64_t> id_level((size_t)n * 2);
    if (!read_all(f, id_level.data(), id_level.size() * 8)) {
        why = "short id/level section";
        return -1;
    }
    g.node_slot.resize((size_t)n);
    if (!read_all(f, g.node_slot.data(), g.node_slot.size() * 4)) {
        why = "short slot section";
        return -1;
    }
    if (qkind >= 0) {  // zero norms, key records, then the flagged sections
        const uint64_t sections = h[25];
        if (!skip(f, (uint64_t)n * 8 + (uint64_t)n * 32)) {
            why = "short norm or key sections";
            return -1;
        }
        q->kind = qkind;
        q->stride = stride;
        if (sections & 1) {
            q->rerank.resize((size_t)n * dim);
            if (!read_all(f, q->rerank.data(), q->rerank.size() * 4)) {
                why = "short FP32 rerank section";
                return -1;
            }
        }
        if (sections & 2) {
            q->qjl.resize((size_t)n * 24);
            q->qjl_res_norms.resize((size_t)n);
            if (!read_all(f, q->qjl.data(), q->qjl.size() * 8) ||
                !read_all(f, q->qjl_res_norms.data(), q->qjl_res_norms.size() * 4)) {
                why = "short QJL section";
                return -1;
            }
        }
        if (qkind == kQuantTurbo) {  // not stored: the LCG seeded 42 (hnsw.mojo:497-509)
            q->random_signs.resize(24);
            qjl_random_signs(q->random_signs.data());
        }
    } else if (q) {
        q->kind = -1;
    }
    // the rest (norms and key records of INT8 files, other sections) is not needed

    g.level.resize((size_t)n);
    g.node_ids.resize((size_t)n);
    g.upper_offset.assign((size_t)n, -1);
    for (int64_t i = 0; i < n; ++i) {
        const int64_t id = id_level[2 * i], lv = id_level[2 * i + 1];
        if (id < 0 || id > 0x7fffffffll) {
            why = "external id outside int32";
            return -3;
        }
        if (lv < 0 || lv > 6) {
            why = "node level outside [0, 6]";
            return -1;
        }
        if (g.node_slot[i] >= (uint64_t)n) {  // _load_body refuses the file too
            why = "slot index out of range";
            return -1;
        }
        g.node_ids[i] = (int32_t)id;
        g.level[i] = (int8_t)lv;
        if (g.l0_compact[(size_t)i * 33] > 32u) {
            why = "level-0 count above 32";
            return -1;
        }
    }
    // upper levels: rows of (count, M neighbours) per node level >= 1
    int64_t rows = 0;
    for (int64_t i = 0; i < n; ++i) rows += g.level[i];
    g.upper_rows = rows;
    g.upper_links.assign((size_t)rows * (1 + M), 0u);
    int64_t r = 0;
    for (int64_t i = 0; i < n; ++i) {
        if (g.level[i] == 0) continue;
        g.upper_offset[i] = r;
        const uint32_t* blk = pool.data() + (size_t)i * pool_per;
        for (int l = 1; l <= g.level[i]; ++l, ++r) {
            uint32_t cnt = blk[8 * M + l];
            if (cnt > (uint32_t)M) cnt = (uint32_t)M;
            uint32_t* row = g.upper_links.data() + (size_t)r * (1 + M);
            row[0] = cnt;
            // the whole level segment: the block-quant greedy reads positions past the
            // count of a node it moved to (bounded by the first node's count), as the
            // reference's loop reads the node's neighbour block
            for (int64_t j = 0; j < M; ++j) row[1 + j] = blk[2 * M + (l - 1) * M + j];
        }
    }
    // _build_l0_slots: the slot of every level-0 neighbour, 0xFFFFFFFF for none
    g.l0_slots.resize((size_t)n * 33);
    for (int64_t i = 0; i < n; ++i) {
        const uint32_t cnt = g.l0_compact[(size_t)i * 33];
        g.l0_slots[(size_t)i * 33] = cnt;
        for (uint32_t k = 0; k < 32; ++k) {
            const uint32_t nb = g.l0_compact[(size_t)i * 33 + 1 + k];
            g.l0_slots[(size_t)i * 33 + 1 + k] =
                k < cnt ? (nb < (uint32_t)n ? g.node_slot[nb] : 0xffffffffu) : 0u;
        }
    }
    return 0;
}

int save_file(const Graph& g, const QuantBuffers* q, const char* path, int64_t max_elements,
              std::string& why) {
    const bool quant = q && q->kind >= kQuantPolar && q->kind <= kQuantTurbo;
    if (quant && (g.n <= 0 || q->stride != quant_stride(q->kind) ||
                  q->compact.size() != (size_t)g.n * q->stride ||
                  (!q->rerank.empty() && q->rerank.size() != (size_t)g.n * g.dim) ||
                  (!q->qjl.empty() && (q->qjl.size() != (size_t)g.n * 24 ||
                                       q->qjl_res_norms.size() != (size_t)g.n)))) {
        why = "quant buffers do not match the graph";
        return -1;
    }
    if (!quant && (g.n <= 0 || g.compact.size() != (size_t)g.n * g.stride || g.hdr != 8)) {
        why = "graph has no compact layout";
        return -1;
    }
    const int64_t n = g.n, M = g.M, pool_per = 8 * M + 7;
    int64_t map_ids = 0;
    for (int64_t i = 0; i < n; ++i)
        map_ids = g.node_ids[i] + 1 > map_ids ? g.node_ids[i] + 1 : map_ids;
    if (max_elements <= 0) max_elements = map_ids > n ? map_ids : n;
    if (max_elements < n || max_elements < map_ids) {
        why = "max_elements below the node count or an external id";
        return -1;
    }
    if (M < 1 || 2 * M > 32) {
        why = "bad M";
        return -1;
    }
    File fh;
    fh.f = fopen(path, "wb");
    if (!fh.f) {
        why = "cannot create the file";
        return -1;
    }
    FILE* f = fh.f;
    uint64_t h[32];
    memset(h, 0, sizeof(h));
    h[0] = kMagic;
    h[1] = 5;
    h[2] = (uint64_t)n;
    h[3] = (uint64_t)g.dim;
    h[4] = (uint64_t)M;
    h[5] = (uint64_t)g.efc;
    h[6] = (uint64_t)g.entry;
    h[7] = (uint64_t)(g.max_level < 0 ? 0 : g.max_level);
    memcpy(reinterpret_cast<char*>(h) + 64, &g.gmin, 4);
    memcpy(reinterpret_cast<char*>(h) + 68, &g.gmax, 4);
    h[9] = (uint64_t)pool_per;
    h[10] = (uint64_t)max_elements;
    h[20] = (uint64_t)(quant ? q->stride : g.stride);
    h[21] = (uint64_t)(quant ? 0 : g.hdr);
    if (quant) {
        h[22] = q->kind == kQuantPolar ? 1 : q->kind == kQuantTurbo ? 2 : 4;
        h[25] = (q->rerank.empty() ? 0 : 1) | (q->qjl.empty() ? 0 : 2);
    }
    h[24] = (uint64_t)g.metric;
    const std::vector<int8_t>& slots = quant ? q->compact : g.compact;
    bool ok = write_all(f, h, sizeof(h)) && write_all(f, slots.data(), slots.size());
    // node map up to the highest external id
    std::vector<int64_t> map((size_t)map_ids, -1);
    for (int64_t i = 0; i < n; ++i) map[(size_t)g.node_ids[i]] = i;
    const uint64_t mc = (uint64_t)map_ids;
    ok = ok && write_all(f, &mc, 8) && write_all(f, map.data(), map.size() * 8);
    ok = ok && write_all(f, g.l0_compact.data(), (size_t)n * 33 * 4);
    // neighbour blocks
    std::vector<uint32_t> blk((size_t)pool_per);
    for (int64_t i = 0; i < n && ok; ++i) {
        std::fill(blk.begin(), blk.end(), 0u);
        uint32_t c0 = g.l0_compact[(size_t)i * 33];
        if (c0 > (uint32_t)(2 * M)) c0 = (uint32_t)(2 * M);
        for (uint32_t j = 0; j < c0; ++j) blk[j] = g.l0_compact[(size_t)i * 33 + 1 + j];
        blk[8 * M] = c0;
        for (int l = 1; l <= g.level[i]; ++l) {
            const uint32_t* row =
                g.upper_links.data() + (size_t)(g.upper_offset[i] + l - 1) * (1 + M);
            const uint32_t cnt = row[0] > (uint32_t)M ? (uint32_t)M : row[0];
            for (int64_t j = 0; j < M; ++j) blk[2 * M + (l - 1) * M + j] = row[1 + j];
            blk[8 * M + l] = cnt;
        }
        ok = write_all(f, blk.data(), blk.size() * 4);
    }
    std::vector<int64_t> id_level((size_t)n * 2);
    std::vector<float> norms((size_t)n), prefix((size_t)n);
    for (int64_t i = 0; i < n; ++i) {
        id_level[2 * i] = g.node_ids[i];
        id_level[2 * i + 1] = g.level[i];
        if (quant) continue;  // the block formats keep no node norms: zeros
        const int8_t* s = g.compact.data() + (size_t)g.node_slot[i] * g.stride;
        memcpy(&norms[i], s, 4);
        memcpy(&prefix[i], s + 4, 4);
    }
    ok = ok && write_all(f, id_level.data(), id_level.size() * 8) &&
         write_all(f, g.node_slot.data(), (size_t)n * 4) &&
         write_all(f, norms.data(), (size_t)n * 4) && write_all(f, prefix.data(), (size_t)n * 4);
    std::vector<uint8_t> keys((size_t)n * 32, 0);  // no key records: the engine's slot map
    ok = ok && write_all(f, keys.data(), keys.size());
    if (quant) {
        ok = ok && write_all(f, q->rerank.data(), q->rerank.size() * 4);
        const size_t res_bytes = q->qjl.empty() ? 0 : q->qjl_res_norms.size() * 4;
        ok = ok && write_all(f, q->qjl.data(), q->qjl.size() * 8) &&
             write_all(f, q->qjl_res_norms.data(), res_bytes);
    }
    if (!ok) {
        why = "write failed";
        return -1;
    }
    if (fflush(f) != 0) {
        why = "write failed";
        return -1;
    }
    return 0;
}

}  // namespace hnsw
}  // namespace pion
