// Host-side HNSW graph in the reference's compact level-0 layout (the buffers that
// src/vector/hnsw.mojo:2761-2990 builds and src/vector/beam_view.mojo:11-26 hands to
// the beam), plus the upper levels.  Built by hnsw_build.cpp.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace pion {
namespace hnsw {

struct Graph {
    int64_t n = 0, dim = 0, M = 0, efc = 0, id_base = 0;
    int metric = 0;  // 0 = L2, 1 = COSINE
    float gmin = 0.0f, gmax = 0.0f;
    int64_t entry = -1;
    int max_level = -1;
    std::vector<int8_t> level;  // per node
    std::vector<int8_t> codes;  // n x dim in node order (released after compaction)
    // compact layout
    int64_t stride = 0, hdr = 8;
    std::vector<int8_t> compact;          // n x stride, BFS slot order
    std::vector<uint32_t> l0_compact;     // n x 33: count, <= 32 level-0 neighbour nodes
    std::vector<uint32_t> l0_slots;       // n x 33: count, their compact slots
    std::vector<uint32_t> node_slot;      // n
    std::vector<int32_t> node_ids;        // n: external id of each node
    std::vector<int64_t> upper_offset;    // n: first upper row of the node, -1 at level 0
    std::vector<uint32_t> upper_links;    // rows of (1 + M): count, <= M neighbour nodes
    int64_t upper_rows = 0;
};

struct BuildStats {
    int64_t lanes = 0;
    int64_t link_drops = 0;
    int64_t relinked = 0;
    int64_t repaired_exits = 0;
    int64_t repaired_links = 0;
    int64_t planned_elsewhere = 0;  // nodes a BatchPlanner planned
};

// The search half of one node's insertion (greedy descent, _search_layer_mt at
// efConstruction, _prune_neighbors on every level it joins): the pruned neighbours per
// level, from the top level `top` down to 0, level l's at [offs[k], offs[k + 1]) with k
// counted from the top, and their distances (exact INT8 L2) to the node.
struct BuildPlan {
    std::vector<uint32_t> ids;
    std::vector<float> d;
    std::vector<uint32_t> offs;
    int top = -1;
};

// Plans whole batches of insertions elsewhere (a GPU), identically to the host's plan.
// The builder keeps every node's lists in one array: node i's level-l list (capacity 2M at
// level 0, M above) starts at link_base[i] + (l == 0 ? 0 : 2M + (l - 1) M), its count at
// cnt_base[i] + l.
class BatchPlanner {
  public:
    virtual ~BatchPlanner() {}
    // Once, before any batch: codes (n x dim, node order), levels, list layout, the
    // greedy descent's dequantisation (x = c * scale + offset), the largest batch.
    virtual int begin(const Graph& g, const int8_t* codes, const int64_t* link_base,
                      const int64_t* cnt_base, int64_t n_links, int64_t n_counts, float scale,
                      float offset, int64_t max_batch) = 0;
    // Node blocks (all its lists and counts) that changed since the last call.
    virtual int update(const int64_t* nodes, int64_t count, const uint32_t* links,
                       const uint32_t* counts) = 0;
    // Plans for nodes ids[0..count) against the graph as last updated; rows[j] is the fp32
    // row node ids[j] is linked with (normalised under COSINE).  Nonzero: plan on the host.
    virtual int plan(const int64_t* ids, int64_t count, const float* rows,
                     std::vector<BuildPlan>& out) = 0;
};

// Builds the graph of n rows (fp32, n x dim, normalised first under COSINE) with the
// reference's parameters; node i gets external id id_base + i.  n_threads link lanes, or
// with max_batch > 0 batched insertion (deterministic; n_threads plan each batch).  With a
// planner, batches of at least planner_min nodes are planned by it (the graph is the
// same).
int build(const float* rows, int64_t n, int64_t dim, int64_t M, int64_t efc, int metric,
          int64_t id_base, int n_threads, Graph& g, BuildStats* stats, int64_t max_batch = 0,
          BatchPlanner* planner = nullptr, int64_t planner_min = 64);

// Block-quantised slot formats (the reference's PolarQuant / NanoQuant / TurboQuant
// compact_vectors): kinds, and the buffers quantize() fills from the rows the graph was
// built from (normalised first under COSINE).
constexpr int kQuantPolar = 0;  // INT4, stride 868
constexpr int kQuantNano = 1;   // INT2, stride 484
constexpr int kQuantTurbo = 2;  // INT3 + QJL, stride 676

struct QuantBuffers {
    int kind = 0;
    int64_t stride = 0;
    std::vector<int8_t> compact;        // n x stride, the graph's slot order
    std::vector<uint64_t> qjl;          // TurboQuant: n x 24 sign words, by node
    std::vector<float> qjl_res_norms;   // by node
    std::vector<uint64_t> random_signs; // 24 words
    std::vector<float> rerank;          // n x 1536 FP32 rows by node
};

int64_t quant_stride(int kind);
void qjl_random_signs(uint64_t* out24);
int quantize(const Graph& g, const float* rows, int kind, QuantBuffers& out, std::string& why);

// The reference's index file (pion.hnsw.0, format v3 to v5, src/vector/hnsw.mojo:
// 1209-1700): load into a Graph (0, or -1 / -3 with the reason), and save a Graph as v5.
// A block-quantised file needs `q` (its slots, rerank rows and QJL sections go there; kind
// -1 after an INT8 file); save writes the block format of `q` when it has one.
int load_file(const char* path, Graph& g, QuantBuffers* q, std::string& why);
int save_file(const Graph& g, const QuantBuffers* q, const char* path, int64_t max_elements,
              std::string& why);

}  // namespace hnsw
}  // namespace pion

// The objects behind the C handles pion_b200_hnsw_graph and pion_b200_hnsw_quant.
struct pion_b200_hnsw_graph {
    pion::hnsw::Graph g;
    pion::hnsw::BuildStats stats;
};

struct pion_b200_hnsw_quant {
    pion::hnsw::QuantBuffers q;
    int64_t n = 0;
};
