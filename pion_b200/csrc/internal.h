// Host-side declarations shared by the .cu files of libpion_vector_b200: the
// context and index objects behind the opaque C handles, and the kernel launchers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "../../include/pion_vector_b200.h"

namespace pion {

// Default budget of a device-side wait (ns): kernels finish in milliseconds, so two
// seconds without progress means a stuck pipeline.
constexpr uint64_t kDefaultWaitNs = 2000000000ull;

// A grow-only device buffer.
struct DevBuf {
    void* ptr = nullptr;
    size_t bytes = 0;
};

enum IndexKind { kFlatI8 = 1, kFlatF32 = 2, kBQ = 3, kHNSW = 4, kHNSWQuant = 5 };

// Block-quantised slot formats of an HNSW graph (PION_B200_QUANT_*).
constexpr int kQPolar = 0;  // INT4
constexpr int kQNano = 1;   // INT2
constexpr int kQTurbo = 2;  // INT3 + QJL

// ---- flat_f32.cu
int ff32_tile_rows();
int ff32_query_tile();
int ff32_k_elems();
int ff32_kc(int k);
int ff32_exact_chunks();
struct Ff32TcLaunch {
    const CUtensorMap* tmap_qh = nullptr;  // queries, bf16 hi / lo halves
    const CUtensorMap* tmap_ql = nullptr;
    const CUtensorMap* tmap_rh = nullptr;  // rows, bf16 hi / lo halves
    const CUtensorMap* tmap_rl = nullptr;
    const float* thr0 = nullptr;
    int thr0_stride = 0;
    int64_t n_rows = 0;
    int nq = 0;
    int dim = 0;
    int kc = 0;
    int tile_begin = 0;
    int tile_end = 0;
    int n_splits = 1;
    int n_lists = 1;
    int list_base = 0;
    int bound_mode = 0;  // 1: threshold pass (one approximate dot per 32-row chunk)
    float* cand_val = nullptr;
    int32_t* cand_idx = nullptr;
    int* status = nullptr;
};
int launch_flat_bf16x3_tc(const Ff32TcLaunch& launch, cudaStream_t st);
int launch_split_bf16(const float* x, size_t n, void* hi, void* lo, cudaStream_t st);
// exact_knn's query normalisation; with `codes` also the BQ sign code (and +-1 bytes
// into `pm` when given) of the normalised query.
int launch_query_normalize(const float* q, int nq, int dim, float* out, float* qnorm,
                           cudaStream_t st, int8_t* pm = nullptr, uint64_t* codes = nullptr);
int launch_l2_normalize_rows(const float* src, int64_t n_rows, int dim, float* dst, float* norms,
                             cudaStream_t st);
int launch_row_norms(const float* rows, int64_t n_rows, int dim, float* norms, cudaStream_t st);
int launch_max_reduce(const float* x, int64_t n, float* out, cudaStream_t st);
int launch_rescore_certify(const float* rows, int dim, const float* qn, const float* qnorm,
                           float row_norm_max, const float* cand_v, const int32_t* cand_i, int nq,
                           int kc, int k, int64_t id_base, float* out_d, int32_t* out_i,
                           int* flagged, int* n_flagged, int force_exact, cudaStream_t st);
// exact_knn for one query as an HBM stream: per CTA the k best (distance asc, row asc)
// of its contiguous row range, [ctas][k] into cand_d / cand_i (rows local, +inf / -1
// padding); merge them with launch_merge_lists (ascending).
bool ff32_scan1_supported(int dim, int k);
int ff32_scan1_ctas(int64_t n_rows, int num_sms);
int launch_flat_f32_scan1(const float* rows, int64_t n_rows, int dim, const float* qn, int k,
                          int ctas, float* cand_d, int32_t* cand_i, cudaStream_t st);
int launch_exact_fallback(const float* rows, int64_t n_rows, int dim, const float* qn,
                          const int* flagged, const int* n_flagged, int nq, int k,
                          int64_t id_base, float* chunk_d, int32_t* chunk_i, float* out_d,
                          int32_t* out_i, int num_sms, cudaStream_t st);

}  // namespace pion

struct pion_b200_ctx {
    int device = 0;
    int worker_id = 0;
    int num_sms = 148;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    int* d_status = nullptr;       // device status words written by bounded waits:
                                   // [0] host-memory calls, [1] device-memory calls
    int* h_status = nullptr;       // pinned mirror of both words
    pion::DevBuf scratch;          // per-call candidate lists
    pion::DevBuf scratch2;         // second-level scratch (merges, shortlists)
    pion::DevBuf stage_in;         // device copies of host inputs
    pion::DevBuf stage_out;        // device outputs copied back to host
    pion::DevBuf hnsw_visited;     // HNSW visited bitmaps, one per resident warp
    pion::DevBuf hnsw_touched;     // per resident warp: the bitmap words a query touched
    bool vis_clean = false;        // hnsw_visited is all zero (the beam kernel keeps it so)
    pion::DevBuf hnsw_misc;        // HNSW work counters and query counter
    std::string last_error;
    int64_t launches = 0;
    cudaEvent_t switch_ev = nullptr;  // orders scratch use across set_stream switches
    int64_t slot_exact = 0;           // queries of the last slot scan that took the exact path
    uint64_t wait_ns = pion::kDefaultWaitNs;  // budget of the FLAT INT8 kernels' waits
    // scoring-kernel timing (pion_v_b200_timing_*)
    bool timing = false;
    std::vector<cudaEvent_t> ev_start, ev_end;
    std::vector<int> ev_tag;       // PION_B200_TIMING_* of each event pair
    std::vector<bool> ev_closed;   // its end event was recorded
    size_t ev_used = 0;
    int ev_open = -1;              // the pair opened last
};

struct pion_b200_index {
    int kind = 0;
    int device = 0;
    int64_t n_rows = 0;
    int64_t dim = 0;
    int64_t id_base = 0;
    bool owns = true;
    // FLAT INT8
    int8_t* rows_i8 = nullptr;
    float* row_scale = nullptr;
    float* tile_rs_max = nullptr;
    // FLAT FP32 and BQ rerank rows
    float* rows_f32 = nullptr;
    float row_norm_max = 0.0f;  // largest row L2 norm (bounds the shortlist error)
    void* rows_hi = nullptr;    // bf16 split of rows_f32: hi = bf16(x), lo = bf16(x - hi)
    void* rows_lo = nullptr;
    CUtensorMap tmap_rows_lo;
    // BQ sign codes, uint64 words per row
    uint64_t* codes = nullptr;
    int64_t words = 0;
    CUtensorMap tmap_rows;
    bool has_tmap = false;
    // HNSW: the compact level-0 layout and the upper levels, on the device
    struct {
        int8_t* codes = nullptr;  // [slot][1536], 16-byte aligned
        float* norms = nullptr;   // [slot]: the slot header's |code|^2
        uint32_t* l0_compact = nullptr;
        uint32_t* l0_slots = nullptr;
        uint32_t* node_slot = nullptr;
        int32_t* node_ids = nullptr;
        uint8_t* deleted = nullptr;
        int8_t* node_level = nullptr;
        int64_t* upper_offset = nullptr;
        uint32_t* upper_links = nullptr;
        uint32_t* upper_slots = nullptr;
        int32_t* ext_to_node = nullptr;  // external id - ext_base -> node (-1: none)
        int32_t* slot_ext = nullptr;     // slot -> external id (-1: no node)
        float* rerank = nullptr;         // FP32 rows by slot for the brute-force rerank
        int* chunk_vmin = nullptr;       // per 32 slots: min floor(norm) (whole tiles)
        // block-quantised graphs (kHNSWQuant): per slot |v|^2 in `norms`, 48 f16 scales
        // and the packed block codes; QJL signs and residual norms by node; FP32 rerank
        // rows by node
        int quant_kind = -1;
        int code_bytes = 0;
        uint8_t* qcodes = nullptr;
        uint16_t* qscales = nullptr;
        uint64_t* qjl = nullptr;
        float* qjl_res = nullptr;
        uint64_t* qjl_rs = nullptr;
        float qjl_lambda = 1.0f;
        float* rerank_node = nullptr;
        int64_t ext_base = 0, ext_count = 0;
        int M = 0;
        int max_level = 0;
        int64_t entry = -1;
        int metric = 0;
        float gmin = 0.0f, gmax = 0.0f;
    } hnsw;
};

namespace pion {

// ---- hnsw.cu
struct HnswLaunch {
    const int8_t* codes = nullptr;  // [slot][1536]
    const float* norms = nullptr;   // [slot]
    const uint32_t* l0_compact = nullptr;
    const uint32_t* l0_slots = nullptr;
    const uint32_t* node_slot = nullptr;
    const int32_t* node_ids = nullptr;
    const uint8_t* deleted = nullptr;
    const int8_t* node_level = nullptr;
    const int64_t* upper_offset = nullptr;
    const uint32_t* upper_links = nullptr;
    const uint32_t* upper_slots = nullptr;
    int M = 0;
    int max_level = 0;
    int64_t num_nodes = 0;
    int64_t entry = 0;
    const int8_t* qcodes = nullptr;
    const int32_t* qblk = nullptr;
    int nq = 0, k = 0, ef = 0;
    uint32_t* visited = nullptr;  // all zero on entry, left all zero (launch_hnsw_beam)
    int64_t vis_words = 0;
    uint32_t* touched = nullptr;  // touch_cap words per resident warp
    int touch_cap = 0;
    int32_t* out_ids = nullptr;
    float* out_dist = nullptr;
    unsigned long long* stats = nullptr;
    unsigned* next_query = nullptr;
    int* status = nullptr;
    int ctas = 0;
    // from-pool mode (pion_v_beam_1536, hnsw_beam_batch): per query a pool of
    // (f32 dist, u32 id) entries, pool_stride entries apart, its size, cursor and norm
    void* pool_io = nullptr;
    int64_t pool_stride = 0;
    const int* pool_size = nullptr;
    const int* pool_cursor = nullptr;
    const float* qn_given = nullptr;
    int* pool_size_out = nullptr;
};
int hnsw_dim();
int hnsw_warps_per_cta();
size_t hnsw_warp_smem(int ef);
int hnsw_ctas_per_sm(int ef);
int launch_hnsw_quantize(const float* q, int nq, float gmin, float scale, int8_t* codes,
                         int32_t* blk, cudaStream_t st);
int launch_hnsw_beam(const HnswLaunch& launch, cudaStream_t st);
// Visited bitmaps (all zero) and touched-word lists for `warps` resident warps of the beam
// kernel in the context's scratch, into L.visited / L.vis_words / L.touched / L.touch_cap.
int hnsw_visit_buffers(pion_b200_ctx* ctx, int64_t warps, int64_t num_nodes, HnswLaunch& L);
int launch_hnsw_relayout(const int8_t* src, int64_t n, int64_t stride, int64_t hdr,
                         int8_t* codes, float* norms, cudaStream_t st);
// rows: the FP32 copy by node (the metric then reads it, unclamped), or null (the codes)
int launch_hnsw_metric(const float* qn, int nq, int k, const int32_t* ids,
                       const int32_t* ext_to_node, int64_t ext_base, int64_t ext_count,
                       const uint32_t* node_slot, const int8_t* codes, float gmin, float gmax,
                       int cosine, const float* rows, float* scores, cudaStream_t st);

// ---- quant.cu
struct QuantLaunch {
    int kind = 0, metric = 0;
    const uint8_t* codes = nullptr;
    int code_bytes = 0;
    const uint16_t* scales = nullptr;
    const float* norms = nullptr;
    const uint64_t* qjl = nullptr;
    const float* res_norms = nullptr;
    const uint64_t* rsigns = nullptr;
    float lambda = 1.0f;
    const float* rerank = nullptr;
    const uint32_t* l0_compact = nullptr;
    const uint32_t* l0_slots = nullptr;
    const uint32_t* node_slot = nullptr;
    const int32_t* node_ids = nullptr;
    const uint8_t* deleted = nullptr;
    const int8_t* node_level = nullptr;
    const int64_t* upper_offset = nullptr;
    const uint32_t* upper_links = nullptr;
    const uint32_t* upper_slots = nullptr;
    int M = 0, max_level = 0;
    int64_t num_nodes = 0, entry = 0;
    const float* queries = nullptr;
    int nq = 0, k = 0, ef = 0;
    const int* qlist = nullptr;    // queries to run (null: all)
    const int* qlist_n = nullptr;  // their count, in device memory
    uint32_t* visited = nullptr;
    int64_t vis_words = 0;
    void* cand_tail = nullptr;  // per warp (cand_cap - top entries) x 8 bytes
    int64_t cand_cap = 0;
    int32_t* out_ids = nullptr;
    float* out_scores = nullptr;
    int32_t* out_found = nullptr;
    int* overflow = nullptr;  // null: an outgrown heap is an error
    int* overflow_n = nullptr;
    unsigned* next_query = nullptr;
    unsigned long long* stats = nullptr;
    int* status = nullptr;
    int ctas = 0;
    // from-heaps mode (pion_v_quant_beam_1536): one query given as codes, scales,
    // {|q|^2, |residual|^2} and QJL signs; the caller's heaps in and out
    int from_heaps = 0;
    const int8_t* given_codes = nullptr;
    const float* given_scales = nullptr;
    const float* given_norms = nullptr;
    const uint64_t* given_signs = nullptr;
    void* cand_io = nullptr;  // cand_io_cap entries of 8 bytes (f32 dist, u32 node)
    int64_t cand_io_cap = 0;
    void* res_io = nullptr;   // ef entries
    int* heap_meta = nullptr; // 6 ints
};
size_t quant_warp_smem(int ef);
int quant_warps_per_cta();
int quant_top_entries();
int quant_ctas_per_sm(int ef);
int launch_quant_search(const QuantLaunch& launch, cudaStream_t st);
// abi_quant.cu: drops the graphs pion_v_quant_beam_1536 registered (all when null)
void quant_beam_forget(const uint32_t* l0_compact);

// ---- compat.cu: the per-thread default context of the reference-compatible symbols
pion_b200_ctx* compat_default_ctx(const char* who);

// ---- shared ABI helpers (abi.cu)
int set_error(pion_b200_ctx* ctx, int code, const char* fmt, ...);
int queue_status_readback(pion_b200_ctx* ctx);
// The status word a call's kernels record into: word 0 for host-memory calls (checked
// by the call itself), word 1 for device-memory calls (reported by pion_v_b200_sync).
int* call_status(pion_b200_ctx* ctx, int mem);
int finish_sync(pion_b200_ctx* ctx);
bool valid_ctx(const pion_b200_ctx* ctx);
int use_device(pion_b200_ctx* ctx);
size_t align_up(size_t x, size_t a);
int prepass_tiles(int k);
int bound_tiles(int n_tiles, int k);
bool use_prepass(int n_tiles, int k, const char* env);
int ensure(DevBuf& b, size_t bytes);
// Raises `kernel`'s dynamic shared-memory limit to `bytes` on the CURRENT device
// (cudaFuncSetAttribute is per device), remembered per (kernel, device) under a lock,
// so a process that uses several GPUs from several host threads configures each one.
int set_smem_limit(const void* kernel, int bytes);
// Content fingerprint of a host table: `h` mixed with the first `take_bytes` bytes of
// 64 evenly spaced rows and the last one.  Guards caches keyed by host pointers
// against a different table allocated at the same address.
uint64_t sample_rows_hash(uint64_t h, const void* base, int64_t n_rows, int64_t row_bytes,
                          int64_t take_bytes);
int make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                 uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                 uint32_t box_outer, CUtensorMapSwizzle swizzle);

// ---- flat_i8.cu
int fi8_tile_rows();
int fi8_query_tile();
int fi8_k_block();
int fi8_kcap(int k);
int fi8_choose_splits(int n_qt, int n_tiles, int num_sms);
int fi8_scan1_ctas(int64_t n_rows, int num_sms);
int launch_tile_max(const float* rs, int64_t n_rows, float* out, cudaStream_t st);
int launch_quantize_rows_i8(const float* src, int64_t n_rows, int d, int d_pad, int8_t* dst,
                            float* dst_scale, cudaStream_t st);
// n result slots of (value, id -1); es = 2 for interleaved (score, id) pairs (v = the
// pairs, i = v + 1 as ints)
int launch_fill_results(float* v, int32_t* i, size_t n, float value, cudaStream_t st,
                        int es = 1);
int launch_merge_lists(const float* cv, const int32_t* ci, int nq, int n_lists, int k,
                       int64_t id_offset, bool descending, float* out_v, int32_t* out_i,
                       cudaStream_t st, bool lists_major = false, int out_stride = 0,
                       bool pairs = false, int out_es = 1, int lm_nq = 0);
// ---- exchange.cu: publish this rank's pairs to every rank, wait for theirs, merge
int exchange_merge(pion_b200_ctx* ctx, pion_b200_exchange* e, int region, const void* pairs,
                   int64_t nq, int64_t k, uint32_t epoch, bool descending, float* out_v,
                   int32_t* out_i, int out_es);
// The largest n_lists exchange_lists_merge takes.
int exchange_max_lists();
// The same from this shard's candidate lists [nq][n_lists][k]: merged, offset by
// id_offset and published by one kernel, then waited for and merged by another.
int exchange_lists_merge(pion_b200_ctx* ctx, pion_b200_exchange* e, int region,
                         const float* cv, const int32_t* ci, int n_lists, int64_t id_offset,
                         int64_t nq, int64_t k, uint32_t epoch, bool descending, float* out_v,
                         int32_t* out_i, int out_es);
// Event pair around one scoring-kernel launch (or one phase of it, `tag` =
// PION_B200_TIMING_*) when timing is enabled.  timing_begin returns the pair's slot
// (-1 when timing is off); timing_end closes `slot`, or the pair opened last.
int timing_begin(pion_b200_ctx* ctx, int tag = PION_B200_TIMING_SCORING);
void timing_end(pion_b200_ctx* ctx, int slot = -1);
// One launch of the tensor-core FLAT INT8 kernel over index tiles [tile_begin,
// tile_end) (tiles of fi8_tile_rows() rows).  Each (query, split) writes
// fi8_lists_per_split(k) sorted lists of k (score, id) pairs at list
// list_base + split * lists_per_split + slice of the [nq][n_lists][k] layout.
// `thr0` (optional) points at a per-query lower bound of the final k-th score,
// `thr0_stride` elements apart.
struct Fi8TcLaunch {
    const CUtensorMap* tmap_q = nullptr;
    const CUtensorMap* tmap_rows = nullptr;
    const float* row_scale = nullptr;
    const float* tile_rs_max = nullptr;
    const float* q_scale = nullptr;
    const float* thr0 = nullptr;
    int thr0_stride = 0;
    int64_t n_rows = 0;
    int nq = 0;
    int dim = 0;
    int k = 0;
    int tile_begin = 0;
    int tile_end = 0;
    int n_splits = 1;
    int n_lists = 1;
    int list_base = 0;
    int bound_mode = 0;  // 1: threshold pass (one exact score per 32-row chunk)
    float* cand_val = nullptr;
    int32_t* cand_idx = nullptr;
    int* status = nullptr;
    uint64_t wait_ns = kDefaultWaitNs;  // budget of every mbarrier wait in the kernel
    int test_stall = 0;  // 1: one CTA waits on a barrier nothing arrives on (tests)
};
int fi8_lists_per_split(int k);
int launch_flat_i8_tc(const Fi8TcLaunch& launch, cudaStream_t st);
int launch_flat_i8_scan1(const int8_t* rows, const float* row_scale, int64_t n_rows, int dim,
                         const int8_t* q, const float* q_scale, int k, int ctas, float* cand_val,
                         int32_t* cand_idx, cudaStream_t st);

// ---- delta.cu, and the exact scan of flat_f32.cu for every query
int delta_kg_max();
int launch_delta_rescore(const float* rows, int dim, int64_t built, int l2, const float* q, int nq,
                         int kg, int32_t* ids, float* scores, int* n_graph, cudaStream_t st);
int launch_delta_merge(const int32_t* gi, const float* gs, const int* n_graph, int kg,
                       const int32_t* di, const float* ds, int kd, int nq, int k, int32_t* out_i,
                       float* out_s, cudaStream_t st);
int launch_exact_scan_all(const float* rows, int64_t n_rows, int dim, const float* q, int nq,
                          int k, int64_t id_base, int l2, int* queue, float* chunk_d,
                          int32_t* chunk_i, float* out_d, int32_t* out_i, int num_sms,
                          cudaStream_t st);

// ---- slot_scan.cu
int slot_tile_rows();
int slot_query_tile();
int slot_k_block();
int slot_kmax();
struct SlotTcLaunch {
    const CUtensorMap* tmap_q = nullptr;     // query codes [nq x 1536]
    const CUtensorMap* tmap_rows = nullptr;  // slot codes [n x 1536]
    int k = 1;                               // loop entries
    const float* bound = nullptr;            // per query: collect d < bound
    const float* qnorm = nullptr;
    const float* vnorm = nullptr;
    int64_t n_rows = 0;
    int nq = 0;
    int tile_begin = 0;
    int tile_end = 0;
    int n_splits = 1;
    int cap = 0;
    float* cand_d = nullptr;
    int32_t* cand_i = nullptr;
    int* cand_n = nullptr;
    int* status = nullptr;
    float* dense = nullptr;        // dense mode (exact path): [query][slot - dense_base]
    int64_t dense_base = 0;
    int64_t dense_ld = 0;
    const int* n_dense = nullptr;  // queries in the dense rows (null: nq)
    float* pub = nullptr;          // [nq][n_splits][2] published list thresholds, or null
    const int* chunk_vmin = nullptr;  // per 32-slot chunk min floor(norm), whole tiles
};
int launch_slot_chunk_vmin(const float* vnorm, int64_t n, int* out, cudaStream_t st);
int launch_slot_prep(const int8_t* codes, const float* qnorm_in, int nq, int k, float* qnorm,
                     float* st_d, int32_t* st_i, float* st_worst, int* st_widx, int* qflag,
                     int* flags, int force_exact, cudaStream_t st);
int launch_slot_tc(const SlotTcLaunch& launch, cudaStream_t st);
int launch_slot_replay(const float* cand_d, const int32_t* cand_i, const int* cand_n, int n_lists,
                       int cap, int nq, int k, float* st_d, int32_t* st_i, float* st_worst,
                       int* st_widx, int* qflag, int* flags, unsigned long long* counters,
                       cudaStream_t st);
int launch_slot_gather(const int8_t* qcodes, const float* qnorm, const int* flags, int first,
                       int count, int k, int8_t* fcodes, float* fqn, int* n_dense, float* fd,
                       int32_t* fi, float* fworst, int* fwidx, cudaStream_t st);
int launch_slot_dense_replay(const float* dense, int64_t ld, int64_t base, int64_t len,
                             const int* n_dense, int count, int k, float* fd, int32_t* fi,
                             float* fworst, int* fwidx, int last, const int* flags, int first,
                             float* st_d, int32_t* st_i, float* st_worst, int* st_widx,
                             const int* qflag, cudaStream_t st);
int launch_slot_emit(const float* st_d, const int32_t* st_i, int nq, int k, int k_out,
                     int32_t* out_slots, float* out_d, cudaStream_t st);
int launch_slot_finish(const float* st_d, const int32_t* st_i, int nq, int k, const float* q_raw,
                       const float* rerank, const int32_t* slot_ext, int64_t n, int final_k,
                       int k_out, int32_t* out_ids, float* out_scores, int32_t* out_found,
                       cudaStream_t st);

// ---- bq.cu
int bq_tile_rows();
int bq_query_tile();
int bq_k_block();
int bq_cap();
int bq_lists_per_split();
struct BqTcLaunch {
    const CUtensorMap* tmap_q = nullptr;     // queries as ±1 int8
    const CUtensorMap* tmap_rows = nullptr;  // rows as ±1 int8
    const int* dot_min = nullptr;            // per query, or nullptr (collect everything)
    int64_t n_rows = 0;
    int nq = 0;
    int dim = 0;
    int tile_begin = 0;
    int tile_end = 0;
    int n_splits = 1;
    int n_lists = 1;
    int list_base = 0;
    int32_t* cand_id = nullptr;
    uint16_t* cand_h = nullptr;
    int* cand_n = nullptr;
    int* status = nullptr;
};
int launch_signs(const float* x, int64_t n_rows, int dim, int8_t* pm, uint64_t* codes,
                 cudaStream_t st);
int launch_bq_tc(const BqTcLaunch& launch, cudaStream_t st);
int launch_bq_select(const int32_t* cid, const uint16_t* ch, const int* cn, int nq, int n_lists,
                     int dim, int S, int32_t* out_id, uint16_t* out_h, int* out_n,
                     int out_qstride, int n_qstride, int* next_dot_min, int* flagged,
                     int* n_flagged, int force_flag, cudaStream_t st);
int launch_bq_fallback(const uint64_t* codes, int64_t n_rows, int words, const uint64_t* qcodes,
                       const int* flagged, const int* n_flagged, int S, int32_t* out_id,
                       uint16_t* out_h, int* out_n, int num_sms, cudaStream_t st);
// One query's Hamming shortlist as an HBM popcount stream over the packed codes: the S
// smallest distances by (distance, row), sorted, into sl_id / sl_h / sl_n (three
// kernels; `scratch` holds bq_scan1_scratch bytes).
bool bq_scan1_supported(int words, int S);
int bq_scan1_ctas(int64_t n_rows, int words, int num_sms, int stream_path = 0);
size_t bq_scan1_scratch(int64_t n_rows, int words);
// The first pass streams the codes through shared memory by bulk copies (rows of at most
// 384 bytes, unless stream_path == 1) or through registers; `status` / `wait_ns` bound its
// waits.  bq_scan1_ctas sizes the grid to one full wave of the pass that runs.
int launch_bq_scan1(const uint64_t* codes, int64_t n_rows, int words, const uint64_t* qcode,
                    int S, int ctas, void* scratch, int32_t* sl_id, uint16_t* sl_h, int* sl_n,
                    int* status, uint64_t wait_ns, int stream_path, cudaStream_t st);
// The same rerank for few queries: shortlist rows spread over CTAs (dim % 16 == 0,
// S <= 256), `dist` holds nq * S floats of scratch.
int launch_bq_rerank_wide(const float* rows, int dim, const float* qn, const int32_t* sl_id,
                          const int* sl_n, int S, int nq, int k, int64_t id_base, float* dist,
                          float* out_d, int32_t* out_i, cudaStream_t st);
// The same with the shortlist rows bulk-copied into shared memory (8 per one-warp CTA)
// and the pick done by each query's last CTA; `done` holds nq counters of scratch.
int launch_bq_rerank_staged(const float* rows, int dim, const float* qn, const int32_t* sl_id,
                            const int* sl_n, int S, int nq, int k, int64_t id_base, float* dist,
                            unsigned* done, int* status, uint64_t wait_ns, float* out_d,
                            int32_t* out_i, cudaStream_t st);
int launch_bq_rerank(const float* rows, int dim, const float* qn, const int32_t* sl_id,
                     const int* sl_n, int S, int nq, int k, int64_t id_base, float* out_d,
                     int32_t* out_i, cudaStream_t st);

}  // namespace pion
