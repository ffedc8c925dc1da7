// Device workspaces and launch entry points of the histogram tree trainer.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "common.h"

namespace xgbb {

// Quantised feature matrix in HBM: row-major ELLPACK, one code per
// (row, feature), uint8 or uint16. `missing` is the code of a missing value:
// the cut stride B (the histogram's missing bin) when it fits, else 255 for
// uint8 codes with B = 256, or 0x100 when all 256 uint8 codes are bins and no
// value is missing. Each row is padded to `stride` codes (a multiple of 16
// bytes).
struct Ellpack {
  const void* codes = nullptr;
  const void* codes_fm = nullptr;           // optional feature-major copy [cols][rows]
  uint32_t rows = 0, cols = 0, stride = 0;  // stride in codes
  uint32_t bytes_per_code = 1;              // 1 or 2
  uint32_t missing = 0xff;
  uint32_t bins = 0;                        // cut stride B (histogram has B + 1 bins)
  const float* cuts = nullptr;              // [cols][bins]
  const uint32_t* counts = nullptr;         // [cols]
  const float* minima = nullptr;            // [cols]
};

// Exact magnitude accumulators for the gradient scales, one entry per
// (group, part) with part 0 = g, 1 = h; separate arrays so that each can be
// reduced over ranks with one NCCL call.
struct MassAccum {
  unsigned int* max_bits;         // [2G] max |value| bits (max over ranks)
  unsigned int* fallback;         // [2G] 1 when the windowed sum cannot decide
  unsigned long long* window;     // [2G][2] 128-bit windowed sum (lo, hi)
  unsigned long long* limbs;      // [2G][4] the windowed sum as 32-bit limbs (sum over ranks)
  unsigned long long* exact;      // [2G][10] 32-bit limb sums of the exact magnitude
};
// Bytes of the accumulators for `groups` output groups (one allocation).
inline size_t mass_bytes(uint32_t groups) { return size_t(groups) * 2 * (4 + 4 + 16 + 32 + 80); }
MassAccum mass_view(void* base, uint32_t groups);
// Cross-rank transport of the windowed sums: window -> limbs and back.
void launch_window_to_limbs(MassAccum m, uint32_t groups, cudaStream_t stream);
void launch_limbs_to_window(MassAccum m, uint32_t groups, cudaStream_t stream);

// Everything one tree needs on the device; pointers are fixed for a booster,
// so the launch sequence can be captured once as a CUDA graph and replayed.
struct TreeWorkspace {
  DriverState* state;
  uint32_t* ids[2];
  long long* sums[2];        // [slot][2]
  uint32_t* seg_begin[2];
  uint32_t* seg_count[2];
  uint32_t* parent_slot;     // next-level pair -> parent slot
  uint32_t* built_left;      // pair -> 1 when the left child is built
  uint32_t* tile_offset;     // [pairs + 1] tiles of built children (exclusive scan)
  uint32_t* ptile_offset;    // [frontier + 1] tiles of all frontier nodes
  uint32_t* cursor_l;        // partition cursors per slot
  uint32_t* cursor_r;
  uint32_t* counts_local;    // [slot][2] left/right child counts of this rank
  uint32_t* counts_global;   // [slot][2] summed over ranks (== local on one GPU)
  uint32_t* mode;            // per slot: 0 retire, 1 split, 2 terminal split
  float* slot_leaf;          // [slot][2]
  unsigned long long* keys[2];  // best (gain, feature) key per slot
  DevSplit* cand;            // [kMaxFrontier][cols]
  DevNode* nodes;            // [node_capacity]
  longlong2* built;          // [pairs][cols][bins + 1]
  longlong2* bank[2];        // [slots][cols][bins + 1]
  uint32_t* rows[2];         // row ids per level (level 0 uses the identity)
  float2* ord[2];            // per row of rows[] (level >= 1): its gradient pair
  uint32_t node_capacity;
  unsigned long long* level_rows;  // [kMaxDepth] rows in built nodes per level
  uint32_t* level_nodes;           // [kMaxDepth] built nodes per level
};

struct TreeLaunch {
  Ellpack ell;
  TreeParams params;
  const float2* pairs;       // gradient pairs of this group [rows]
  const float2* scale;       // power-of-two scales of this group
  const unsigned int* max_bits;  // largest |g|, |h| of this group (float bits)
  float* margins;            // [rows][groups]
  uint32_t groups, group;
  bool unit_hessian;
  int hist_blocks, hist_threads, eval_blocks, part_blocks;
  uint32_t feature_group;    // features per histogram CTA
  uint32_t min_limbs;        // 3 forces three-limb histogram accumulation
  bool staged3 = true;       // uint8 rounds of three-limb values take the staged three-limb kernel
  size_t hist_smem;
  uint32_t cols_pad;         // features in the built layout (a multiple of the ranks)
  uint32_t f_lo, f_hi;       // features whose splits this rank evaluates
  // Sparse matrices: the rows' present codes (row pointers and
  // feature << 16 | code entries) and the built nodes' totals [pairs][2];
  // csr_ptr null builds histograms from the dense codes.
  const unsigned long long* csr_ptr = nullptr;
  const uint32_t* csr_entries = nullptr;
  unsigned long long* csr_totals = nullptr;
};

// Streaming multiprocessors of the current device (queried once per device).
int device_sms();
// SM cycles per warp-level shared-memory instruction of one probe variant
// (probe.cu) on the current device.
double probe_shared_pipe(int variant, uint32_t warps, uint32_t iters);

// Launch helpers (tree.cu). All are asynchronous on `stream`.
void launch_narrow_codes(const void* src, uint32_t rows, uint32_t cols, uint32_t s16, uint32_t s8,
                         uint32_t pad, void* dst, cudaStream_t stream);
void launch_transpose_codes(const void* codes, uint32_t rows, uint32_t cols, uint32_t stride,
                            uint32_t bytes_per_code, void* fm, cudaStream_t stream);
// missing_cells (or null) gains the number of NaN values among the rows.
void launch_quantize(const float* X, uint32_t rows, uint32_t cols, const float* cuts,
                     const uint32_t* counts, uint32_t bins, void* codes, uint32_t stride,
                     uint32_t bytes_per_code, uint32_t missing, unsigned long long* missing_cells,
                     cudaStream_t stream);
// flags[0] |= any NaN, flags[1] |= any infinity over n values.
void launch_validate(const float* X, uint64_t n, unsigned int* flags, cudaStream_t stream);
void launch_gradients(int objective, const float* margins, const float* labels,
                      const float* weights, uint32_t rows, uint32_t groups, float scale_pos_weight,
                      float2* pairs, MassAccum mass, cudaStream_t stream);
void launch_mass_window(const float2* pairs, uint32_t rows, uint32_t groups, MassAccum mass,
                        cudaStream_t stream);
// Reduces per-rank accumulators (already summed across ranks if sharded) to
// scales; runs the exact fallback when needed. rows_total = rows over ranks.
void launch_scales(const float2* pairs, uint32_t rows, uint32_t groups, MassAccum mass,
                   float2* scales, unsigned long long rows_total, bool may_fallback,
                   cudaStream_t stream);
void launch_mass_exact(const float2* pairs, uint32_t rows, uint32_t groups, MassAccum mass,
                       cudaStream_t stream);
void launch_scales_exact(uint32_t groups, MassAccum mass, float2* scales, cudaStream_t stream);
// Gradient pairs and scales into caller-owned device buffers with the scale
// accumulators in a fixed array of the library (no device allocation; at most
// 64 groups; calls that overlap on one device race). Defined in noalloc.cu.
void gradients_no_alloc(int objective, const float* margins, const float* labels,
                        const float* weights, uint64_t rows, uint32_t groups,
                        float scale_pos_weight, float2* pairs, float2* scales, cudaStream_t stream);
void launch_base_chunks(int objective, const float* labels, const float* weights, uint32_t rows,
                        uint32_t group, float scale_pos_weight, double* chunk_sums,
                        cudaStream_t stream);
void launch_fill_margins(float* margins, const float* base, uint32_t rows, uint32_t groups,
                         cudaStream_t stream);

struct HistConfig {
  uint32_t feature_group;
  size_t smem;
  int threads;
};
HistConfig hist_config(const Ellpack& ell, bool unit_hessian);

void tree_init(const TreeWorkspace& ws, const TreeLaunch& tl, cudaStream_t stream);
void tree_level_hist(const TreeWorkspace& ws, const TreeLaunch& tl, uint32_t depth,
                     cudaStream_t stream);
void tree_level_eval(const TreeWorkspace& ws, const TreeLaunch& tl, uint32_t depth,
                     cudaStream_t stream);
// Multi-GPU split search: this rank's best candidate per slot into `out`
// ([kMaxFrontier] records of best_record_bytes()), and the best of all ranks'
// records ([ranks][kMaxFrontier]) back into the keys and candidates.
void tree_level_pack_best(const TreeWorkspace& ws, const TreeLaunch& tl, uint32_t depth, void* out,
                          cudaStream_t stream);
void tree_level_merge_best(const TreeWorkspace& ws, const TreeLaunch& tl, uint32_t depth,
                           const void* all, uint32_t ranks, cudaStream_t stream);
size_t best_record_bytes();
void tree_level_control(const TreeWorkspace& ws, const TreeLaunch& tl, uint32_t depth,
                        cudaStream_t stream);
void tree_level_partition(const TreeWorkspace& ws, const TreeLaunch& tl, uint32_t depth,
                          cudaStream_t stream);
void tree_level_counts(const TreeWorkspace& ws, uint32_t depth, cudaStream_t stream);
void tree_level_plan(const TreeWorkspace& ws, const TreeLaunch& tl, uint32_t next_depth,
                     cudaStream_t stream);

// Bytes of one node's histogram and the largest pair / slot counts at a depth.
inline size_t hist_node_bytes(const Ellpack& e) {
  return size_t(e.cols) * (e.bins + 1) * sizeof(longlong2);
}
// Bytes of one node's histogram in the built buffer, whose feature count is
// padded to a multiple of the ranks (each rank receives whole features).
inline size_t hist_node_bytes(const Ellpack& e, uint32_t cols_pad) {
  return size_t(cols_pad) * (e.bins + 1) * sizeof(longlong2);
}
inline uint32_t max_pairs_at(uint32_t depth) { return depth ? (1u << (depth - 1)) : 1u; }
inline uint32_t max_slots_at(uint32_t depth) { return 1u << depth; }

// Host-driven trees (grower.cpp): each node's split from its own histogram.
// The best candidate of each node, as gathered for the host.
struct NodeBest {
  unsigned long long key;  // 0 when the node had no candidate
  DevSplit split;
};
// Evaluates `slots` nodes (<= kMaxFrontier) whose histograms are in `built`
// ([cols][slots][bins + 1]): the root (totals from its histogram) or children
// whose exact totals are sums[slot][2]. Writes best[kMaxFrontier].
void queue_evaluate(const Ellpack& e, const TreeParams& tp, const float2* scale, DriverState* state,
                    uint32_t slots, bool root, const longlong2* built, const long long* sums, DevSplit* cand,
                    unsigned long long* keys, NodeBest* best, int blocks, cudaStream_t stream);
// Row order of a host-driven tree: 0, 1, ..., rows - 1.
void launch_queue_iota(uint32_t* rows, uint32_t n, cudaStream_t stream);
// Histograms of `slots` nodes: node s owns order[seg[2s] .. seg[2s] + seg[2s+1]);
// tiles[s] is the exclusive scan of the nodes' tile counts (kQueueTileRows
// rows per tile), tiles[slots] the total. `built` is cleared first.
constexpr uint32_t kQueueTileRows = 2048;
void launch_queue_hist(const Ellpack& e, const uint32_t* order, const float2* pairs, const float2* scale,
                       const uint32_t* seg, const uint32_t* tiles, uint32_t slots, uint32_t total_tiles,
                       longlong2* built, int blocks, cudaStream_t stream);
// Splits the segment of each item between its children: items[i] = (begin,
// count, feature, split_bin, default_left); cursor[i] = (begin, begin +
// count) on entry, (begin + left rows, begin + left rows) on exit. `scratch`
// has as many rows as `order`.
constexpr uint32_t kQueuePartRows = 1024;
void launch_queue_partition(const Ellpack& e, uint32_t* order, uint32_t* scratch, const uint32_t* items,
                            const uint32_t* tiles, uint32_t nitems, uint32_t total_tiles, uint32_t* cursor,
                            int blocks, cudaStream_t stream);
// Sparse rows of the ELLPACK codes: row_ptr [rows + 1] (returns the entry
// count after a stream synchronisation; tile_sums holds one word per 4096
// rows), then entries [nnz] = feature << 16 | code in feature order.
uint64_t queue_csr_row_ptr(const Ellpack& e, unsigned long long* row_ptr, unsigned long long* tile_sums,
                           cudaStream_t stream);
void queue_csr_fill(const Ellpack& e, const unsigned long long* row_ptr, uint32_t* entries, cudaStream_t stream);
// Node histograms from the sparse rows: work per present value; each node's
// missing bin is its total (node_totals [slots][2]) minus its present bins.
void launch_queue_hist_csr(const Ellpack& e, const unsigned long long* row_ptr, const uint32_t* entries,
                           const uint32_t* order, const float2* pairs, const float2* scale, const uint32_t* seg,
                           const uint32_t* tiles, uint32_t slots, uint32_t total_tiles,
                           unsigned long long* node_totals, longlong2* built, int blocks, cudaStream_t stream);
// margins[row][group] += the leaf each row reaches in `nodes`, walking the
// quantised codes.
void launch_queue_margins(const Ellpack& e, const DevNode* nodes, uint32_t node_count, float* margins,
                          uint32_t groups, uint32_t group, cudaStream_t stream);

void launch_predict(const float* X, uint32_t rows, uint32_t cols, const DevNode* nodes,
                    const uint32_t* tree_begin, const uint32_t* tree_group, uint32_t trees,
                    const float* base_margin, uint32_t groups, float* out, cudaStream_t stream);
// Node id (float) of the leaf each row reaches in each tree: out[rows][trees].
void launch_leaf_index(const float* X, uint32_t rows, uint32_t cols, const DevNode* nodes,
                       const uint32_t* tree_begin, uint32_t trees, float* out, cudaStream_t stream);
void launch_transform(int objective, float* values, uint32_t rows, uint32_t groups,
                      cudaStream_t stream);

}  // namespace xgbb
