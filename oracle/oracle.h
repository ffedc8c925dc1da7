/* CPU oracle for histogram tree training (tree_method="hist").
 *
 * TEST INFRASTRUCTURE ONLY. This single-threaded C restatement of the
 * reference's training semantics is the checker for the CUDA product: only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.
 * The product never links, calls or falls back to it.
 *
 * Layouts used throughout:
 *   X          row-major float32 [rows][cols], NaN = missing
 *   cuts       [cols][stride] float32, counts[cols], minima[cols]
 *   bins       row-major uint32 [rows][cols], ORC_MISSING = missing
 *   pairs      float32 (g, h) per (row, group): [rows][groups][2]
 *   q          int64 (g, h) per row of one group: [rows][2]
 *   hist       int64 (g, h) pairs [nodes][cols][stride + 1]; index stride
 *              is the missing bin
 */
#ifndef XGB_ORACLE_H
#define XGB_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_MISSING 0xffffffffu

/* Same field order and size (96 bytes) as the reference's Split record
 * (include/metalgb/shared.h:124-134), so both can be compared bytewise. */
typedef struct {
  float gain, threshold, applied_parent_weight, left_h, applied_parent_hessian, right_h;
  int32_t feature;
  uint32_t default_left;
  float left_weight, right_weight, total_g, total_h;
  uint32_t split_type, category_begin, category_count;
  float parent_weight;
  int64_t left_sum_g, left_sum_h, right_sum_g, right_sum_h;
} orc_split;

/* A tree node: reference Node fields (include/metalgb/shared.h:25-29) used by
 * numeric trees, plus split_bin: a present row goes left iff bin <= split_bin
 * (as a signed value; -1 sends every present row right). */
typedef struct {
  int32_t left, right, feature, parent;
  float threshold, leaf, cover, gain;
  uint32_t default_left;
  int32_t split_bin;
} orc_node;

typedef struct {
  uint32_t max_depth;
  float eta, reg_lambda, reg_alpha, min_child_weight, max_delta_step, min_split_loss;
} orc_tree_params;

enum { ORC_SQUAREDERROR = 0, ORC_LOGISTIC = 1, ORC_SOFTPROB = 3 };

uint32_t orc_cut_stride(uint32_t rows, uint32_t max_bin);
uint32_t orc_sketch_cuts(const float* X, uint32_t rows, uint32_t cols, const float* weights,
                         uint32_t max_bin, float* cuts, uint32_t* counts, float* minima);
void orc_quantize(const float* X, uint32_t rows, uint32_t cols, const float* cuts,
                  uint32_t stride, const uint32_t* counts, uint32_t* bins);

float orc_expf(float x);
void orc_gradients(int objective, const float* margins, const float* labels,
                   const float* weights, uint32_t rows, uint32_t groups, float scale_pos_weight,
                   float* pairs);
void orc_gradient_scales(const float* pairs, uint32_t rows, uint32_t groups, float* scales);
void orc_quantize_gradients(const float* pairs, uint32_t rows, uint32_t groups,
                            const float* scales, int64_t* q);

void orc_histogram(const uint32_t* bins, uint32_t cols, uint32_t stride, const int64_t* q,
                   const uint32_t* rows, uint32_t nrows, int64_t* hist);
void orc_evaluate_splits(const int64_t* hist, uint32_t nodes, uint32_t cols, uint32_t stride,
                         const float* scale, const float* cuts, const uint32_t* counts,
                         const float* minima, float reg_lambda, float reg_alpha,
                         float min_child_weight, float max_delta_step, uint32_t use_parent_sums,
                         const int64_t* node_sums, orc_split* out);
void orc_select_splits(const orc_split* candidates, uint32_t nodes, uint32_t cols,
                       const float* scale, float reg_lambda, float reg_alpha,
                       float max_delta_step, orc_split* best);

int orc_grow_tree(const uint32_t* bins, uint32_t rows, uint32_t cols, const int64_t* q,
                  const float* scale, const float* cuts, uint32_t stride,
                  const uint32_t* counts, const float* minima, const orc_tree_params* tp,
                  orc_node* nodes, uint32_t capacity, float* row_leaf);

/* The host-driven grower (the reference's fallback driver for loss-guided
 * trees, max_leaves and depth > 10): depth-wise batches of at most 256
 * leaves in node-id order, or one leaf at a time by largest gain when
 * `lossguide`; max_leaves 0 and max_depth 0 mean unlimited. Returns the node
 * count or a negative value on error. */
int orc_grow_tree_queue(const uint32_t* bins, uint32_t rows, uint32_t cols, const int64_t* q,
                        const float* scale, const float* cuts, uint32_t stride, const uint32_t* counts,
                        const float* minima, const orc_tree_params* tp, uint32_t lossguide,
                        uint32_t max_leaves, orc_node* nodes, uint32_t capacity, float* row_leaf);

void orc_base_score(int objective, const float* labels, const float* weights, uint32_t rows,
                    uint32_t groups, float scale_pos_weight, float* score, float* margin);

/* Whole training run: cuts, bins, base score, then `rounds` boosting rounds
 * of `groups` trees each. Trees are written back to back into `nodes`
 * (at most node_capacity records) with tree_sizes[round * groups + group];
 * margins receives the final training margins [rows][groups]. Returns the
 * total node count or a negative value on error. */
typedef struct {
  int objective;
  uint32_t num_class, max_bin, rounds;
  float scale_pos_weight;
  int has_base_score;
  float base_score;
  orc_tree_params tree;
  /* grow_policy="lossguide" and max_leaves (0 = no limit); either, or a
   * max_depth of 0 or above 10, selects the host-driven grower. */
  uint32_t lossguide, max_leaves;
} orc_train_params;

int64_t orc_train(const float* X, uint32_t rows, uint32_t cols, const float* labels,
                  const float* weights, const orc_train_params* p, orc_node* nodes,
                  uint64_t node_capacity, uint32_t* tree_sizes, float* margins,
                  float* base_margin_out);

#ifdef __cplusplus
}
#endif
#endif
