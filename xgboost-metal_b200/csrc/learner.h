// Host runtime: DMatrix (data + quantised ELLPACK in HBM) and Booster (model,
// parameters, per-matrix training state), driving the CUDA kernels.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "common.h"
#include "json.h"
#include "tree.h"

namespace xgbb {

// Owning device allocation.
class DeviceBuffer {
 public:
  DeviceBuffer() = default;
  explicit DeviceBuffer(size_t bytes) { resize(bytes); }
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  DeviceBuffer(DeviceBuffer&& o) noexcept : p_(o.p_), n_(o.n_) { o.p_ = nullptr; o.n_ = 0; }
  DeviceBuffer& operator=(DeviceBuffer&& o) noexcept {
    release();
    p_ = o.p_; n_ = o.n_; o.p_ = nullptr; o.n_ = 0;
    return *this;
  }
  ~DeviceBuffer() { release(); }
  void resize(size_t bytes) {
    if (bytes <= n_ && p_) return;
    release();
    if (bytes) XGBB_CUDA(cudaMalloc(&p_, bytes));
    n_ = bytes;
  }
  void release() {
    if (p_) cudaFree(p_);
    p_ = nullptr;
    n_ = 0;
  }
  template <class T> T* as() const { return static_cast<T*>(p_); }
  void* get() const { return p_; }
  size_t size() const { return n_; }
  explicit operator bool() const { return p_ != nullptr; }

 private:
  void* p_ = nullptr;
  size_t n_ = 0;
};

// Cut values shared by every matrix quantised with them.
struct Cuts {
  uint32_t cols = 0, stride = 0, max_bin = 0;
  std::vector<float> values, minima;
  std::vector<uint32_t> counts;
  DeviceBuffer d_values, d_counts, d_minima;
  void upload();
};

class DMatrix {
 public:
  uint32_t rows = 0, cols = 0;
  // Row-major values, NaN = missing: either `owned`, or a caller buffer that
  // the caller keeps alive and unchanged (zero-copy ingestion).
  std::vector<float> owned;
  const float* host = nullptr;
  bool validated = false;
  std::vector<float> labels, weights, base_margin;
  bool has_missing = false;
  // "feature_name" / "feature_type" lists (empty = unnamed).
  std::map<std::string, std::vector<std::string>> feature_info;
  // Quantised at construction (QuantileDMatrix): no row slices.
  bool quantile = false;

  // Quantised form.
  std::shared_ptr<Cuts> cuts;
  DeviceBuffer codes;
  DeviceBuffer codes_fm;  // feature-major copy for the partition, when memory allows
  Ellpack ell;
  uint32_t max_bin = 0;
  bool quantised() const { return bool(cuts) && (codes || rows == 0); }
  void quantise(uint32_t max_bin, const DMatrix* ref, cudaStream_t stream, int threads);
  void set_cuts(std::shared_ptr<Cuts> c, cudaStream_t stream);
  // Sparse rows of the codes (present codes only, feature << 16 | code),
  // made on first use for sparse node histograms.
  DeviceBuffer sparse_ptr, sparse_entries;
  uint64_t sparse_nnz = 0;
  uint64_t missing_cells = 0;  // NaN values among the rows, counted while binning
  bool sparse_ready = false;
  void build_sparse_rows(cudaStream_t stream);

  // Device copies on demand.
  DeviceBuffer d_data, d_labels, d_weights;
  uint64_t generation = 0, labels_generation = 0;
  const float* device_data(cudaStream_t stream);
  void upload_info(cudaStream_t stream);
  size_t uploaded_labels = 0;
  uint64_t uploaded_generation = ~0ull;
};

struct HostTree {
  std::vector<DevNode> nodes;
  uint32_t group = 0;
};

// Phases of a tree level timed with cuda_profile=2 (CUDA events around each
// launch group on the booster's stream).
enum : uint32_t {
  kPhaseHist = 0,       // histogram kernels
  kPhaseReduce,         // reduce-scatter of the built histograms over ranks
  kPhaseEval,           // subtraction, prefix scan and split gain
  kPhaseGather,         // best-split records gathered over ranks and merged
  kPhasePartition,      // control (expansion rule) and row partition
  kPhaseCounts,         // child counts, their sum over ranks, the next plan
  kPhases
};
struct Profile {
  bool csr = false;  // the level histograms came from the rows' present codes
  double phase_ms[kPhases] = {};
  double level_phase_ms[kMaxDepth][kPhases] = {};
  double hist_ms = 0, total_ms = 0;
  double hist_bytes = 0;
  uint64_t hist_launches = 0, kernel_launches = 0, rounds = 0;
  // Per tree level: histogram time, rows in built nodes, built nodes.
  double level_ms[kMaxDepth] = {}, level_rows[kMaxDepth] = {}, level_nodes[kMaxDepth] = {};
};

class Booster {
 public:
  explicit Booster(std::vector<std::shared_ptr<DMatrix>> cache);
  ~Booster();
  void set_param(const std::string& key, const std::string& value);
  std::string get_param(const std::string& key, const std::string& def) const;
  void update(const std::shared_ptr<DMatrix>& d, int iteration);
  // One round from caller-supplied gradients and Hessians, `count` values
  // each in row-major [rows][groups] order (a custom objective).
  void update_custom(const std::shared_ptr<DMatrix>& d, const float* grad, const float* hess, size_t count);
  // Returns values [rows][groups] (margins if output_margin).
  std::vector<float> predict(const std::shared_ptr<DMatrix>& d, bool output_margin,
                             uint32_t iter_begin, uint32_t iter_end, bool training,
                             std::vector<uint64_t>& shape);
  // Node id (as float) of the leaf each row reaches in each tree of rounds
  // [begin, end): [rows][trees] (strict: [rows][rounds][groups][1]).
  std::vector<float> predict_leaf(const std::shared_ptr<DMatrix>& d, uint32_t begin, uint32_t end, bool strict,
                                  std::vector<uint64_t>& shape);
  uint32_t boosted_rounds() const { return rounds_; }
  uint32_t num_feature() const { return num_feature_; }
  uint32_t groups() const { return groups_; }
  const std::vector<HostTree>& trees() { sync(); return trees_; }
  // A round returns once it is enqueued; its trees reach trees_ when the next
  // round is enqueued or when anything reads the model (this call).
  void finish_pending();
  std::string save_json();
  void load_json(const std::string& text);
  // Evaluation line of XGBoosterEvalOneIter.
  std::string evaluate(int iteration, const std::vector<std::shared_ptr<DMatrix>>& data,
                       const std::vector<std::string>& names);
  // Training configuration (upstream layout) and its inverse.
  std::string config_json();
  void load_config(const std::string& text);
  // Rounds begin, begin+step, ... < end (0 = all) as a new booster.
  std::unique_ptr<Booster> slice(int begin, int end, int step);
  // Releases the training state of every matrix; the model stays.
  void reset_training();
  std::map<std::string, std::string> attrs;
  std::map<std::string, std::vector<std::string>> feature_info;
  Profile profile;
  // Held by every C-ABI call on this booster (the reference's per-booster
  // recursive mutex, include/metalgb/engine.hpp:201, src/c_api.cpp:37-39).
  std::recursive_mutex& mutex() { return mutex_; }
  bool profiling = false;
  int profile_level = 0;  // cuda_profile: 1 histogram events, 2 every phase
  // Built histograms of one level of the first tree of the next round, for
  // checking them word for word. `depth` >= 0 requests a capture; the round
  // that takes it runs that tree without a CUDA graph. `hist` holds
  // [pairs][f_hi - f_lo][bins1][2] int64 words: the exact sums of this rank's
  // feature range over the rows of every rank (the whole histogram on one
  // GPU); node_ids[p] is the node whose histogram pair p built.
  struct LevelCapture {
    int depth = -1;
    bool ready = false;
    uint32_t pairs = 0, f_lo = 0, f_hi = 0, bins1 = 0;
    std::vector<long long> hist;
    std::vector<uint32_t> node_ids;
  } capture;
  void sync();
  // CUDA events on the booster's stream, for timing whole rounds on the device.
  void record_event(int slot);
  float elapsed_ms(int a, int b);

 private:
  struct TrainState;
  void configure();
  // Gradient pairs of a custom objective in the device layout [groups][rows],
  // and per group the largest |g| and |h| bit patterns.
  struct CustomGradients {
    std::vector<float2> pairs;
    std::vector<uint32_t> max_bits;
  };
  void initialize(DMatrix& d, bool custom = false);
  TrainState& train_state(const std::shared_ptr<DMatrix>& d, bool custom = false);
  void run_round(TrainState& ts, const CustomGradients* custom = nullptr);
  void finish_round(TrainState& ts);
  void gpu();  // makes the booster's device current; fails without a GPU
  void wait_stream(const char* what);
  void evaluate_across_ranks(const std::vector<std::string>& metrics, const std::vector<float>& pred,
                             const DMatrix& d, bool multiclass, std::vector<double>& values);
  void grow_host_driven(TrainState& ts);
  void record_tree_launches(TrainState& ts, uint32_t group, cudaStream_t stream, bool capturing,
                            uint32_t parity);
  void capture_level(TrainState& ts, uint32_t depth, const TreeLaunch& tl);
  void materialize();
  Json model_param_json() const;
  std::vector<float> score_margins(const std::vector<float>& scores) const;
  Json objective_json() const;

  std::map<std::string, std::string> params_;
  std::vector<std::weak_ptr<DMatrix>> cache_;
  bool configured_ = false, initialized_ = false;
  int objective_ = kSquaredError;
  uint32_t groups_ = 1, num_feature_ = 0, rounds_ = 0, max_bin_ = 256;
  TreeParams tp_{};
  // Trees the level-synchronous device driver does not grow (loss-guided,
  // leaf budgets, depth 0 or above 10) grow host-driven (grower.h).
  bool host_driven_ = false, lossguide_ = false, sparse_hist_ = false;
  uint32_t max_leaves_ = 0;
  float spw_ = 1.0f;
  std::vector<float> base_score_, base_margin_;
  std::vector<HostTree> trees_;
  cudaStream_t stream_ = nullptr;
  int device_ = 0;
  std::unique_ptr<TrainState> state_;
  std::vector<cudaEvent_t> user_events_;
  cudaEvent_t wait_event_ = nullptr;
  std::recursive_mutex mutex_;
};

}  // namespace xgbb
