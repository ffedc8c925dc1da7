// Booster and DMatrix runtime (host C++20). Mirrors the reference learner's
// round structure (tabulai/xgboost-metal src/learner.cpp:632-985): gradients
// for every output group, exact fixed-point scales, one depthwise tree per
// group (all trees of a round use the round's starting margins), margins
// advanced by the new trees.
#include "learner.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <sstream>

#include "comm.h"
#include "grower.h"
#include "json.h"
#include "metrics.h"
#include "sketch.h"
#include "split_select.h"

namespace xgbb {

// ---------------------------------------------------------------------------
// Cuts / DMatrix
// ---------------------------------------------------------------------------
void Cuts::upload() {
  d_values.resize(std::max<size_t>(values.size(), 1) * sizeof(float));
  d_counts.resize(std::max<size_t>(counts.size(), 1) * sizeof(uint32_t));
  d_minima.resize(std::max<size_t>(minima.size(), 1) * sizeof(float));
  if (!values.empty())
    XGBB_CUDA(cudaMemcpy(d_values.get(), values.data(), values.size() * 4, cudaMemcpyHostToDevice));
  if (!counts.empty())
    XGBB_CUDA(cudaMemcpy(d_counts.get(), counts.data(), counts.size() * 4, cudaMemcpyHostToDevice));
  if (!minima.empty())
    XGBB_CUDA(cudaMemcpy(d_minima.get(), minima.data(), minima.size() * 4, cudaMemcpyHostToDevice));
}

const float* DMatrix::device_data(cudaStream_t stream) {
  const size_t bytes = size_t(rows) * cols * sizeof(float);
  if (!d_data && bytes) {
    d_data.resize(bytes);
    XGBB_CUDA(cudaMemcpyAsync(d_data.get(), host, bytes, cudaMemcpyHostToDevice, stream));
    if (!validated) {
      // Zero-copy input is checked on the device: NaN marks missing values,
      // any infinity is an error (src/data.cpp:433).
      DeviceBuffer flags(8);
      unsigned int h[2] = {0, 0};
      XGBB_CUDA(cudaMemsetAsync(flags.get(), 0, 8, stream));
      launch_validate(d_data.as<float>(), uint64_t(rows) * cols, flags.as<unsigned int>(), stream);
      XGBB_CUDA(cudaMemcpyAsync(h, flags.get(), 8, cudaMemcpyDeviceToHost, stream));
      XGBB_CUDA(cudaStreamSynchronize(stream));
      if (h[1]) {
        d_data.release();
        throw Error("Input data contains infinity or a value too large for float32.");
      }
      has_missing = h[0] != 0;
      validated = true;
    }
  }
  return d_data.as<float>();
}

void DMatrix::upload_info(cudaStream_t stream) {
  if (uploaded_generation == generation) return;
  require(labels.size() == rows || labels.empty(), "Label length must equal the number of rows.");
  d_labels.resize(std::max<size_t>(labels.size(), 1) * 4);
  if (!labels.empty())
    XGBB_CUDA(cudaMemcpyAsync(d_labels.get(), labels.data(), labels.size() * 4,
                              cudaMemcpyHostToDevice, stream));
  if (!weights.empty()) {
    d_weights.resize(weights.size() * 4);
    XGBB_CUDA(cudaMemcpyAsync(d_weights.get(), weights.data(), weights.size() * 4,
                              cudaMemcpyHostToDevice, stream));
  } else {
    d_weights.release();
  }
  uploaded_generation = generation;
}

namespace {
// Missing code and row stride of the ELLPACK for a code width: the missing
// code is the cut stride B (the histogram's missing bin) when it fits the
// code type; with uint8 codes and B = 256 it is 255 (a missing value then
// implies at most 255 bins), and with 256 bins and no missing value it is
// 0x100, which no stored code can equal.
void code_layout(Ellpack& ell, uint32_t cols, uint32_t B, uint32_t max_count, bool narrow) {
  ell.bytes_per_code = narrow ? 1 : 2;
  if (!narrow) ell.missing = B;
  else if (B <= 255) ell.missing = B;
  else ell.missing = max_count <= 255 ? 0xffu : 0x100u;
  const uint32_t align = 16 / ell.bytes_per_code;
  ell.stride = std::max(align, (cols + align - 1) / align * align);
}
}  // namespace

void DMatrix::set_cuts(std::shared_ptr<Cuts> c, cudaStream_t stream) {
  require(c->cols == cols, "Quantile reference does not match the feature count.");
  uint32_t max_count = 0;
  for (uint32_t v : c->counts) max_count = std::max(max_count, v);
  const uint32_t B = c->stride;
  ell = Ellpack{};
  ell.rows = rows;
  ell.cols = cols;
  ell.bins = c->stride;
  ell.cuts = c->d_values.as<float>();
  ell.counts = c->d_counts.as<uint32_t>();
  ell.minima = c->d_minima.as<float>();
  // uint8 codes whenever every feature's codes, missing included, fit 256
  // symbols. Whether a value is missing is only known once the data has been
  // read, so with exactly 256 bins an unread matrix is quantised to uint16
  // and narrowed afterwards if it holds no missing value.
  const bool decided = max_count <= 255 || validated || bool(d_data);
  bool narrow = max_count <= 255 || (!has_missing && max_count <= 256);
  if (!decided) narrow = false;
  code_layout(ell, cols, B, max_count, narrow);
  codes.resize(std::max<size_t>(size_t(rows) * ell.stride * ell.bytes_per_code, 16));
  // The binning kernels count the NaN cells, which decides later whether the
  // level histograms come from the rows' present codes.
  DeviceBuffer d_missing(8);
  unsigned long long h_missing = 0;
  XGBB_CUDA(cudaMemsetAsync(d_missing.get(), 0, 8, stream));
  if (rows && d_data) {
    launch_quantize(d_data.as<float>(), rows, cols, ell.cuts, ell.counts, ell.bins, codes.get(), ell.stride,
                    ell.bytes_per_code, ell.missing, d_missing.as<unsigned long long>(), stream);
  } else if (rows) {
    // Stream the host matrix through two staging buffers: the copy of one
    // chunk overlaps the validation and quantisation of the other, and the
    // raw values never occupy the device as a whole.
    const size_t row_bytes = size_t(cols) * sizeof(float);
    const uint32_t chunk = uint32_t(std::max<size_t>(1, std::min<size_t>(rows, (256ull << 20) / row_bytes)));
    DeviceBuffer stage[2], flags(8);
    stage[0].resize(size_t(chunk) * row_bytes);
    stage[1].resize(size_t(chunk) * row_bytes);
    XGBB_CUDA(cudaMemsetAsync(flags.get(), 0, 8, stream));
    cudaStream_t cs;
    XGBB_CUDA(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
    cudaEvent_t copied[2], consumed[2];
    for (int b = 0; b < 2; ++b) {
      XGBB_CUDA(cudaEventCreateWithFlags(&copied[b], cudaEventDisableTiming));
      XGBB_CUDA(cudaEventCreateWithFlags(&consumed[b], cudaEventDisableTiming));
    }
    // The copy stream must not start before the flags are cleared and the
    // previous users of `stream` are done with the staging memory.
    XGBB_CUDA(cudaEventRecord(consumed[0], stream));
    XGBB_CUDA(cudaStreamWaitEvent(cs, consumed[0], 0));
    const size_t code_row = size_t(ell.stride) * ell.bytes_per_code;
    uint32_t i = 0;
    for (uint32_t r0 = 0; r0 < rows; r0 += chunk, ++i) {
      const uint32_t n = std::min(chunk, rows - r0);
      const int b = int(i & 1);
      if (i >= 2) XGBB_CUDA(cudaStreamWaitEvent(cs, consumed[b], 0));
      XGBB_CUDA(cudaMemcpyAsync(stage[b].get(), host + size_t(r0) * cols, size_t(n) * row_bytes,
                                cudaMemcpyHostToDevice, cs));
      XGBB_CUDA(cudaEventRecord(copied[b], cs));
      XGBB_CUDA(cudaStreamWaitEvent(stream, copied[b], 0));
      if (!validated)
        launch_validate(stage[b].as<float>(), uint64_t(n) * cols, flags.as<unsigned int>(), stream);
      launch_quantize(stage[b].as<float>(), n, cols, ell.cuts, ell.counts, ell.bins,
                      static_cast<char*>(codes.get()) + size_t(r0) * code_row, ell.stride,
                      ell.bytes_per_code, ell.missing, d_missing.as<unsigned long long>(), stream);
      XGBB_CUDA(cudaEventRecord(consumed[b], stream));
    }
    unsigned int h[2] = {0, 0};
    if (!validated) XGBB_CUDA(cudaMemcpyAsync(h, flags.get(), 8, cudaMemcpyDeviceToHost, stream));
    XGBB_CUDA(cudaStreamSynchronize(stream));
    for (int b = 0; b < 2; ++b) {
      cudaEventDestroy(copied[b]);
      cudaEventDestroy(consumed[b]);
    }
    cudaStreamDestroy(cs);
    if (!validated) {
      // Zero-copy input is checked on the device: NaN marks missing values,
      // any infinity is an error (src/data.cpp:433).
      if (h[1]) {
        codes.release();
        throw Error("Input data contains infinity or a value too large for float32.");
      }
      has_missing = h[0] != 0;
      validated = true;
    }
    if (!decided && !has_missing) {
      // 256 bins and no missing value: every code is a bin below 256.
      Ellpack n8 = ell;
      code_layout(n8, cols, B, max_count, true);
      DeviceBuffer c8(std::max<size_t>(size_t(rows) * n8.stride, 16));
      launch_narrow_codes(codes.get(), rows, cols, ell.stride, n8.stride, n8.missing, c8.get(), stream);
      XGBB_CUDA(cudaStreamSynchronize(stream));
      codes = std::move(c8);
      ell = n8;
    }
  }
  XGBB_CUDA(cudaMemcpyAsync(&h_missing, d_missing.get(), 8, cudaMemcpyDeviceToHost, stream));
  XGBB_CUDA(cudaStreamSynchronize(stream));
  missing_cells = h_missing;
  ell.codes = codes.get();
  sparse_ready = false;
  sparse_ptr.release();
  sparse_entries.release();
  // A feature-major copy lets the partition read a node's split feature from
  // a dense column; it is made when it leaves a quarter of the device free.
  codes_fm.release();
  ell.codes_fm = nullptr;
  if (rows && cols) {
    const size_t fm_bytes = size_t(rows) * cols * ell.bytes_per_code;
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) == cudaSuccess && fm_bytes + total_b / 4 <= free_b) {
      codes_fm.resize(fm_bytes);
      launch_transpose_codes(codes.get(), rows, cols, ell.stride, ell.bytes_per_code, codes_fm.get(),
                             stream);
      ell.codes_fm = codes_fm.get();
    }
  }
  cuts = std::move(c);
}

void DMatrix::build_sparse_rows(cudaStream_t stream) {
  if (sparse_ready) return;
  sparse_ptr.resize((size_t(rows) + 1) * 8);
  DeviceBuffer tile_sums((size_t(rows) / 4096 + 1) * 8);
  const uint64_t nnz =
      queue_csr_row_ptr(ell, sparse_ptr.as<unsigned long long>(), tile_sums.as<unsigned long long>(), stream);
  sparse_nnz = nnz;
  sparse_entries.resize(std::max<size_t>(nnz, 1) * 4);
  queue_csr_fill(ell, sparse_ptr.as<unsigned long long>(), sparse_entries.as<uint32_t>(), stream);
  XGBB_CUDA(cudaStreamSynchronize(stream));
  sparse_ready = true;
}

namespace {
// Cuts of the rows of every rank of a row-sharded job, identical on every
// rank and bit for bit the cuts one GPU holding all rows would compute. Each
// rank's rows (and weights, 1 where a rank has none) are assembled in rank
// order on every GPU with one NCCL broadcast per rank, and the GPU sketch
// runs over all of them; NVLink moves the whole matrix in a few tens of
// milliseconds, and the assembled copy is freed afterwards.
void sketch_all_ranks(DMatrix& d, uint32_t mb, Cuts& c, cudaStream_t stream) {
  Comm& comm = Comm::get();
  const int world = comm.world(), rank = comm.rank();
  // Row counts and weight flags of every rank.
  DeviceBuffer mine(16), all(size_t(world) * 16);
  const uint64_t info[2] = {d.rows, d.weights.empty() ? 0u : 1u};
  XGBB_CUDA(cudaMemcpyAsync(mine.get(), info, 16, cudaMemcpyHostToDevice, stream));
  comm.all_gather(mine.get(), all.get(), 16, stream);
  std::vector<uint64_t> got(size_t(world) * 2);
  XGBB_CUDA(cudaMemcpyAsync(got.data(), all.get(), got.size() * 8, cudaMemcpyDeviceToHost, stream));
  cudaEvent_t ev;
  XGBB_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  XGBB_CUDA(cudaEventRecord(ev, stream));
  comm.wait(ev, "the row counts of every rank");
  std::vector<uint64_t> off(size_t(world) + 1, 0);
  bool weighted = false;
  for (int r = 0; r < world; ++r) {
    off[r + 1] = off[r] + got[2 * r];
    weighted = weighted || got[2 * r + 1];
  }
  const uint64_t total = off[world];
  require(total <= 0xffffffffull, "more than 2^32 - 1 rows over all ranks");
  c.stride = cut_stride(uint32_t(total), mb);
  c.values.assign(size_t(d.cols) * c.stride, 0.0f);
  const size_t row_bytes = size_t(d.cols) * sizeof(float);
  DeviceBuffer X(std::max<size_t>(total * row_bytes, 16)), W;
  if (d.rows) {
    XGBB_CUDA(cudaMemcpyAsync(X.as<char>() + off[rank] * row_bytes, d.device_data(stream), d.rows * row_bytes,
                              cudaMemcpyDeviceToDevice, stream));
  }
  if (weighted) {
    W.resize(std::max<size_t>(total * 4, 16));
    std::vector<float> w = d.weights.empty() ? std::vector<float>(d.rows, 1.0f) : d.weights;
    if (d.rows)
      XGBB_CUDA(cudaMemcpyAsync(W.as<float>() + off[rank], w.data(), d.rows * 4, cudaMemcpyHostToDevice, stream));
    XGBB_CUDA(cudaStreamSynchronize(stream));  // `w` leaves scope
  }
  for (int r = 0; r < world; ++r) {
    const uint64_t n = off[r + 1] - off[r];
    if (!n) continue;
    comm.broadcast(X.as<char>() + off[r] * row_bytes, n * row_bytes, r, stream);
    if (weighted) comm.broadcast(W.as<float>() + off[r], n * 4, r, stream);
  }
  XGBB_CUDA(cudaEventRecord(ev, stream));
  comm.wait(ev, "the rows of every rank");
  cudaEventDestroy(ev);
  if (total && d.cols)
    sketch_cuts_device(X.as<float>(), uint32_t(total), d.cols, weighted ? W.as<float>() : nullptr, mb,
                       c.values.data(), c.counts.data(), c.minima.data(), stream);
}
}  // namespace

void DMatrix::quantise(uint32_t mb, const DMatrix* ref, cudaStream_t stream, int threads) {
  if (quantised() && max_bin == mb) return;
  require(mb >= 2, "max_bin must be at least 2.");
  require(mb <= kMaxBins, "max_bin above 256 is not supported by the CUDA histogram kernels.");
  std::shared_ptr<Cuts> c;
  const bool uploaded = bool(d_data);
  Trace trace("quantise");
  if (ref) {
    require(ref->cuts && ref->max_bin == mb, "Quantile reference does not match max_bin.");
    c = ref->cuts;
  } else if (Comm::get().active()) {
    // Rows are split over the ranks of a multi-GPU job (every rank quantises
    // its matrix together): the cuts cover all ranks' rows.
    c = std::make_shared<Cuts>();
    c->cols = cols;
    c->max_bin = mb;
    c->counts.assign(cols, 0);
    c->minima.assign(cols, -INFINITY);
    sketch_all_ranks(*this, mb, *c, stream);
    c->upload();
  } else {
    c = std::make_shared<Cuts>();
    c->cols = cols;
    c->max_bin = mb;
    c->stride = cut_stride(rows, mb);
    c->values.assign(size_t(cols) * c->stride, 0.0f);
    c->counts.assign(cols, 0);
    c->minima.assign(cols, -INFINITY);
    // The GPU sketch (the same cuts, bit for bit) takes matrices of 2^24
    // values or more when the device holds the matrix plus its runs; the
    // host sketch takes smaller ones. XGBB_SKETCH=host|device overrides.
    const char* where = std::getenv("XGBB_SKETCH");
    bool on_device = false;
    if (rows && cols) {
      size_t free_b = 0, total_b = 0;
      const size_t need = size_t(rows) * cols * sizeof(float) + size_t(rows) * 32 + (1ull << 30);
      on_device = uint64_t(rows) * cols >= (1ull << 24) && cudaMemGetInfo(&free_b, &total_b) == cudaSuccess &&
                  need <= free_b;
      if (where && std::strcmp(where, "device") == 0) on_device = true;
      if (where && std::strcmp(where, "host") == 0) on_device = false;
    }
    if (on_device) {
      const float* X = device_data(stream);
      trace.mark("upload and validate", stream);
      DeviceBuffer w;
      if (!weights.empty()) {
        w.resize(weights.size() * 4);
        XGBB_CUDA(cudaMemcpyAsync(w.get(), weights.data(), weights.size() * 4, cudaMemcpyHostToDevice, stream));
      }
      sketch_cuts_device(X, rows, cols, w.as<float>(), mb, c->values.data(), c->counts.data(), c->minima.data(),
                         stream);
    } else {
      sketch_cuts(host, rows, cols, weights.empty() ? nullptr : weights.data(), mb, c->values.data(),
                  c->counts.data(), c->minima.data(), threads);
    }
    c->upload();
  }
  max_bin = mb;
  trace.mark("cuts", stream);
  set_cuts(std::move(c), stream);
  trace.mark("binning and feature-major copy", stream);
  // The raw matrix was uploaded only for the sketch; predictions upload it
  // again on demand.
  if (!uploaded && d_data) {
    XGBB_CUDA(cudaStreamSynchronize(stream));
    d_data.release();
    trace.mark("release of the uploaded matrix", stream);
  }
}

// ---------------------------------------------------------------------------
// Training state for one matrix.
// ---------------------------------------------------------------------------
// Pinned upload words of a host-driven tree: an evaluation's segments and
// tile offsets (3 * kMaxFrontier + 1), or a partition's items, tile offsets
// and cursors (8 * kQueueBatch + 1).
constexpr size_t kQueueUpWords = 3 * size_t(kMaxFrontier) + 1 > 8 * size_t(kQueueBatch) + 1
                                     ? 3 * size_t(kMaxFrontier) + 1
                                     : 8 * size_t(kQueueBatch) + 1;

struct Booster::TrainState {
  std::weak_ptr<DMatrix> owner;
  DMatrix* d = nullptr;
  uint32_t rows = 0, groups = 1, margin_rounds = 0;
  unsigned long long rows_total = 0;  // rows over all ranks
  DeviceBuffer margins, pairs, mass, scales, best_mine, best_all;
  uint32_t cols_pad = 0;
  DeviceBuffer state, ids[2], sums[2], seg_begin[2], seg_count[2], parent_slot, built_left,
      tile_offset, ptile_offset, cursor_l, cursor_r, counts_local, counts_global, mode, slot_leaf,
      keys[2], cand, nodes, built, bank[2], rows_buf[2], level_rows, level_nodes, ord[2];
  TreeWorkspace ws{};
  HistConfig hc{};
  std::vector<cudaGraphExec_t> graphs;
  // Host copies of each round's trees, two sets: a round's copies land in
  // set (round & 1) while the host reads the previous round's set.
  DevNode* host_nodes[2] = {};                       // pinned [groups][capacity]
  DriverState* host_state[2] = {};                   // pinned [groups]
  unsigned long long* host_level_rows[2] = {};       // pinned [groups][kMaxDepth]
  uint32_t* host_level_nodes[2] = {};                // pinned [groups][kMaxDepth]
  cudaEvent_t copied[2] = {};                        // the set's copies are complete
  // Squared error without weights: every Hessian is 1 and the histograms
  // count rows instead of summing Hessians. Baked into the histogram
  // configuration and the captured graphs.
  bool unit_hessian = false;
  int pending = -1;        // set of a launched round not yet turned into trees
  bool pending_captured = false;
  uint32_t parity = 0;
  uint32_t capacity = 0;
  std::vector<cudaEvent_t> events;  // profiling: [parity][groups][levels][phase marks]
  // Host-driven trees (loss-guided, leaf budgets, depth > 10): row order and
  // its partition scratch, node histograms and candidates of one batch, the
  // batch descriptors, and pinned landing buffers for the host's reads.
  DeviceBuffer q_order, q_scratch, q_built, q_cand, q_keys, q_sums, q_seg, q_items, q_cursor, q_best, q_nodes,
      q_totals;
  // Level histograms from the rows' present codes (sparse matrices).
  bool csr = false;
  DeviceBuffer csr_totals;
  uint32_t q_slots = 0;
  NodeBest* q_best_host = nullptr;   // pinned [kMaxFrontier]
  uint32_t* q_cursor_host = nullptr; // pinned [2 * kQueueBatch]
  uint32_t* q_up_host = nullptr;     // pinned upload staging
  long long* q_sums_host = nullptr;  // pinned [2 * kMaxFrontier]
  cudaEvent_t q_done = nullptr;
  ~TrainState() {
    if (q_best_host) cudaFreeHost(q_best_host);
    if (q_cursor_host) cudaFreeHost(q_cursor_host);
    if (q_up_host) cudaFreeHost(q_up_host);
    if (q_sums_host) cudaFreeHost(q_sums_host);
    if (q_done) cudaEventDestroy(q_done);
    for (auto g : graphs)
      if (g) cudaGraphExecDestroy(g);
    for (auto e : events) cudaEventDestroy(e);
    for (int b = 0; b < 2; ++b) {
      if (copied[b]) cudaEventDestroy(copied[b]);
      if (host_nodes[b]) cudaFreeHost(host_nodes[b]);
      if (host_state[b]) cudaFreeHost(host_state[b]);
      if (host_level_rows[b]) cudaFreeHost(host_level_rows[b]);
      if (host_level_nodes[b]) cudaFreeHost(host_level_nodes[b]);
    }
  }
};

Booster::Booster(std::vector<std::shared_ptr<DMatrix>> cache) {
  for (auto& d : cache) cache_.push_back(d);
  // The device current at creation trains this booster. Without a GPU a
  // booster still loads, saves and describes models; training and
  // prediction then fail with a clear error.
  int n = 0;
  if (cudaGetDeviceCount(&n) == cudaSuccess && n > 0) {
    XGBB_CUDA(cudaGetDevice(&device_));
    XGBB_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
  } else {
    cudaGetLastError();
  }
}

void Booster::gpu() {
  require(stream_ != nullptr, "No CUDA device is available; this library trains on CUDA GPUs only.");
  XGBB_CUDA(cudaSetDevice(device_));
}

Booster::~Booster() {
  Comm::get().remove_release_hook(this);
  if (Comm::get().failed()) {
    // Kernels of an aborted communicator may still use this state; waiting
    // for them or freeing under them could block, so it is left to the
    // process exit that must follow such a failure.
    (void)state_.release();
    return;
  }
  // Copies into pinned buffers may still be in flight.
  if (stream_) cudaStreamSynchronize(stream_);
  state_.reset();
  for (auto e : user_events_)
    if (e) cudaEventDestroy(e);
  if (wait_event_) cudaEventDestroy(wait_event_);
  if (stream_) cudaStreamDestroy(stream_);
}

void Booster::set_param(const std::string& key, const std::string& value) {
  static const std::map<std::string, std::string> alias = {
      {"eta", "learning_rate"}, {"lambda", "reg_lambda"}, {"alpha", "reg_alpha"},
      {"gamma", "min_split_loss"}};
  auto it = alias.find(key);
  if (key == "eval_metric") {
    // Each setting adds a metric to the list (upstream Learner::SetParam).
    std::string& list = params_["eval_metric"];
    size_t b = 0;
    bool present = false;
    while (b <= list.size() && !list.empty()) {
      size_t e = list.find(',', b);
      if (e == std::string::npos) e = list.size();
      present = present || list.compare(b, e - b, value) == 0;
      b = e + 1;
    }
    if (!present && !value.empty()) list += (list.empty() ? "" : ",") + value;
    return;
  }
  params_[it == alias.end() ? key : it->second] = value;
  configured_ = false;
}

// "[iteration]\t<name>-<metric>:<value>..." for every matrix and metric (the
// reference's Learner::evaluate, src/learner.cpp:1025-1048).
std::string Booster::evaluate(int iteration, const std::vector<std::shared_ptr<DMatrix>>& data,
                              const std::vector<std::string>& names) {
  configure();
  require(data.empty() || initialized_, "Model is not yet initialized (not fitted).");
  std::vector<std::string> metrics;
  const std::string list = get_param("eval_metric", "");
  for (size_t b = 0; b < list.size();) {
    size_t e = list.find(',', b);
    if (e == std::string::npos) e = list.size();
    if (e > b) metrics.push_back(list.substr(b, e - b));
    b = e + 1;
  }
  const std::string disable = get_param("disable_default_eval_metric", "0");
  if (metrics.empty() && (disable.empty() || std::stod(disable) == 0))
    metrics.push_back(default_metric(get_param("objective", "reg:squarederror")));
  const bool multiclass = objective_ == kSoftprob || objective_ == kSoftmax;
  std::string out = "[" + std::to_string(iteration) + "]";
  for (size_t i = 0; i < data.size(); ++i) {
    DMatrix& d = *data[i];
    std::vector<uint64_t> shape;
    std::vector<float> pred;
    if (objective_ == kSoftmax) {
      // Metrics read class probabilities, not the predicted classes.
      pred = predict(data[i], true, 0, 0, false, shape);
      for (uint32_t r = 0; r < d.rows; ++r) {
        float* row = pred.data() + size_t(r) * groups_;
        const float mx = *std::max_element(row, row + groups_);
        double sum = 0;
        for (uint32_t k = 0; k < groups_; ++k) sum += std::exp(double(row[k] - mx));
        for (uint32_t k = 0; k < groups_; ++k) row[k] = float(std::exp(double(row[k] - mx)) / sum);
      }
    } else {
      pred = predict(data[i], false, 0, 0, false, shape);
    }
    require(metrics.empty() || d.labels.size() == d.rows, "Evaluation data requires labels.");
    require(d.weights.empty() || d.weights.size() == d.rows, "Evaluation weights must have one entry per row.");
    const float* weights = d.weights.empty() ? nullptr : d.weights.data();
    std::vector<double> values(metrics.size());
    if (!Comm::get().active()) {
      for (size_t j = 0; j < metrics.size(); ++j)
        values[j] = eval_metric(metrics[j], pred.data(), d.rows, groups_, d.labels.data(), weights, multiclass);
    } else {
      evaluate_across_ranks(metrics, pred, d, multiclass, values);
    }
    for (size_t j = 0; j < metrics.size(); ++j) {
      char buf[64];
      std::snprintf(buf, sizeof buf, "%.10g", values[j]);
      out += "\t" + names[i] + "-" + metrics[j] + ":" + buf;
    }
  }
  return out;
}

// Row-sharded evaluation: every rank holds some rows of the matrix, and each
// metric is the metric of all ranks' rows, so that every rank reports the
// same score and early stopping ends training on the same round everywhere.
// The reference evaluates in one process (src/metrics.cpp); this is the
// row-sharded form of the same metrics. Mean-type metrics add up (weighted loss, weight) pairs over the ranks; AUC
// sorts all rows, so its predictions, labels and weights are gathered first.
void Booster::evaluate_across_ranks(const std::vector<std::string>& metrics, const std::vector<float>& pred,
                                    const DMatrix& d, bool multiclass, std::vector<double>& values) {
  Comm& comm = Comm::get();
  const uint32_t world = uint32_t(comm.world());
  const float* weights = d.weights.empty() ? nullptr : d.weights.data();
  std::vector<double> sums(2 * metrics.size(), 0.0);
  bool gather = false;
  for (size_t j = 0; j < metrics.size(); ++j) {
    if (metric_needs_all_rows(metrics[j])) {
      gather = true;
      continue;
    }
    metric_sums(metrics[j], pred.data(), d.rows, groups_, d.labels.data(), weights, multiclass, &sums[2 * j],
                &sums[2 * j + 1]);
  }
  if (!sums.empty()) {
    DeviceBuffer buf(sums.size() * 8);
    XGBB_CUDA(cudaMemcpyAsync(buf.get(), sums.data(), sums.size() * 8, cudaMemcpyHostToDevice, stream_));
    comm.sum_f64(buf.get(), sums.size(), stream_);
    XGBB_CUDA(cudaMemcpyAsync(sums.data(), buf.get(), sums.size() * 8, cudaMemcpyDeviceToHost, stream_));
    wait_stream("an evaluation sum");
  }
  for (size_t j = 0; j < metrics.size(); ++j)
    if (!metric_needs_all_rows(metrics[j])) values[j] = metric_from_sums(metrics[j], sums[2 * j], sums[2 * j + 1]);
  if (!gather) return;
  // Row counts and weight presence of every rank, then each rank's rows
  // padded to the largest count: [world][max_rows] slots.
  std::vector<uint64_t> mine = {d.rows, weights ? 1u : 0u}, counts(2 * size_t(world));
  {
    DeviceBuffer send(16), recv(16 * size_t(world));
    XGBB_CUDA(cudaMemcpyAsync(send.get(), mine.data(), 16, cudaMemcpyHostToDevice, stream_));
    comm.all_gather(send.get(), recv.get(), 16, stream_);
    XGBB_CUDA(cudaMemcpyAsync(counts.data(), recv.get(), counts.size() * 8, cudaMemcpyDeviceToHost, stream_));
    wait_stream("evaluation row counts");
  }
  uint64_t widest = 0, total = 0;
  bool any_weights = false;
  for (uint32_t r = 0; r < world; ++r) {
    widest = std::max(widest, counts[2 * r]);
    total += counts[2 * r];
    any_weights = any_weights || counts[2 * r + 1];
  }
  require(total <= UINT32_MAX, "Evaluation data has too many rows across workers.");
  // One record per row: groups predictions, the label and the weight.
  const size_t width = size_t(groups_) + 2;
  std::vector<float> local(size_t(widest) * width, 0.0f), all(local.size() * world);
  for (uint32_t r = 0; r < d.rows; ++r) {
    std::copy(pred.data() + size_t(r) * groups_, pred.data() + size_t(r + 1) * groups_, &local[r * width]);
    local[r * width + groups_] = d.labels[r];
    local[r * width + groups_ + 1] = weights ? weights[r] : 1.0f;
  }
  if (!local.empty()) {
    DeviceBuffer send(local.size() * 4), recv(all.size() * 4);
    XGBB_CUDA(cudaMemcpyAsync(send.get(), local.data(), local.size() * 4, cudaMemcpyHostToDevice, stream_));
    comm.all_gather(send.get(), recv.get(), local.size() * 4, stream_);
    XGBB_CUDA(cudaMemcpyAsync(all.data(), recv.get(), all.size() * 4, cudaMemcpyDeviceToHost, stream_));
    wait_stream("evaluation rows");
  }
  std::vector<float> p, l, w;
  p.reserve(size_t(total) * groups_);
  l.reserve(total);
  w.reserve(total);
  for (uint32_t r = 0; r < world; ++r)
    for (uint64_t k = 0; k < counts[2 * r]; ++k) {
      const float* rec = &all[(size_t(r) * widest + k) * width];
      p.insert(p.end(), rec, rec + groups_);
      l.push_back(rec[groups_]);
      w.push_back(rec[groups_ + 1]);
    }
  for (size_t j = 0; j < metrics.size(); ++j)
    if (metric_needs_all_rows(metrics[j]))
      values[j] = eval_metric(metrics[j], p.data(), uint32_t(total), groups_, l.data(),
                              any_weights ? w.data() : nullptr, multiclass);
}

std::string Booster::get_param(const std::string& key, const std::string& def) const {
  auto it = params_.find(key);
  return it == params_.end() ? def : it->second;
}

namespace {
float number(const std::map<std::string, std::string>& p, const std::string& k, float def) {
  auto it = p.find(k);
  if (it == p.end() || it->second.empty()) return def;
  return std::stof(it->second);
}
long integer(const std::map<std::string, std::string>& p, const std::string& k, long def) {
  auto it = p.find(k);
  if (it == p.end() || it->second.empty()) return def;
  return std::lround(std::stod(it->second));
}
}  // namespace

void Booster::configure() {
  if (configured_) return;
  static const std::map<std::string, int> objectives = {
      {"reg:squarederror", kSquaredError}, {"reg:linear", kSquaredError},
      {"binary:logistic", kLogistic},       {"reg:logistic", kLogistic},
      {"binary:logitraw", kLogitRaw},       {"multi:softprob", kSoftprob},
      {"multi:softmax", kSoftmax}};
  const std::string obj = get_param("objective", "reg:squarederror");
  auto it = objectives.find(obj);
  require(it != objectives.end(), "Objective is not implemented by the CUDA backend: " + obj);
  const int new_objective = it->second;
  require(!initialized_ || new_objective == objective_, "The objective cannot change after training starts.");
  objective_ = new_objective;
  const std::string device = get_param("device", "cuda");
  require(device == "cuda" || device == "gpu" || device.rfind("cuda:", 0) == 0,
          "This build trains on CUDA devices only; device must be 'cuda', 'cuda:N' or 'gpu'.");
  if (device.rfind("cuda:", 0) == 0) {
    // A booster trains on the device current when it was created (one
    // process per GPU); an explicit ordinal must name that device.
    char* end = nullptr;
    const long ordinal = std::strtol(device.c_str() + 5, &end, 10);
    require(end && *end == '\0' && ordinal >= 0, "Invalid device ordinal: " + device);
    require(!stream_ || ordinal == device_,
            "device '" + device + "' differs from this booster's CUDA device " + std::to_string(device_) +
                "; select the device (xgboost.core.set_device or CUDA_VISIBLE_DEVICES) before creating "
                "the booster.");
  }
  const std::string method = get_param("tree_method", "hist");
  require(method == "hist" || method == "auto" || method == "gpu_hist",
          "CUDA tree training requires tree_method='hist' or 'auto'.");
  require(get_param("booster", "gbtree") == "gbtree", "Only the gbtree booster is implemented.");
  const std::string policy = get_param("grow_policy", "depthwise");
  require(policy == "depthwise" || policy == "lossguide", "grow_policy must be depthwise or lossguide.");
  require(number(params_, "subsample", 1) == 1.0f, "subsample < 1 is not implemented by the CUDA backend.");
  for (auto k : {"colsample_bytree", "colsample_bylevel", "colsample_bynode"})
    require(number(params_, k, 1) == 1.0f, std::string(k) + " < 1 is not implemented by the CUDA backend.");
  require(integer(params_, "num_parallel_tree", 1) == 1, "num_parallel_tree > 1 is not implemented.");
  for (auto k : {"monotone_constraints", "interaction_constraints"}) {
    auto v = get_param(k, "");
    require(v.empty() || v == "()" || v == "[]", std::string(k) + " are not implemented.");
  }
  // The reference's limits (src/learner.cpp:258-260). Loss-guided trees,
  // leaf budgets and depths the level-synchronous device driver does not
  // cover (0 = unlimited, or above 10) grow host-driven (src/tree.cpp:376-384).
  const long max_depth = integer(params_, "max_depth", 6), max_leaves = integer(params_, "max_leaves", 0);
  require(max_depth >= 0 && max_leaves >= 0, "max_depth and max_leaves must be nonnegative.");
  require(max_depth <= 30 || max_leaves, "max_depth must not exceed 30 unless max_leaves is constrained.");
  require(max_leaves <= (long(INT32_MAX) + 1) / 2, "max_leaves exceeds the tree node index range.");
  require(max_depth || max_leaves, "max_depth and max_leaves cannot both be unconstrained.");
  tp_.max_depth = uint32_t(std::min<long>(max_depth, INT32_MAX));
  lossguide_ = policy == "lossguide";
  max_leaves_ = uint32_t(max_leaves);
  // cuda_sparse_hist=1: node histograms from each row's present values (the
  // reference's CSR histograms, kernels/histogram_csr.metal.h), on the
  // host-driven path; the trees are the same.
  sparse_hist_ = integer(params_, "cuda_sparse_hist", 0) != 0;
  host_driven_ = lossguide_ || max_leaves_ || tp_.max_depth == 0 || tp_.max_depth > kMaxDepth || sparse_hist_;
  tp_.eta = number(params_, "learning_rate", 0.3f);
  tp_.reg_lambda = number(params_, "reg_lambda", 1.0f);
  tp_.reg_alpha = number(params_, "reg_alpha", 0.0f);
  tp_.min_split_loss = number(params_, "min_split_loss", 0.0f);
  tp_.min_child_weight = number(params_, "min_child_weight", 1.0f);
  tp_.max_delta_step = number(params_, "max_delta_step", 0.0f);
  for (float v : {tp_.reg_lambda, tp_.reg_alpha, tp_.min_split_loss, tp_.min_child_weight,
                  tp_.max_delta_step, tp_.eta})
    require(v >= 0 && std::isfinite(v), "Tree parameters must be finite and nonnegative.");
  spw_ = number(params_, "scale_pos_weight", 1.0f);
  const uint32_t mb = uint32_t(integer(params_, "max_bin", 256));
  // A loaded (or reset) model has no quantised training state yet, so its
  // continued training may pick any max_bin.
  require(!initialized_ || mb == max_bin_ || trees_.empty() || !state_,
          "max_bin cannot change after training starts.");
  max_bin_ = mb;
  if (objective_ == kSoftprob || objective_ == kSoftmax) {
    const long nc = integer(params_, "num_class", 0);
    require(nc >= 2, "Multiclass requires num_class >= 2.");
    require(!initialized_ || uint32_t(nc) == groups_, "num_class cannot change after training starts.");
    groups_ = uint32_t(nc);
  } else {
    groups_ = 1;
  }
  profile_level = int(integer(params_, "cuda_profile", 0));
  profiling = profile_level != 0;
  configured_ = true;
  if (state_) state_.reset();  // parameters are baked into captured graphs
}

void Booster::initialize(DMatrix& d, bool custom) {
  require(d.cols > 0, "Data must contain at least one feature.");
  num_feature_ = d.cols;
  base_score_.assign(groups_, 0.5f);
  const auto bs = params_.find("base_score");
  if (bs != params_.end()) {
    base_score_.assign(groups_, std::stof(bs->second));
  } else if (custom) {
    // A custom objective starts from 0.5: the intercept is only estimated
    // for built-in objectives (src/learner.cpp:300-333 in the reference).
  } else {
    d.upload_info(stream_);
    // The intercept is a fixed-order sum over the rows of every rank: with
    // rows sharded, each rank gathers all labels (and weights) first, so the
    // result does not depend on the number of GPUs.
    Comm& comm = Comm::get();
    const float* labels = d.d_labels.as<float>();
    const float* weights = d.d_weights.as<float>();
    uint64_t total = d.rows;
    DeviceBuffer all_labels, all_weights;
    if (comm.active()) {
      const int world = comm.world(), rank = comm.rank();
      DeviceBuffer counts(size_t(world) * 8);
      std::vector<unsigned long long> hc(world, 0);
      hc[rank] = d.rows;
      XGBB_CUDA(cudaMemcpyAsync(counts.get(), hc.data(), world * 8, cudaMemcpyHostToDevice, stream_));
      comm.sum_u64(counts.get(), world, stream_);
      XGBB_CUDA(cudaMemcpyAsync(hc.data(), counts.get(), world * 8, cudaMemcpyDeviceToHost, stream_));
      XGBB_CUDA(cudaStreamSynchronize(stream_));
      unsigned long long w_flag = d.weights.empty() ? 0 : 1;
      {
        DeviceBuffer f(8);
        XGBB_CUDA(cudaMemcpyAsync(f.get(), &w_flag, 8, cudaMemcpyHostToDevice, stream_));
        comm.sum_u64(f.get(), 1, stream_);
        XGBB_CUDA(cudaMemcpyAsync(&w_flag, f.get(), 8, cudaMemcpyDeviceToHost, stream_));
        XGBB_CUDA(cudaStreamSynchronize(stream_));
      }
      require(w_flag == 0 || w_flag == uint64_t(world), "Either every rank or no rank must set weights.");
      total = 0;
      std::vector<uint64_t> offset(world);
      for (int r = 0; r < world; ++r) {
        offset[r] = total;
        total += hc[r];
      }
      require(total < (1ull << 32), "Too many rows over all ranks.");
      all_labels.resize(std::max<uint64_t>(total, 1) * 4);
      if (w_flag) all_weights.resize(std::max<uint64_t>(total, 1) * 4);
      XGBB_CUDA(cudaMemcpyAsync(all_labels.as<float>() + offset[rank], labels, size_t(d.rows) * 4,
                                cudaMemcpyDeviceToDevice, stream_));
      if (w_flag)
        XGBB_CUDA(cudaMemcpyAsync(all_weights.as<float>() + offset[rank], weights, size_t(d.rows) * 4,
                                  cudaMemcpyDeviceToDevice, stream_));
      for (int r = 0; r < world; ++r) {
        comm.broadcast(all_labels.as<float>() + offset[r], hc[r] * 4, r, stream_);
        if (w_flag) comm.broadcast(all_weights.as<float>() + offset[r], hc[r] * 4, r, stream_);
      }
      labels = all_labels.as<float>();
      weights = w_flag ? all_weights.as<float>() : nullptr;
    }
    const uint32_t chunks = uint32_t((total + 1023) / 1024);
    DeviceBuffer sums(std::max<uint32_t>(chunks, 1) * 2 * sizeof(double));
    std::vector<double> host(size_t(chunks) * 2);
    for (uint32_t k = 0; k < groups_; ++k) {
      launch_base_chunks(objective_, labels, weights, uint32_t(total), k, spw_, sums.as<double>(),
                         stream_);
      if (chunks)
        XGBB_CUDA(cudaMemcpyAsync(host.data(), sums.get(), host.size() * 8, cudaMemcpyDeviceToHost, stream_));
      XGBB_CUDA(cudaStreamSynchronize(stream_));
      double sy = 0, sw = 0;
      for (uint32_t c = 0; c < chunks; ++c) {
        sy = sy + host[2 * c];
        sw = sw + host[2 * c + 1];
      }
      base_score_[k] = sw > 0 ? float(sy / sw) : (objective_ == kSquaredError && total == 0 ? 0.0f : 0.5f);
    }
  }
  base_margin_ = score_margins(base_score_);
  if ((objective_ == kSoftprob || objective_ == kSoftmax) && bs == params_.end()) base_score_ = base_margin_;
  initialized_ = true;
}

// Scores to margins (src/objectives.cpp:17-31; the multiclass intercept of
// kernels/boost.metal:404-420): logit for logistic loss, centred logs for
// multiclass scores that were not given as base_score, identity otherwise.
std::vector<float> Booster::score_margins(const std::vector<float>& scores) const {
  std::vector<float> m = scores;
  const size_t G = scores.size();
  if ((objective_ == kSoftprob || objective_ == kSoftmax) && !params_.count("base_score")) {
    float mean = 0;
    for (size_t j = 0; j < G; ++j) mean += std::log(std::max(scores[j], 1.0e-6f));
    for (size_t k = 0; k < G; ++k) m[k] = std::log(std::max(scores[k], 1.0e-6f)) - mean / float(G);
  } else if (objective_ == kLogistic) {
    for (size_t k = 0; k < G; ++k) {
      require(scores[k] >= 0 && scores[k] <= 1, "base_score must be in [0,1] for logistic loss.");
      const float v = std::min(std::max(scores[k], 1.0e-6f), 1.0f - 1.0e-6f);
      m[k] = -std::log(1.0f / v - 1.0f);
    }
  }
  return m;
}

Booster::TrainState& Booster::train_state(const std::shared_ptr<DMatrix>& dp, bool custom) {
  DMatrix& d = *dp;
  const bool unit_hessian = !custom && objective_ == kSquaredError && d.weights.empty();
  if (state_ && state_->d == &d && !state_->owner.expired() && state_->unit_hessian == unit_hessian)
    return *state_;
  if (state_) {
    finish_pending();
    XGBB_CUDA(cudaStreamSynchronize(stream_));
  }
  state_.reset();
  auto ts = std::make_unique<TrainState>();
  ts->owner = dp;
  ts->d = &d;
  ts->rows = d.rows;
  ts->groups = groups_;
  ts->rows_total = d.rows;
  ts->unit_hessian = unit_hessian;
  if (Comm::get().active()) {
    DeviceBuffer n(8);
    XGBB_CUDA(cudaMemcpyAsync(n.get(), &ts->rows_total, 8, cudaMemcpyHostToDevice, stream_));
    Comm::get().sum_u64(n.get(), 1, stream_);
    XGBB_CUDA(cudaMemcpyAsync(&ts->rows_total, n.get(), 8, cudaMemcpyDeviceToHost, stream_));
    XGBB_CUDA(cudaStreamSynchronize(stream_));
  }
  // Host-driven trees use the level-synchronous buffers of a one-level tree
  // only (for the common round setup) and their own below.
  const uint32_t n = d.rows, G = groups_, C = d.cols, D = host_driven_ ? 1u : tp_.max_depth;
  const Ellpack& e = d.ell;
  if (host_driven_) {
    require(e.bins <= kMaxBins, "host-driven trees support at most 256 bins per feature");
    ts->q_slots = lossguide_ ? 2u : kMaxFrontier;
    ts->q_order.resize(std::max<size_t>(n, 1) * 4);
    ts->q_scratch.resize(std::max<size_t>(n, 1) * 4);
    ts->q_built.resize(size_t(C) * ts->q_slots * (e.bins + 1) * sizeof(longlong2));
    ts->q_cand.resize(size_t(ts->q_slots) * C * sizeof(DevSplit));
    ts->q_keys.resize(kMaxFrontier * 8);
    ts->q_sums.resize(kMaxFrontier * 16);
    ts->q_seg.resize((3 * size_t(kMaxFrontier) + 1) * 4);
    ts->q_items.resize((6 * size_t(kQueueBatch) + 1) * 4);
    ts->q_cursor.resize(2 * size_t(kQueueBatch) * 4);
    ts->q_best.resize(kMaxFrontier * sizeof(NodeBest));
    ts->q_totals.resize(size_t(ts->q_slots) * 16);
    if (sparse_hist_) d.build_sparse_rows(stream_);
    XGBB_CUDA(cudaMallocHost(reinterpret_cast<void**>(&ts->q_best_host), kMaxFrontier * sizeof(NodeBest)));
    XGBB_CUDA(cudaMallocHost(reinterpret_cast<void**>(&ts->q_cursor_host), 2 * size_t(kQueueBatch) * 4));
    XGBB_CUDA(cudaMallocHost(reinterpret_cast<void**>(&ts->q_up_host), kQueueUpWords * 4));
    XGBB_CUDA(cudaMallocHost(reinterpret_cast<void**>(&ts->q_sums_host), 2 * size_t(kMaxFrontier) * 8));
    XGBB_CUDA(cudaEventCreateWithFlags(&ts->q_done, cudaEventDisableTiming));
  }
  // Sparse matrices build the level histograms from the rows' present codes
  // when at most a quarter of the cells hold a value (cuda_csr_hist: -1
  // decides so, 0 never, 1 always); the results are the same.
  const long csr_mode = integer(params_, "cuda_csr_hist", -1);
  if (!host_driven_ && csr_mode != 0 && (csr_mode == 1 || d.has_missing) && C <= 0x10000u && n) {
    const double density = 1.0 - double(d.missing_cells) / (double(n) * C);
    ts->csr = csr_mode == 1 || density <= 0.25;
    if (ts->csr) {
      d.build_sparse_rows(stream_);
      ts->csr_totals.resize(size_t(kMaxFrontier) * 16);
    }
  }
  ts->margins.resize(std::max<size_t>(size_t(n) * G, 1) * 4);
  ts->pairs.resize(std::max<size_t>(size_t(n) * G, 1) * 8);
  ts->mass.resize(mass_bytes(G));
  ts->scales.resize(size_t(G) * sizeof(float2));
  ts->state.resize(sizeof(DriverState));
  for (int i = 0; i < 2; ++i) {
    ts->ids[i].resize(kMaxFrontier * 4);
    ts->sums[i].resize(kMaxFrontier * 16);
    ts->seg_begin[i].resize(kMaxFrontier * 4);
    ts->seg_count[i].resize(kMaxFrontier * 4);
    ts->keys[i].resize(kMaxFrontier * 8);
    ts->rows_buf[i].resize(std::max<size_t>(n, 1) * 4);
    ts->ord[i].resize(std::max<size_t>(n, 1) * sizeof(float2));
  }
  ts->parent_slot.resize(kMaxFrontier * 4);
  ts->built_left.resize(kMaxFrontier * 4);
  ts->tile_offset.resize((kMaxFrontier + 1) * 4);
  ts->ptile_offset.resize((kMaxFrontier + 1) * 4);
  ts->cursor_l.resize(kMaxFrontier * 4);
  ts->cursor_r.resize(kMaxFrontier * 4);
  ts->counts_local.resize(kMaxFrontier * 8);
  ts->counts_global.resize(kMaxFrontier * 8);
  ts->mode.resize(kMaxFrontier * 4);
  ts->slot_leaf.resize(kMaxFrontier * 8);
  const size_t node_bytes = hist_node_bytes(e);
  const uint32_t max_slots = max_slots_at(D - 1);
  ts->cand.resize(size_t(max_slots) * C * sizeof(DevSplit));
  ts->capacity = (2u << D) - 1;
  ts->nodes.resize(size_t(ts->capacity) * sizeof(DevNode));
  // The built histograms are feature-major, [cols_pad][pairs][bins + 1], with
  // the features padded to a multiple of the ranks so that a reduce-scatter
  // hands every rank whole features.
  const uint32_t world = uint32_t(Comm::get().world());
  uint32_t lo, hi;
  rank_features(C, world, uint32_t(Comm::get().rank()), &ts->cols_pad, &lo, &hi);
  ts->built.resize(size_t(max_pairs_at(D - 1)) * hist_node_bytes(e, ts->cols_pad));
  if (world > 1) {
    ts->best_mine.resize(size_t(kMaxFrontier) * best_record_bytes());
    ts->best_all.resize(size_t(world) * kMaxFrontier * best_record_bytes());
  }
  const uint32_t bank_slots = D >= 2 ? max_slots_at(D - 2) : 1u;
  ts->bank[0].resize(size_t(bank_slots) * node_bytes);
  ts->bank[1].resize(size_t(bank_slots) * node_bytes);
  for (int b = 0; b < 2; ++b) {
    XGBB_CUDA(cudaMallocHost(reinterpret_cast<void**>(&ts->host_nodes[b]),
                             size_t(G) * ts->capacity * sizeof(DevNode)));
    XGBB_CUDA(cudaMallocHost(reinterpret_cast<void**>(&ts->host_state[b]), size_t(G) * sizeof(DriverState)));
    XGBB_CUDA(cudaMallocHost(reinterpret_cast<void**>(&ts->host_level_rows[b]), size_t(G) * kMaxDepth * 8));
    XGBB_CUDA(cudaMallocHost(reinterpret_cast<void**>(&ts->host_level_nodes[b]), size_t(G) * kMaxDepth * 4));
    XGBB_CUDA(cudaEventCreateWithFlags(&ts->copied[b], cudaEventDisableTiming));
  }
  ts->level_rows.resize(kMaxDepth * 8);
  ts->level_nodes.resize(kMaxDepth * 4);

  TreeWorkspace& ws = ts->ws;
  ws.state = ts->state.as<DriverState>();
  for (int i = 0; i < 2; ++i) {
    ws.ids[i] = ts->ids[i].as<uint32_t>();
    ws.sums[i] = ts->sums[i].as<long long>();
    ws.seg_begin[i] = ts->seg_begin[i].as<uint32_t>();
    ws.seg_count[i] = ts->seg_count[i].as<uint32_t>();
    ws.keys[i] = ts->keys[i].as<unsigned long long>();
    ws.bank[i] = ts->bank[i].as<longlong2>();
    ws.rows[i] = ts->rows_buf[i].as<uint32_t>();
    ws.ord[i] = ts->ord[i].as<float2>();
  }
  ws.parent_slot = ts->parent_slot.as<uint32_t>();
  ws.built_left = ts->built_left.as<uint32_t>();
  ws.tile_offset = ts->tile_offset.as<uint32_t>();
  ws.ptile_offset = ts->ptile_offset.as<uint32_t>();
  ws.cursor_l = ts->cursor_l.as<uint32_t>();
  ws.cursor_r = ts->cursor_r.as<uint32_t>();
  ws.counts_local = ts->counts_local.as<uint32_t>();
  ws.counts_global = Comm::get().active() ? ts->counts_global.as<uint32_t>() : ws.counts_local;
  ws.mode = ts->mode.as<uint32_t>();
  ws.slot_leaf = ts->slot_leaf.as<float>();
  ws.cand = ts->cand.as<DevSplit>();
  ws.nodes = ts->nodes.as<DevNode>();
  ws.built = ts->built.as<longlong2>();
  ws.node_capacity = ts->capacity;
  ws.level_rows = ts->level_rows.as<unsigned long long>();
  ws.level_nodes = ts->level_nodes.as<uint32_t>();
  ts->hc = hist_config(e, ts->unit_hessian);
  // One graph per group and round parity: the two differ only in the
  // profiling events they record, so a round's events are read after the
  // next round has been enqueued.
  ts->graphs.assign(size_t(G) * 2, nullptr);
  if (profiling) {
    ts->events.resize(size_t(2) * G * D * (kPhases + 1));
    for (auto& ev : ts->events) XGBB_CUDA(cudaEventCreate(&ev));
  }
  // Margins start from the base margins plus every tree already in the model.
  d.upload_info(stream_);
  DeviceBuffer base(G * 4);
  XGBB_CUDA(cudaMemcpyAsync(base.get(), base_margin_.data(), G * 4, cudaMemcpyHostToDevice, stream_));
  if (trees_.empty()) {
    launch_fill_margins(ts->margins.as<float>(), base.as<float>(), n, G, stream_);
  } else {
    std::vector<uint64_t> shape;
    auto m = predict(dp, true, 0, 0, false, shape);
    XGBB_CUDA(cudaMemcpyAsync(ts->margins.get(), m.data(), m.size() * 4, cudaMemcpyHostToDevice, stream_));
  }
  XGBB_CUDA(cudaStreamSynchronize(stream_));
  ts->margin_rounds = rounds_;
  state_ = std::move(ts);
  if (Comm::get().active()) {
    // Sharded training captures NCCL calls in its graphs; the communicator
    // drops this state (graphs included) before it is destroyed.
    Comm::get().add_release_hook(this, [this] {
      if (Comm::get().failed()) {
        (void)state_.release();  // see ~Booster
        return;
      }
      if (state_) {
        cudaStreamSynchronize(stream_);
        try {
          finish_pending();
        } catch (const std::exception&) {
          // The communicator is going away; a failed round has no model to keep.
        }
      }
      state_.reset();
    });
  }
  return *state_;
}

namespace {
// Device buffers of one group's host-driven tree (owned by the training
// state).
struct QueueDevice {
  Ellpack e;
  TreeParams tp;
  const float2* pairs;  // this group's gradient pairs by row id
  const float2* scale;  // this group's scales (device)
  uint32_t* order;      // row order: each node owns a segment
  uint32_t* scratch;
  longlong2* built;     // [cols][slots][bins + 1]
  DevSplit* cand;       // [slots][cols]
  unsigned long long* keys;
  long long* sums;      // [slots][2]
  DriverState* state;
  uint32_t* seg;        // [slots][2] segments, then [slots + 1] tile offsets
  uint32_t* items;      // [kQueueBatch][5] partition items, then [kQueueBatch + 1] tile offsets
  uint32_t* cursor;     // [kQueueBatch][2]
  NodeBest* best;       // [kMaxFrontier]
  NodeBest* best_host;  // pinned [kMaxFrontier]
  uint32_t* cursor_host;  // pinned [kQueueBatch][2]
  // Pinned staging of the uploads: a pageable copy would wait for the
  // stream's earlier collectives outside the communicator's time limit.
  uint32_t* up_host;      // pinned [kQueueUpWords]
  long long* sums_host;   // pinned [kMaxFrontier][2]
  uint32_t slots;       // node capacity of one evaluation
  // Sparse rows (null for dense histograms) and per-node totals.
  const unsigned long long* sparse_ptr;
  const uint32_t* sparse_entries;
  unsigned long long* node_totals;  // [slots][2]
  cudaEvent_t done;
  cudaStream_t stream;
  int hist_blocks, eval_blocks, part_blocks;
};

// The GPU backend of host-driven trees: node histograms (queue_hist_kernel),
// summed over ranks when the rows are sharded so that every rank takes the
// same decisions, split evaluation (eval_kernel), and row partitions; the
// host waits once per evaluation and once per partition.
class DeviceGrower final : public GrowerBackend {
 public:
  explicit DeviceGrower(const QueueDevice& q) : q_(q) {}

  void evaluate(const std::vector<Segment>& nodes, bool root, const std::vector<long long>& sums,
                std::vector<DevSplit>& out) override {
    const uint32_t n = uint32_t(nodes.size());
    require(n >= 1 && n <= q_.slots, "host-driven tree batch exceeds its buffers");
    uint32_t* up = q_.up_host;
    uint32_t tiles = 0;
    for (uint32_t s = 0; s < n; ++s) {
      up[2 * s] = nodes[s].begin;
      up[2 * s + 1] = nodes[s].count;
      up[2 * size_t(n) + s] = tiles;
      tiles += (nodes[s].count + kQueueTileRows - 1) / kQueueTileRows;
    }
    up[3 * size_t(n)] = tiles;
    XGBB_CUDA(cudaMemcpyAsync(q_.seg, up, (3 * size_t(n) + 1) * 4, cudaMemcpyHostToDevice, q_.stream));
    if (!root) {
      require(sums.size() == 2 * size_t(n), "host-driven tree node sums missing");
      std::copy(sums.begin(), sums.end(), q_.sums_host);
      XGBB_CUDA(cudaMemcpyAsync(q_.sums, q_.sums_host, sums.size() * 8, cudaMemcpyHostToDevice, q_.stream));
    }
    if (q_.sparse_ptr)
      launch_queue_hist_csr(q_.e, q_.sparse_ptr, q_.sparse_entries, q_.order, q_.pairs, q_.scale, q_.seg,
                            q_.seg + 2 * size_t(n), n, tiles, q_.node_totals, q_.built, q_.hist_blocks, q_.stream);
    else
      launch_queue_hist(q_.e, q_.order, q_.pairs, q_.scale, q_.seg, q_.seg + 2 * size_t(n), n, tiles, q_.built,
                        q_.hist_blocks, q_.stream);
    Comm::get().sum_u64(q_.built, size_t(q_.e.cols) * n * (q_.e.bins + 1) * 2, q_.stream);
    queue_evaluate(q_.e, q_.tp, q_.scale, q_.state, n, root, q_.built, q_.sums, q_.cand, q_.keys, q_.best,
                   q_.eval_blocks, q_.stream);
    XGBB_CUDA(cudaMemcpyAsync(q_.best_host, q_.best, size_t(n) * sizeof(NodeBest), cudaMemcpyDeviceToHost,
                              q_.stream));
    XGBB_CUDA(cudaEventRecord(q_.done, q_.stream));
    Comm::get().wait(q_.done, "a host-driven tree's split evaluation");
    out.resize(n);
    for (uint32_t s = 0; s < n; ++s) {
      out[s] = q_.best_host[s].split;
      if (!q_.best_host[s].key) {
        out[s] = DevSplit{};
        out[s].feature = -1;
        out[s].split_bin = -1;
        out[s].gain = -INFINITY;
      }
    }
  }

  void partition(const std::vector<PartitionItem>& items, std::vector<uint32_t>& left) override {
    const uint32_t m = uint32_t(items.size());
    require(m <= kQueueBatch, "host-driven tree batch exceeds its buffers");
    left.assign(m, 0);
    if (!m) return;
    uint32_t* up = q_.up_host;
    uint32_t* cursor = q_.up_host + 6 * size_t(m) + 1;
    uint32_t tiles = 0;
    for (uint32_t i = 0; i < m; ++i) {
      const PartitionItem& it = items[i];
      require(it.feature >= 0 && uint32_t(it.feature) < q_.e.cols, "host-driven tree split feature out of range");
      uint32_t* d = &up[5 * size_t(i)];
      d[0] = it.begin;
      d[1] = it.count;
      d[2] = uint32_t(it.feature);
      d[3] = uint32_t(it.split_bin);
      d[4] = it.default_left;
      up[5 * size_t(m) + i] = tiles;
      tiles += (it.count + kQueuePartRows - 1) / kQueuePartRows;
      cursor[2 * i] = it.begin;
      cursor[2 * i + 1] = it.begin + it.count;
    }
    up[6 * size_t(m)] = tiles;
    XGBB_CUDA(cudaMemcpyAsync(q_.items, up, (6 * size_t(m) + 1) * 4, cudaMemcpyHostToDevice, q_.stream));
    XGBB_CUDA(cudaMemcpyAsync(q_.cursor, cursor, 2 * size_t(m) * 4, cudaMemcpyHostToDevice, q_.stream));
    launch_queue_partition(q_.e, q_.order, q_.scratch, q_.items, q_.items + 5 * size_t(m), m, tiles, q_.cursor,
                           q_.part_blocks, q_.stream);
    XGBB_CUDA(cudaMemcpyAsync(q_.cursor_host, q_.cursor, 2 * size_t(m) * 4, cudaMemcpyDeviceToHost, q_.stream));
    XGBB_CUDA(cudaEventRecord(q_.done, q_.stream));
    Comm::get().wait(q_.done, "a host-driven tree's row partition");
    for (uint32_t i = 0; i < m; ++i) {
      const uint32_t l = q_.cursor_host[2 * i], r = q_.cursor_host[2 * i + 1];
      require(l == r && l >= items[i].begin && l - items[i].begin <= items[i].count,
              "host-driven tree partition lost rows");
      left[i] = l - items[i].begin;
    }
  }

 private:
  QueueDevice q_;
};
}  // namespace

void Booster::record_tree_launches(TrainState& ts, uint32_t g, cudaStream_t s, bool capturing,
                                   uint32_t parity) {
  // Inside a capture the profiling events become external event-record nodes,
  // recorded again at every launch of the graph.
  auto mark = [&](cudaEvent_t ev) {
    if (capturing) XGBB_CUDA(cudaEventRecordWithFlags(ev, s, cudaEventRecordExternal));
    else XGBB_CUDA(cudaEventRecord(ev, s));
  };
  DMatrix& d = *ts.d;
  Comm& comm = Comm::get();
  TreeLaunch tl{};
  tl.ell = d.ell;
  tl.params = tp_;
  tl.pairs = ts.pairs.as<float2>() + size_t(g) * ts.rows;
  tl.scale = ts.scales.as<float2>() + g;
  tl.max_bits = mass_view(ts.mass.get(), ts.groups).max_bits + 2 * g;
  tl.margins = ts.margins.as<float>();
  tl.groups = ts.groups;
  tl.group = g;
  tl.unit_hessian = ts.unit_hessian;
  tl.feature_group = ts.hc.feature_group;
  tl.min_limbs = uint32_t(integer(params_, "cuda_hist_limbs", 0));
  // cuda_hist_staged3=0 keeps three-limb rounds on the unstaged kernel
  // (tuning and cross-checks; results are identical).
  tl.staged3 = integer(params_, "cuda_hist_staged3", 1) != 0;
  tl.hist_smem = ts.hc.smem;
  tl.hist_threads = ts.hc.threads;
  const int sms = device_sms();
  tl.hist_blocks = sms;
  tl.eval_blocks = sms * 8;
  tl.part_blocks = sms * 8;
  const TreeWorkspace& ws = ts.ws;
  const uint32_t D = tp_.max_depth;
  // Each rank evaluates the splits of its own feature range; one GPU evaluates
  // them all.
  const uint32_t world = uint32_t(comm.world()), rank = uint32_t(comm.rank());
  rank_features(d.ell.cols, world, rank, &tl.cols_pad, &tl.f_lo, &tl.f_hi);
  if (ts.csr) {
    tl.csr_ptr = d.sparse_ptr.as<unsigned long long>();
    tl.csr_entries = d.sparse_entries.as<uint32_t>();
    tl.csr_totals = ts.csr_totals.as<unsigned long long>();
  }
  const uint32_t per_rank = tl.cols_pad / world;
  // Phase marks of a level: mark k opens phase k and closes phase k - 1.
  // cuda_profile=1 records the histogram's two marks only.
  auto phase = [&](uint32_t depth, uint32_t k) {
    if (!profiling || (profile_level < 2 && k > kPhaseHist + 1)) return;
    mark(ts.events[(((size_t(parity) * ts.groups + g) * D + depth) * (kPhases + 1)) + k]);
  };
  tree_init(ws, tl, s);
  for (uint32_t depth = 0; depth < D; ++depth) {
    phase(depth, kPhaseHist);
    tree_level_hist(ws, tl, depth, s);
    phase(depth, kPhaseReduce);
    // Sum the built histograms over ranks, each rank receiving its features.
    comm.reduce_scatter_u64(ws.built, size_t(per_rank) * max_pairs_at(depth) * (d.ell.bins + 1) * 2, s);
    if (!capturing && g == 0 && capture.depth == int(depth) && !capture.ready) capture_level(ts, depth, tl);
    phase(depth, kPhaseEval);
    tree_level_eval(ws, tl, depth, s);
    phase(depth, kPhaseGather);
    if (comm.active()) {
      tree_level_pack_best(ws, tl, depth, ts.best_mine.get(), s);
      comm.all_gather(ts.best_mine.get(), ts.best_all.get(), size_t(kMaxFrontier) * best_record_bytes(), s);
      tree_level_merge_best(ws, tl, depth, ts.best_all.get(), world, s);
    }
    phase(depth, kPhasePartition);
    tree_level_control(ws, tl, depth, s);
    tree_level_partition(ws, tl, depth, s);
    phase(depth, kPhaseCounts);
    if (depth + 1 < D) {
      tree_level_counts(ws, depth, s);
      if (comm.active()) {
        XGBB_CUDA(cudaMemcpyAsync(ws.counts_global, ws.counts_local, kMaxFrontier * 8,
                                  cudaMemcpyDeviceToDevice, s));
        comm.sum_u32(ws.counts_global, kMaxFrontier * 2, s);
      }
      tree_level_plan(ws, tl, depth + 1, s);
    }
    phase(depth, kPhases);
  }
}

// Copies this level's built histograms (after the sum over ranks) and the
// nodes they belong to into `capture`. The built layout is feature-major,
// [cols_pad][pair_stride][B + 1]; the capture is node-major.
void Booster::capture_level(TrainState& ts, uint32_t depth, const TreeLaunch& tl) {
  wait_stream("a level-histogram capture");
  const TreeWorkspace& ws = ts.ws;
  DriverState st{};
  XGBB_CUDA(cudaMemcpy(&st, ws.state, sizeof st, cudaMemcpyDeviceToHost));
  const uint32_t pairs = st.frontier ? (depth ? st.pairs : 1u) : 0u;
  const uint32_t stride = max_pairs_at(depth), B1 = ts.d->ell.bins + 1, nf = tl.f_hi - tl.f_lo;
  std::vector<long long> built(size_t(nf) * stride * B1 * 2);
  if (!built.empty())
    XGBB_CUDA(cudaMemcpy(built.data(), ws.built + size_t(tl.f_lo) * stride * B1, built.size() * 8,
                         cudaMemcpyDeviceToHost));
  std::vector<uint32_t> ids(size_t(2) * std::max(pairs, 1u)), left(std::max(pairs, 1u));
  if (pairs) {
    XGBB_CUDA(cudaMemcpy(ids.data(), ws.ids[depth & 1], ids.size() * 4, cudaMemcpyDeviceToHost));
    XGBB_CUDA(cudaMemcpy(left.data(), ws.built_left, left.size() * 4, cudaMemcpyDeviceToHost));
  }
  capture.pairs = pairs;
  capture.f_lo = tl.f_lo;
  capture.f_hi = tl.f_hi;
  capture.bins1 = B1;
  capture.node_ids.assign(pairs, 0);
  capture.hist.assign(size_t(pairs) * nf * B1 * 2, 0);
  for (uint32_t p = 0; p < pairs; ++p) {
    capture.node_ids[p] = depth ? ids[2 * p + (left[p] ? 0 : 1)] : ids[0];
    for (uint32_t f = 0; f < nf; ++f)
      std::memcpy(&capture.hist[(size_t(p) * nf + f) * B1 * 2], &built[(size_t(f) * stride + p) * B1 * 2],
                  size_t(B1) * 16);
  }
  capture.ready = true;
}

// Group g's tree (node table, driver state, level statistics) into host set
// `b`, ordered after the tree on the stream; the next group reuses the device
// buffers.
static void copy_tree_out(const TreeWorkspace& ws, uint32_t capacity, uint32_t g, DevNode* nodes,
                          DriverState* state, unsigned long long* level_rows, uint32_t* level_nodes,
                          cudaStream_t s) {
  XGBB_CUDA(cudaMemcpyAsync(nodes + size_t(g) * capacity, ws.nodes, size_t(capacity) * sizeof(DevNode),
                            cudaMemcpyDeviceToHost, s));
  XGBB_CUDA(cudaMemcpyAsync(state + g, ws.state, sizeof(DriverState), cudaMemcpyDeviceToHost, s));
  XGBB_CUDA(cudaMemcpyAsync(level_rows + size_t(g) * kMaxDepth, ws.level_rows, kMaxDepth * 8,
                            cudaMemcpyDeviceToHost, s));
  XGBB_CUDA(cudaMemcpyAsync(level_nodes + size_t(g) * kMaxDepth, ws.level_nodes, kMaxDepth * 4,
                            cudaMemcpyDeviceToHost, s));
}

void Booster::run_round(TrainState& ts, const CustomGradients* custom) {
  // With collectives on the stream, the previous round must have completed
  // before new NCCL calls are enqueued: an enqueue behind a collective that
  // can no longer complete (a rank failed or left) could block inside NCCL,
  // out of reach of the communicator's time limit.
  if (Comm::get().active() && ts.pending >= 0)
    Comm::get().wait(ts.copied[ts.pending], "the previous training round");
  DMatrix& d = *ts.d;
  const uint32_t n = ts.rows, G = ts.groups;
  d.upload_info(stream_);
  const MassAccum mass = mass_view(ts.mass.get(), G);
  float2* pairs = ts.pairs.as<float2>();
  Comm& comm = Comm::get();
  // Exact gradient masses are summed over ranks, so every rank derives the
  // same power-of-two scales as a single GPU holding all rows would.
  XGBB_CUDA(cudaMemsetAsync(ts.mass.get(), 0, mass_bytes(G), stream_));
  if (custom) {
    // Caller-supplied pairs and their largest magnitudes, as the gradient
    // kernel would have written them. The copies leave pageable memory
    // before cudaMemcpyAsync returns.
    if (n) XGBB_CUDA(cudaMemcpyAsync(pairs, custom->pairs.data(), size_t(n) * G * sizeof(float2),
                                     cudaMemcpyHostToDevice, stream_));
    XGBB_CUDA(cudaMemcpyAsync(mass.max_bits, custom->max_bits.data(), size_t(2) * G * sizeof(uint32_t),
                              cudaMemcpyHostToDevice, stream_));
  } else {
    launch_gradients(objective_, ts.margins.as<float>(), d.d_labels.as<float>(),
                     d.d_weights.as<float>(), n, G, spw_, pairs, mass, stream_);
  }
  comm.max_u32(mass.max_bits, 2 * G, stream_);
  launch_mass_window(pairs, n, G, mass, stream_);
  if (comm.active()) {
    launch_window_to_limbs(mass, G, stream_);
    comm.sum_u64(mass.limbs, 8 * size_t(G), stream_);
    launch_limbs_to_window(mass, G, stream_);
  }
  launch_scales(pairs, n, G, mass, ts.scales.as<float2>(), ts.rows_total, true, stream_);
  launch_mass_exact(pairs, n, G, mass, stream_);
  comm.sum_u64(mass.exact, 20 * size_t(G), stream_);
  launch_scales_exact(G, mass, ts.scales.as<float2>(), stream_);
  if (host_driven_) {
    grow_host_driven(ts);
    return;
  }
  const bool use_graph = integer(params_, "cuda_graph", 1) != 0;
  bool captured = false;
  const uint32_t b = ts.parity;
  for (uint32_t g = 0; g < G; ++g) {
    // A level capture reads the histograms between two launches, so that
    // tree runs without its graph (the same launches, issued one by one).
    const bool capture_here = g == 0 && capture.depth >= 0 && !capture.ready;
    if (use_graph && !capture_here) {
      cudaGraphExec_t& exec = ts.graphs[size_t(g) * 2 + b];
      if (!exec) {
        // Kernel attributes are set on first use, outside any capture.
        record_tree_launches(ts, g, stream_, false, b);
        wait_stream("the first tree of a group");
        // The eager tree above already trained this group; replaying it would
        // train the same tree twice, so the graphs of both parities are only
        // captured here.
        for (uint32_t p = 0; p < 2; ++p) {
          cudaGraph_t graph;
          XGBB_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
          record_tree_launches(ts, g, stream_, true, p);
          XGBB_CUDA(cudaStreamEndCapture(stream_, &graph));
          XGBB_CUDA(cudaGraphInstantiate(&ts.graphs[size_t(g) * 2 + p], graph, 0));
          XGBB_CUDA(cudaGraphDestroy(graph));
        }
        captured = true;
      } else {
        XGBB_CUDA(cudaGraphLaunch(exec, stream_));
      }
    } else {
      record_tree_launches(ts, g, stream_, false, b);
    }
    copy_tree_out(ts.ws, ts.capacity, g, ts.host_nodes[b], ts.host_state[b], ts.host_level_rows[b],
                  ts.host_level_nodes[b], stream_);
  }
  XGBB_CUDA(cudaEventRecord(ts.copied[b], stream_));
  profile.csr = ts.csr;
  ++rounds_;
  ts.margin_rounds = rounds_;
  ts.parity ^= 1u;
  // The round runs on while the host turns the previous round into trees.
  finish_round(ts);
  ts.pending = int(b);
  ts.pending_captured = captured;
}

// One round of host-driven trees (grower.cpp), one per group, each grown to
// completion before the next; the margins take each tree's leaves on the
// device.
void Booster::grow_host_driven(TrainState& ts) {
  DMatrix& d = *ts.d;
  const uint32_t n = ts.rows, G = ts.groups;
  // The scales follow the round's collectives on the stream: wait for them
  // within the communicator's limit, then read.
  wait_stream("a training round's gradient scales");
  std::vector<float2> scales(G);
  XGBB_CUDA(cudaMemcpyAsync(scales.data(), ts.scales.get(), G * sizeof(float2), cudaMemcpyDeviceToHost, stream_));
  XGBB_CUDA(cudaStreamSynchronize(stream_));
  const int sms = device_sms();
  QueueDevice q{};
  q.e = d.ell;
  q.tp = tp_;
  q.order = ts.q_order.as<uint32_t>();
  q.scratch = ts.q_scratch.as<uint32_t>();
  q.built = ts.q_built.as<longlong2>();
  q.cand = ts.q_cand.as<DevSplit>();
  q.keys = ts.q_keys.as<unsigned long long>();
  q.sums = ts.q_sums.as<long long>();
  q.state = ts.state.as<DriverState>();
  q.seg = ts.q_seg.as<uint32_t>();
  q.items = ts.q_items.as<uint32_t>();
  q.cursor = ts.q_cursor.as<uint32_t>();
  q.best = ts.q_best.as<NodeBest>();
  q.best_host = ts.q_best_host;
  q.cursor_host = ts.q_cursor_host;
  q.up_host = ts.q_up_host;
  q.sums_host = ts.q_sums_host;
  q.slots = ts.q_slots;
  q.sparse_ptr = sparse_hist_ ? d.sparse_ptr.as<unsigned long long>() : nullptr;
  q.sparse_entries = sparse_hist_ ? d.sparse_entries.as<uint32_t>() : nullptr;
  q.node_totals = ts.q_totals.as<unsigned long long>();
  q.done = ts.q_done;
  q.stream = stream_;
  q.hist_blocks = sms * 8;
  q.eval_blocks = sms * 8;
  q.part_blocks = sms * 8;
  GrowerParams gp;
  gp.tree = tp_;
  gp.lossguide = lossguide_;
  gp.max_leaves = max_leaves_;
  std::vector<HostTree> grown(G);
  for (uint32_t g = 0; g < G; ++g) {
    q.pairs = ts.pairs.as<float2>() + size_t(g) * n;
    q.scale = ts.scales.as<float2>() + g;
    gp.scale_g = scales[g].x;
    gp.scale_h = scales[g].y;
    launch_queue_iota(q.order, n, stream_);
    DeviceGrower backend(q);
    HostTree& t = grown[g];
    t.group = g;
    t.nodes = grow_tree_host_driven(backend, n, gp);
    // The previous group's margin update has completed (the growth above
    // waited on the stream), so the node buffer may be reallocated.
    ts.q_nodes.resize(t.nodes.size() * sizeof(DevNode));
    XGBB_CUDA(cudaMemcpyAsync(ts.q_nodes.get(), t.nodes.data(), t.nodes.size() * sizeof(DevNode),
                              cudaMemcpyHostToDevice, stream_));
    launch_queue_margins(d.ell, ts.q_nodes.as<DevNode>(), uint32_t(t.nodes.size()), ts.margins.as<float>(), G, g,
                         stream_);
  }
  wait_stream("a host-driven round's margin update");
  for (HostTree& t : grown) trees_.push_back(std::move(t));
  ++rounds_;
  ts.margin_rounds = rounds_;
}

// Turns the pending round's host copies into trees (and profile figures).
void Booster::finish_round(TrainState& ts) {
  if (ts.pending < 0) return;
  const int b = ts.pending;
  const bool captured = ts.pending_captured;
  ts.pending = -1;
  Comm::get().wait(ts.copied[b], "a training round");
  DMatrix& d = *ts.d;
  const uint32_t G = ts.groups;
  for (uint32_t g = 0; g < G; ++g) {
    const DriverState st = ts.host_state[b][g];
    require(!(st.error & kErrLayout), "Histogram kernel: shared memory is not 128-byte aligned.");
    require(!st.error, "GPU tree driver produced an invalid tree.");
    require(st.node_count >= 1 && st.node_count <= ts.capacity, "GPU tree driver node count out of range.");
    HostTree t;
    t.group = g;
    const DevNode* src = ts.host_nodes[b] + size_t(g) * ts.capacity;
    t.nodes.assign(src, src + st.node_count);
    trees_.push_back(std::move(t));
  }
  if (profiling && !captured) {
    // Algorithmic bytes of a histogram launch: per row the feature codes, the
    // float gradient pair and (below the root) the row id; per built node the
    // int64 histogram written.
    const uint32_t D = tp_.max_depth;
    const Ellpack& e = d.ell;
    const double node_bytes = double(hist_node_bytes(e));
    for (uint32_t g = 0; g < G; ++g) {
      // Per row the histogram reads its codes, its float gradient pair (8
      // bytes, from which either kernel forms the exact integer values) and
      // below the root its row id.
      const double row_bytes = double(e.cols) * e.bytes_per_code + 8.0;
      for (uint32_t depth = 0; depth < D; ++depth) {
        float ms = 0;
        const size_t e = ((size_t(b) * G + g) * D + depth) * (kPhases + 1);
        XGBB_CUDA(cudaEventElapsedTime(&ms, ts.events[e], ts.events[e + 1]));
        const double rows = double(ts.host_level_rows[b][size_t(g) * kMaxDepth + depth]);
        const double nodes = double(ts.host_level_nodes[b][size_t(g) * kMaxDepth + depth]);
        if (profile_level >= 2) {
          for (uint32_t k = 0; k < kPhases; ++k) {
            float pm = 0;
            XGBB_CUDA(cudaEventElapsedTime(&pm, ts.events[e + k], ts.events[e + k + 1]));
            profile.phase_ms[k] += pm;
            profile.level_phase_ms[depth][k] += pm;
          }
        }
        if (nodes == 0) continue;
        profile.hist_ms += ms;
        profile.hist_bytes += rows * (row_bytes + (depth ? 4.0 : 0.0)) + nodes * node_bytes;
        ++profile.hist_launches;
        profile.level_ms[depth] += ms;
        profile.level_rows[depth] += rows;
        profile.level_nodes[depth] += nodes;
      }
    }
  }
  ++profile.rounds;
}

void Booster::finish_pending() {
  if (state_) finish_round(*state_);
}

void Booster::update(const std::shared_ptr<DMatrix>& d, int) {
  gpu();
  configure();
  d->upload_info(stream_);
  require(d->labels.size() == d->rows, "Labels must be provided for training.");
  if (!initialized_) initialize(*d);
  require(d->cols == num_feature_, "Number of columns does not match the trained model.");
  if (!d->quantised() || d->max_bin != max_bin_)
    d->quantise(max_bin_, nullptr, stream_, int(integer(params_, "nthread", 0)));
  TrainState& ts = train_state(d);
  run_round(ts);
}

void Booster::update_custom(const std::shared_ptr<DMatrix>& d, const float* grad, const float* hess,
                            size_t count) {
  configure();
  const uint32_t n = d->rows, G = groups_;
  require(count == size_t(n) * G, "Gradient and Hessian must have shape (n_samples, n_targets).");
  require(count == 0 || (grad != nullptr && hess != nullptr), "Null gradient or Hessian.");
  // The reference's custom_pairs (src/learner.cpp:728-740): finite values, kept
  // as given (trees accept negative Hessians).
  CustomGradients cg;
  cg.pairs.resize(count);
  cg.max_bits.assign(size_t(2) * G, 0);
  for (uint32_t r = 0; r < n; ++r)
    for (uint32_t k = 0; k < G; ++k) {
      const float g = grad[size_t(r) * G + k], h = hess[size_t(r) * G + k];
      require(std::isfinite(g) && std::isfinite(h), "Custom gradients and Hessians must be finite.");
      cg.pairs[size_t(k) * n + r] = make_float2(g, h);
      uint32_t bg, bh;
      std::memcpy(&bg, &g, 4);
      std::memcpy(&bh, &h, 4);
      cg.max_bits[2 * k] = std::max(cg.max_bits[2 * k], bg & 0x7fffffffu);
      cg.max_bits[2 * k + 1] = std::max(cg.max_bits[2 * k + 1], bh & 0x7fffffffu);
    }
  gpu();
  d->upload_info(stream_);
  if (!initialized_) initialize(*d, true);
  require(d->cols == num_feature_, "Number of columns does not match the trained model.");
  if (!d->quantised() || d->max_bin != max_bin_)
    d->quantise(max_bin_, nullptr, stream_, int(integer(params_, "nthread", 0)));
  TrainState& ts = train_state(d, true);
  run_round(ts, &cg);
}

void Booster::sync() {
  if (stream_) wait_stream("the booster's work");
  finish_pending();
}

// Waits for everything enqueued on the booster's stream, through the
// communicator's bounded wait when the stream carries collectives.
void Booster::wait_stream(const char* what) {
  if (!wait_event_) XGBB_CUDA(cudaEventCreateWithFlags(&wait_event_, cudaEventDisableTiming));
  XGBB_CUDA(cudaEventRecord(wait_event_, stream_));
  Comm::get().wait(wait_event_, what);
}

void Booster::record_event(int slot) {
  gpu();
  require(slot >= 0 && slot < 64, "event slot out of range");
  if (user_events_.size() <= size_t(slot)) user_events_.resize(size_t(slot) + 1, nullptr);
  if (!user_events_[slot]) XGBB_CUDA(cudaEventCreate(&user_events_[slot]));
  XGBB_CUDA(cudaEventRecord(user_events_[slot], stream_));
}

float Booster::elapsed_ms(int a, int b) {
  require(a >= 0 && b >= 0 && size_t(a) < user_events_.size() && size_t(b) < user_events_.size() &&
              user_events_[a] && user_events_[b], "event not recorded");
  XGBB_CUDA(cudaEventSynchronize(user_events_[b]));
  float ms = 0;
  XGBB_CUDA(cudaEventElapsedTime(&ms, user_events_[a], user_events_[b]));
  return ms;
}

std::vector<float> Booster::predict(const std::shared_ptr<DMatrix>& dp, bool output_margin,
                                    uint32_t begin, uint32_t end, bool, std::vector<uint64_t>& shape) {
  gpu();
  configure();
  finish_pending();
  DMatrix& d = *dp;
  const uint32_t G = initialized_ ? groups_ : std::max<uint32_t>(groups_, 1);
  require(!initialized_ || d.cols == num_feature_ || d.rows == 0, "Feature shape mismatch.");
  if (end == 0 || end > rounds_) end = rounds_;
  std::vector<float> out(size_t(d.rows) * G);
  // Before the first round: the margins of base_score (0.5 unless given) that
  // the first round starts from.
  std::vector<float> base = base_margin_;
  if (!initialized_) {
    const auto bs = params_.find("base_score");
    base = score_margins(std::vector<float>(G, bs != params_.end() ? std::stof(bs->second) : 0.5f));
  }
  if (d.rows) {
    DeviceBuffer dout(out.size() * 4), dbase(G * 4);
    XGBB_CUDA(cudaMemcpyAsync(dbase.get(), base.data(), G * 4, cudaMemcpyHostToDevice, stream_));
    const bool cached = state_ && state_->d == &d && begin == 0 && end == rounds_ &&
                        state_->margin_rounds == rounds_;
    if (cached) {
      XGBB_CUDA(cudaMemcpyAsync(dout.get(), state_->margins.get(), out.size() * 4,
                                cudaMemcpyDeviceToDevice, stream_));
    } else {
      std::vector<DevNode> all;
      std::vector<uint32_t> tb, tg;
      for (size_t t = size_t(begin) * G; t < size_t(end) * G && t < trees_.size(); ++t) {
        tb.push_back(uint32_t(all.size()));
        tg.push_back(trees_[t].group);
        all.insert(all.end(), trees_[t].nodes.begin(), trees_[t].nodes.end());
      }
      DeviceBuffer dn(std::max<size_t>(all.size(), 1) * sizeof(DevNode)),
          db(std::max<size_t>(tb.size(), 1) * 4), dg(std::max<size_t>(tg.size(), 1) * 4);
      if (!all.empty()) {
        XGBB_CUDA(cudaMemcpyAsync(dn.get(), all.data(), all.size() * sizeof(DevNode), cudaMemcpyHostToDevice, stream_));
        XGBB_CUDA(cudaMemcpyAsync(db.get(), tb.data(), tb.size() * 4, cudaMemcpyHostToDevice, stream_));
        XGBB_CUDA(cudaMemcpyAsync(dg.get(), tg.data(), tg.size() * 4, cudaMemcpyHostToDevice, stream_));
      }
      launch_predict(d.device_data(stream_), d.rows, d.cols, dn.as<DevNode>(), db.as<uint32_t>(),
                     dg.as<uint32_t>(), uint32_t(tb.size()), dbase.as<float>(), G, dout.as<float>(),
                     stream_);
    }
    if (!output_margin) launch_transform(objective_, dout.as<float>(), d.rows, G, stream_);
    XGBB_CUDA(cudaMemcpyAsync(out.data(), dout.get(), out.size() * 4, cudaMemcpyDeviceToHost, stream_));
    XGBB_CUDA(cudaStreamSynchronize(stream_));
  }
  if (!output_margin && objective_ == kSoftmax) {
    std::vector<float> labels(d.rows);
    for (uint32_t r = 0; r < d.rows; ++r) labels[r] = out[size_t(r) * G];
    shape = {d.rows};
    return labels;
  }
  if (G > 1) shape = {d.rows, G};
  else shape = {d.rows};
  return out;
}

// Leaf node ids of rounds [begin, end) (the reference's pred_leaf,
// src/learner.cpp:533-553): [rows][trees], or [rows][rounds][groups][1] when
// strict, [rows] for a single tree.
std::vector<float> Booster::predict_leaf(const std::shared_ptr<DMatrix>& dp, uint32_t begin, uint32_t end,
                                         bool strict, std::vector<uint64_t>& shape) {
  gpu();
  configure();
  finish_pending();
  DMatrix& d = *dp;
  require(!initialized_ || d.cols == num_feature_ || d.rows == 0, "Feature shape mismatch.");
  const uint32_t G = std::max<uint32_t>(groups_, 1);
  if (end == 0 || end > rounds_) end = rounds_;
  if (begin > end) begin = end;
  std::vector<DevNode> all;
  std::vector<uint32_t> tb;
  for (size_t t = size_t(begin) * G; t < size_t(end) * G && t < trees_.size(); ++t) {
    tb.push_back(uint32_t(all.size()));
    all.insert(all.end(), trees_[t].nodes.begin(), trees_[t].nodes.end());
  }
  const uint32_t trees = uint32_t(tb.size());
  std::vector<float> out(size_t(d.rows) * trees);
  if (d.rows && trees) {
    DeviceBuffer dn(all.size() * sizeof(DevNode)), db(tb.size() * 4), dout(out.size() * 4);
    XGBB_CUDA(cudaMemcpyAsync(dn.get(), all.data(), all.size() * sizeof(DevNode), cudaMemcpyHostToDevice, stream_));
    XGBB_CUDA(cudaMemcpyAsync(db.get(), tb.data(), tb.size() * 4, cudaMemcpyHostToDevice, stream_));
    launch_leaf_index(d.device_data(stream_), d.rows, d.cols, dn.as<DevNode>(), db.as<uint32_t>(), trees,
                      dout.as<float>(), stream_);
    XGBB_CUDA(cudaMemcpyAsync(out.data(), dout.get(), out.size() * 4, cudaMemcpyDeviceToHost, stream_));
    XGBB_CUDA(cudaStreamSynchronize(stream_));
  }
  if (strict) shape = {d.rows, end - begin, G, 1};
  else if (trees == 1) shape = {d.rows};
  else shape = {d.rows, trees};
  return out;
}

// ---------------------------------------------------------------------------
// Model files: upstream XGBoost's JSON model schema (the one the reference
// writes, src/model.cpp:28-78, and reads, src/model.cpp:79-240): per tree the
// node arrays, with leaves as split_conditions, and the learner's base score,
// objective and feature count.
// ---------------------------------------------------------------------------
namespace {
Json jnum(const std::string& text) {
  Json v;
  v.kind = Json::Number;
  v.str = text;
  v.num = std::strtod(text.c_str(), nullptr);
  return v;
}
Json jnum(int64_t x) { return jnum(std::to_string(x)); }
// The shortest decimal that reads back as the same float32.
Json jfloat(float x) {
  if (!std::isfinite(x)) x = 0.0f;
  char buf[32];
  for (int digits = 6; digits <= 9; ++digits) {
    std::snprintf(buf, sizeof buf, "%.*g", digits, double(x));
    if (std::strtof(buf, nullptr) == x) break;
  }
  return jnum(buf);
}
Json jstr(const std::string& x) {
  Json v;
  v.kind = Json::String;
  v.str = x;
  return v;
}
Json jarr() {
  Json v;
  v.kind = Json::Array;
  return v;
}
Json jobj() {
  Json v;
  v.kind = Json::Object;
  return v;
}
float jf(const Json& v) {
  if (v.kind == Json::String) return std::strtof(v.str.c_str(), nullptr);
  require(v.kind == Json::Number, "Model contains a non-numeric value.");
  return std::strtof(v.str.c_str(), nullptr);
}
int64_t ji(const Json& v) {
  if (v.kind == Json::String) return std::stoll(v.str);
  if (v.kind == Json::Bool) return v.b ? 1 : 0;
  require(v.kind == Json::Number, "Model contains a non-numeric value.");
  return int64_t(v.num);
}
const char* objective_name(int objective) {
  switch (objective) {
    case kLogistic: return "binary:logistic";
    case kLogitRaw: return "binary:logitraw";
    case kSoftprob: return "multi:softprob";
    case kSoftmax: return "multi:softmax";
    default: return "reg:squarederror";
  }
}
}  // namespace

// learner_model_param of the model file: base scores as a bracketed list,
// class and feature counts (src/model.cpp:28-60).
Json Booster::model_param_json() const {
  const uint32_t G = groups_;
  std::string bs = "[";
  const std::vector<float> scores = initialized_ ? base_score_ : std::vector<float>(G, 0.5f);
  for (size_t k = 0; k < scores.size(); ++k) {
    if (k) bs += ",";
    bs += jfloat(scores[k]).str;
  }
  bs += "]";
  const bool multi = objective_ == kSoftprob || objective_ == kSoftmax;
  Json mp = jobj();
  mp.obj.emplace_back("base_score", jstr(bs));
  mp.obj.emplace_back("boost_from_average", jstr(params_.count("base_score") ? "0" : "1"));
  mp.obj.emplace_back("num_class", jstr(multi ? std::to_string(G) : "0"));
  mp.obj.emplace_back("num_feature", jstr(std::to_string(num_feature_)));
  mp.obj.emplace_back("num_target", jstr("1"));
  return mp;
}

// The objective's name and parameters, shared by the model and the config.
Json Booster::objective_json() const {
  const bool multi = objective_ == kSoftprob || objective_ == kSoftmax;
  Json obj = jobj();
  obj.obj.emplace_back("name", jstr(objective_name(objective_)));
  if (multi) {
    Json smp = jobj();
    smp.obj.emplace_back("num_class", jstr(std::to_string(groups_)));
    obj.obj.emplace_back("softmax_multiclass_param", smp);
  } else {
    Json rlp = jobj();
    rlp.obj.emplace_back("scale_pos_weight", jstr(jfloat(spw_).str));
    obj.obj.emplace_back("reg_loss_param", rlp);
  }
  return obj;
}

std::string Booster::save_json() {
  sync();
  configure();
  const uint32_t G = groups_;
  Json trees = jarr(), info = jarr(), indptr = jarr();
  for (size_t t = 0; t < trees_.size(); ++t) {
    const HostTree& tree = trees_[t];
    Json left = jarr(), right = jarr(), parents = jarr(), idx = jarr(), cond = jarr(), dl = jarr(),
         gain = jarr(), hess = jarr(), bw = jarr(), stype = jarr();
    for (size_t i = 0; i < tree.nodes.size(); ++i) {
      const DevNode& n = tree.nodes[i];
      const bool leaf = n.left < 0;
      left.arr.push_back(jnum(leaf ? -1 : n.left));
      right.arr.push_back(jnum(leaf ? -1 : n.right));
      parents.arr.push_back(jnum(i == 0 ? 2147483647 : n.parent));
      idx.arr.push_back(jnum(leaf ? 0 : n.feature));
      cond.arr.push_back(jfloat(leaf ? n.leaf : n.threshold));
      dl.arr.push_back(jnum(leaf ? 0 : int64_t(n.default_left != 0)));
      gain.arr.push_back(jfloat(leaf ? 0.0f : n.gain));
      hess.arr.push_back(jfloat(n.cover));
      bw.arr.push_back(jfloat(n.base_weight));
      stype.arr.push_back(jnum(0));
    }
    Json tp = jobj();
    tp.obj.emplace_back("num_deleted", jstr("0"));
    tp.obj.emplace_back("num_feature", jstr(std::to_string(num_feature_)));
    tp.obj.emplace_back("num_nodes", jstr(std::to_string(tree.nodes.size())));
    tp.obj.emplace_back("size_leaf_vector", jstr("1"));
    Json tj = jobj();
    tj.obj.emplace_back("base_weights", bw);
    for (const char* empty : {"categories", "categories_nodes", "categories_segments", "categories_sizes"})
      tj.obj.emplace_back(empty, jarr());
    tj.obj.emplace_back("default_left", dl);
    tj.obj.emplace_back("id", jnum(int64_t(t)));
    tj.obj.emplace_back("left_children", left);
    tj.obj.emplace_back("loss_changes", gain);
    tj.obj.emplace_back("parents", parents);
    tj.obj.emplace_back("right_children", right);
    tj.obj.emplace_back("split_conditions", cond);
    tj.obj.emplace_back("split_indices", idx);
    tj.obj.emplace_back("split_type", stype);
    tj.obj.emplace_back("sum_hessian", hess);
    tj.obj.emplace_back("tree_param", tp);
    trees.arr.push_back(tj);
    info.arr.push_back(jnum(tree.group));
  }
  for (size_t r = 0; r <= trees_.size() / std::max<uint32_t>(G, 1); ++r) indptr.arr.push_back(jnum(int64_t(r * G)));
  Json gbp = jobj();
  gbp.obj.emplace_back("num_parallel_tree", jstr("1"));
  gbp.obj.emplace_back("num_trees", jstr(std::to_string(trees_.size())));
  Json model = jobj();
  model.obj.emplace_back("gbtree_model_param", gbp);
  model.obj.emplace_back("iteration_indptr", indptr);
  model.obj.emplace_back("tree_info", info);
  model.obj.emplace_back("trees", trees);
  Json gb = jobj();
  gb.obj.emplace_back("model", model);
  gb.obj.emplace_back("name", jstr("gbtree"));
  const Json mp = model_param_json();
  const Json obj = objective_json();
  Json attributes = jobj();
  for (auto& kv : attrs) attributes.obj.emplace_back(kv.first, jstr(kv.second));
  Json names = jarr(), types = jarr();
  if (auto it = feature_info.find("feature_name"); it != feature_info.end())
    for (auto& x : it->second) names.arr.push_back(jstr(x));
  if (auto it = feature_info.find("feature_type"); it != feature_info.end())
    for (auto& x : it->second) types.arr.push_back(jstr(x));
  Json learner = jobj();
  learner.obj.emplace_back("attributes", attributes);
  learner.obj.emplace_back("feature_names", names);
  learner.obj.emplace_back("feature_types", types);
  learner.obj.emplace_back("gradient_booster", gb);
  learner.obj.emplace_back("learner_model_param", mp);
  learner.obj.emplace_back("objective", obj);
  Json version = jarr();
  for (int v : {3, 5, 0}) version.arr.push_back(jnum(v));
  Json root = jobj();
  root.obj.emplace_back("learner", learner);
  root.obj.emplace_back("version", version);
  return root.dump();
}

void Booster::load_json(const std::string& text) {
  sync();
  const Json root = Json::parse(text);
  const Json& learner = root.at("learner");
  const Json& gb = learner.at("gradient_booster");
  require(gb.at("name").str == "gbtree", "Only gbtree models are supported: " + gb.at("name").str);
  const Json& mp = learner.at("learner_model_param");
  const std::string objective = learner.at("objective").at("name").str;
  const uint32_t nf = uint32_t(ji(mp.at("num_feature")));
  const uint32_t nc = uint32_t(ji(mp.at("num_class")));
  require(!mp.find("num_target") || ji(mp.at("num_target")) <= 1, "Multi-target models are not supported.");
  // Objective and class count decide the output groups, as in training.
  std::map<std::string, std::string> params = params_;
  params["objective"] = objective;
  if (nc > 1) params["num_class"] = std::to_string(nc);
  else params.erase("num_class");
  if (const Json* o = learner.at("objective").find("reg_loss_param"))
    if (const Json* w = o->find("scale_pos_weight")) params["scale_pos_weight"] = w->str;
  params_ = params;
  configured_ = false;
  configure();
  const uint32_t G = groups_;
  // Base score: a number, or an array written as a string.
  std::vector<float> scores;
  const Json& bsj = mp.at("base_score");
  if (bsj.kind == Json::String && !bsj.str.empty() && bsj.str[0] == '[') {
    for (const Json& v : Json::parse(bsj.str).arr) scores.push_back(jf(v));
  } else {
    scores.push_back(jf(bsj));
  }
  if (scores.size() == 1) scores.resize(G, scores[0]);
  require(scores.size() == G, "Invalid base_score shape in model.");
  const Json& model = gb.at("model");
  const Json& trees = model.at("trees");
  const Json& info = model.at("tree_info");
  require(info.arr.size() == trees.arr.size(), "Invalid tree_info length.");
  require(ji(model.at("gbtree_model_param").at("num_parallel_tree")) == 1, "num_parallel_tree > 1 is not supported.");
  require(trees.arr.size() % G == 0, "Invalid model tree count.");
  std::vector<HostTree> loaded;
  for (size_t t = 0; t < trees.arr.size(); ++t) {
    const Json& tj = trees.arr[t];
    const size_t n = size_t(ji(tj.at("tree_param").at("num_nodes")));
    require(n >= 1, "A tree must have a root node.");
    require(ji(tj.at("tree_param").at("size_leaf_vector")) <= 1, "Vector-leaf trees are not supported.");
    for (const char* f : {"left_children", "right_children", "parents", "split_indices", "split_conditions",
                          "default_left", "loss_changes", "sum_hessian"})
      require(tj.at(f).arr.size() == n, "Inconsistent node-array length in model.");
    if (const Json* st = tj.find("split_type"))
      for (const Json& v : st->arr) require(ji(v) == 0, "Categorical splits are not supported.");
    HostTree tree;
    tree.group = uint32_t(ji(info.arr[t]));
    require(tree.group < G, "Tree output group is out of range.");
    const Json* bw = tj.find("base_weights");
    tree.nodes.resize(n);
    for (size_t i = 0; i < n; ++i) {
      DevNode& d = tree.nodes[i];
      d = DevNode{};
      d.left = int32_t(ji(tj.at("left_children").arr[i]));
      d.right = int32_t(ji(tj.at("right_children").arr[i]));
      d.parent = i == 0 ? -1 : int32_t(ji(tj.at("parents").arr[i]));
      const bool leaf = d.left < 0;
      d.feature = leaf ? -1 : int32_t(ji(tj.at("split_indices").arr[i]));
      d.split_bin = -1;
      d.default_left = leaf ? 0u : uint32_t(ji(tj.at("default_left").arr[i]) != 0);
      const float c = jf(tj.at("split_conditions").arr[i]);
      d.threshold = leaf ? 0.0f : c;
      d.leaf = leaf ? c : 0.0f;
      d.cover = jf(tj.at("sum_hessian").arr[i]);
      d.gain = jf(tj.at("loss_changes").arr[i]);
      d.base_weight = bw && bw->arr.size() == n ? jf(bw->arr[i]) : d.leaf;
      d.flags = leaf ? 1u : 3u;
      if (leaf) {
        require(d.right < 0, "Invalid leaf in model.");
      } else {
        require(d.right >= 0 && size_t(d.left) < n && size_t(d.right) < n && d.left != int32_t(i) &&
                    d.right != int32_t(i) && d.feature >= 0 && uint32_t(d.feature) < nf,
                "Model contains an out-of-range tree index.");
      }
    }
    // Every node reachable once from the root, depth bounded.
    std::vector<uint8_t> seen(n, 0);
    std::vector<std::pair<int32_t, uint32_t>> stack{{0, 0}};
    while (!stack.empty()) {
      auto [id, depth] = stack.back();
      stack.pop_back();
      require(depth <= 1024 && !seen[size_t(id)], "Model contains a cyclic or excessively deep tree.");
      seen[size_t(id)] = 1;
      if (tree.nodes[size_t(id)].left >= 0) {
        stack.push_back({tree.nodes[size_t(id)].left, depth + 1});
        stack.push_back({tree.nodes[size_t(id)].right, depth + 1});
      }
    }
    loaded.push_back(std::move(tree));
  }
  // The model replaces this booster's model; its training state is dropped.
  state_.reset();
  trees_ = std::move(loaded);
  rounds_ = uint32_t(trees_.size() / G);
  num_feature_ = nf;
  base_score_ = scores;
  base_margin_ = scores;
  if (objective_ == kLogistic) {
    for (uint32_t k = 0; k < G; ++k) {
      const float v = std::min(std::max(base_score_[k], 1.0e-6f), 1.0f - 1.0e-6f);
      base_margin_[k] = -std::log(1.0f / v - 1.0f);
    }
  }
  initialized_ = true;
  attrs.clear();
  if (const Json* a = learner.find("attributes"))
    for (auto& kv : a->obj) attrs[kv.first] = kv.second.str;
  feature_info.clear();
  if (const Json* f = learner.find("feature_names"); f && !f->arr.empty())
    for (const Json& x : f->arr) feature_info["feature_name"].push_back(x.str);
  if (const Json* f = learner.find("feature_types"); f && !f->arr.empty())
    for (const Json& x : f->arr) feature_info["feature_type"].push_back(x.str);
}

// The training configuration in upstream XGBoost's layout (the reference's
// Learner::config, src/model.cpp:245-286): generic, model, train, booster,
// metric and objective sections, every value a string.
std::string Booster::config_json() {
  sync();
  configure();
  auto str = [&](const char* key, const std::string& def) { return jstr(get_param(key, def)); };
  static const std::pair<const char*, const char*> tree_defaults[] = {
      {"colsample_bylevel", "1"}, {"colsample_bynode", "1"}, {"colsample_bytree", "1"},
      {"grow_policy", "depthwise"}, {"interaction_constraints", ""}, {"learning_rate", "0.300000012"},
      {"max_bin", "256"}, {"max_cat_threshold", "64"}, {"max_cat_to_onehot", "4"},
      {"max_delta_step", "0"}, {"max_depth", "6"}, {"max_leaves", "0"}, {"min_child_weight", "1"},
      {"min_split_loss", "0"}, {"monotone_constraints", "()"}, {"refresh_leaf", "1"},
      {"reg_alpha", "0"}, {"reg_lambda", "1"}, {"sampling_method", "uniform"},
      {"sparse_threshold", "0.2"}, {"subsample", "1"}};
  std::map<std::string, Json> train;
  for (auto& kv : tree_defaults) train[kv.first] = str(kv.first, kv.second);
  train["eta"] = train["learning_rate"];
  train["lambda"] = train["reg_lambda"];
  train["alpha"] = train["reg_alpha"];
  train["gamma"] = train["min_split_loss"];
  Json ttp = jobj();
  for (auto& kv : train) ttp.obj.emplace_back(kv.first, kv.second);

  const std::string updater = "grow_gpu_hist";
  Json gtp = jobj();
  gtp.obj.emplace_back("process_type", jstr("default"));
  gtp.obj.emplace_back("tree_method", str("tree_method", "hist"));
  gtp.obj.emplace_back("updater", jstr(updater));
  gtp.obj.emplace_back("updater_seq", jstr(updater));
  Json gmp = jobj();
  gmp.obj.emplace_back("num_parallel_tree", str("num_parallel_tree", "1"));
  gmp.obj.emplace_back("num_trees", jstr(std::to_string(trees_.size())));
  Json htp = jobj();
  htp.obj.emplace_back("debug_synchronize", jstr("0"));
  htp.obj.emplace_back("max_cached_hist_node", str("max_cached_hist_node", "18446744073709551615"));
  Json up = jobj();
  up.obj.emplace_back("hist_train_param", htp);
  up.obj.emplace_back("name", jstr(updater));
  Json updaters = jarr();
  updaters.arr.push_back(up);
  Json specified;
  specified.kind = Json::Bool;
  specified.b = params_.count("updater") != 0;
  Json gb = jobj();
  gb.obj.emplace_back("gbtree_model_param", gmp);
  gb.obj.emplace_back("gbtree_train_param", gtp);
  gb.obj.emplace_back("name", jstr("gbtree"));
  gb.obj.emplace_back("specified_updater", specified);
  gb.obj.emplace_back("tree_train_param", ttp);
  gb.obj.emplace_back("updater", updaters);

  Json gp = jobj();
  gp.obj.emplace_back("device", jstr("cuda:" + std::to_string(device_)));
  gp.obj.emplace_back("n_jobs", str("nthread", "0"));
  gp.obj.emplace_back("nthread", str("nthread", "0"));
  gp.obj.emplace_back("random_state", str("seed", "0"));
  gp.obj.emplace_back("seed", str("seed", "0"));
  gp.obj.emplace_back("seed_per_iteration", str("seed_per_iteration", "0"));
  gp.obj.emplace_back("validate_parameters", jstr("1"));

  const bool multi = objective_ == kSoftprob || objective_ == kSoftmax;
  Json ltp = jobj();
  ltp.obj.emplace_back("base_score", str("base_score", "[]"));
  ltp.obj.emplace_back("boost_from_average", jstr(params_.count("base_score") ? "0" : "1"));
  ltp.obj.emplace_back("booster", jstr("gbtree"));
  ltp.obj.emplace_back("disable_default_eval_metric", str("disable_default_eval_metric", "0"));
  ltp.obj.emplace_back("multi_strategy", str("multi_strategy", "one_output_per_tree"));
  ltp.obj.emplace_back("num_class", jstr(multi ? std::to_string(groups_) : "0"));
  ltp.obj.emplace_back("num_target", jstr("1"));
  ltp.obj.emplace_back("objective", jstr(objective_name(objective_)));

  Json metrics = jarr();
  const std::string em = get_param("eval_metric", "");
  for (size_t b = 0; b < em.size();) {
    size_t e = em.find(',', b);
    if (e == std::string::npos) e = em.size();
    if (e > b) {
      Json m = jobj();
      m.obj.emplace_back("name", jstr(em.substr(b, e - b)));
      metrics.arr.push_back(m);
    }
    b = e + 1;
  }

  Json learner = jobj();
  learner.obj.emplace_back("generic_param", gp);
  learner.obj.emplace_back("gradient_booster", gb);
  learner.obj.emplace_back("learner_model_param", model_param_json());
  learner.obj.emplace_back("learner_train_param", ltp);
  learner.obj.emplace_back("metrics", metrics);
  learner.obj.emplace_back("objective", objective_json());
  Json version = jarr();
  for (int v : {3, 5, 0}) version.arr.push_back(jnum(v));
  Json root = jobj();
  root.obj.emplace_back("learner", learner);
  root.obj.emplace_back("version", version);
  return root.dump();
}

// Restores the parameters of config_json (the reference's Learner::load_config,
// src/model.cpp:287-333); the model itself is untouched.
void Booster::load_config(const std::string& text) {
  sync();
  const Json root = Json::parse(text);
  const Json& learner = root.at("learner");
  auto value = [](const Json& v) { return v.kind == Json::String ? v.str : v.dump(); };
  std::map<std::string, std::string> params = params_;
  auto put = [&](const std::string& key, const std::string& v) {
    static const std::map<std::string, std::string> alias = {
        {"eta", "learning_rate"}, {"lambda", "reg_lambda"}, {"alpha", "reg_alpha"}, {"gamma", "min_split_loss"}};
    auto it = alias.find(key);
    params[it == alias.end() ? key : it->second] = v;
  };
  const Json& objective = learner.at("objective");
  put("objective", objective.at("name").str);
  for (auto& kv : objective.obj)
    if (kv.second.kind == Json::Object)
      for (auto& p : kv.second.obj) put(p.first, value(p.second));
  if (const Json* gp = learner.find("generic_param"))
    for (auto& kv : gp->obj)
      if (kv.first != "device" && kv.first != "rng_state" && kv.first != "n_jobs" && kv.first != "random_state")
        put(kv.first, value(kv.second));
  if (const Json* gb = learner.find("gradient_booster")) {
    const std::string name = gb->find("name") ? gb->at("name").str : "gbtree";
    require(name == "gbtree", "Only the gbtree booster is implemented: " + name);
    if (const Json* t = gb->find("gbtree_train_param"))
      if (const Json* m = t->find("tree_method")) put("tree_method", value(*m));
    if (const Json* t = gb->find("tree_train_param"))
      for (auto& kv : t->obj) put(kv.first, value(kv.second));
    if (const Json* m = gb->find("gbtree_model_param"))
      if (const Json* n = m->find("num_parallel_tree")) put("num_parallel_tree", value(*n));
  }
  if (const Json* ltp = learner.find("learner_train_param"))
    for (auto& kv : ltp->obj) {
      if (kv.first == "base_score" && value(kv.second) == "[]") continue;
      // Derived flags, not parameters of this build.
      if (kv.first == "boost_from_average" || kv.first == "num_target") continue;
      if (kv.first == "num_class" && value(kv.second) == "0") {
        params.erase("num_class");
        continue;
      }
      put(kv.first, value(kv.second));
    }
  if (const Json* ms = learner.find("metrics")) {
    std::string em;
    for (const Json& m : ms->arr) {
      if (!em.empty()) em += ",";
      em += m.at("name").str;
    }
    if (em.empty()) params.erase("eval_metric");
    else params["eval_metric"] = em;
  }
  params_ = std::move(params);
  configured_ = false;
}

// A new booster holding the rounds begin, begin+step, ... < end of this one
// (end 0 = all rounds), with the same parameters and attributes except
// best_iteration and best_score (the reference's Learner::slice,
// src/model.cpp:430-459).
std::unique_ptr<Booster> Booster::slice(int begin, int end, int step) {
  sync();
  configure();
  require(step > 0 && begin >= 0, "Invalid model slice.");
  if (end == 0) end = int(rounds_);
  require(end <= int(rounds_) && begin < end, "Model slice index out of range.");
  auto out = std::make_unique<Booster>(std::vector<std::shared_ptr<DMatrix>>{});
  out->params_ = params_;
  out->configure();
  out->num_feature_ = num_feature_;
  out->max_bin_ = max_bin_;
  out->base_score_ = base_score_;
  out->base_margin_ = base_margin_;
  out->initialized_ = initialized_;
  out->attrs = attrs;
  out->attrs.erase("best_iteration");
  out->attrs.erase("best_score");
  out->feature_info = feature_info;
  const uint32_t G = groups_;
  for (int r = begin; r < end; r += step) {
    for (uint32_t g = 0; g < G; ++g) out->trees_.push_back(trees_[size_t(r) * G + g]);
    ++out->rounds_;
  }
  return out;
}

// Drops the per-matrix training state (device buffers, captured graphs); the
// model stays. Training again rebuilds it.
void Booster::reset_training() {
  sync();
  state_.reset();
}

}  // namespace xgbb
