// The drop-in C ABI: the upstream XGBoost entry points of the training and
// prediction path (restated by signature in include/xgboost/c_api.h), plus the
// B200 extensions of include/xgb_b200.h. Every entry returns 0 on success and
// -1 on failure with a thread-local message for XGBGetLastError, and output
// pointers stay valid until the next call on the same thread (the reference's
// convention, src/c_api.cpp:16-40).
#include <cuda_runtime.h>

#include <cctype>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "c_api_common.h"
#include "comm.h"
#include "json.h"
#include "learner.h"
#include "metrics.h"
#include "model_dump.h"
#include "sketch.h"
#include "xgb_b200.h"
#include "xgboost/c_api.h"

using namespace xgbb::capi;

namespace {
using xgbb::Error;
using xgbb::Json;
using xgbb::require;

void (*log_callback)(const char*) = nullptr;
}  // namespace

void xgbb::capi::log_message(const char* text) {
  if (log_callback) log_callback(text);
  else std::fprintf(stderr, "%s\n", text);
}

// ---------------------------------------------------------------------------
// Library
// ---------------------------------------------------------------------------
XGB_DLL void XGBoostVersion(int* major, int* minor, int* patch) {
  if (major) *major = 3;
  if (minor) *minor = 5;
  if (patch) *patch = 0;
}

XGB_DLL const char* XGBGetLastError() { return last_error.c_str(); }

XGB_DLL int XGBRegisterLogCallback(void (*callback)(const char*)) {
  log_callback = callback;
  return 0;
}

XGB_DLL int XGBuildInfo(char const** out) {
  return guarded([&] {
    int runtime = 0;
    cudaRuntimeGetVersion(&runtime);
    results.str = std::string("{\"USE_CUDA\":true,\"USE_NCCL\":true,\"USE_OPENMP\":false,") +
                  "\"BUILTIN_PREFETCH_PRESENT\":false,\"DEBUG\":false,\"USE_FEDERATED\":false," +
                  "\"USE_RMM\":false,\"CUDA_VERSION\":[" + std::to_string(runtime / 1000) + "," +
                  std::to_string((runtime % 1000) / 10) + "],\"DEVICE\":\"B200 sm_100a\"}";
    *out = results.str.c_str();
  });
}

namespace {
// Global parameters, per thread as in the reference (src/c_api.cpp:18-29,
// 179-189): verbosity in [0, 3], use_rmm (no RMM allocator here), nthread.
struct GlobalConfig {
  int verbosity = 1;
  bool use_rmm = false;
  long long nthread = 0;
};
thread_local GlobalConfig global_config;
}  // namespace

XGB_DLL int XGBSetGlobalConfig(char const* config) {
  return guarded([&] {
    const Json c = Json::parse(config && *config ? config : "{}");
    require(c.kind == Json::Object, "The global configuration must be a JSON object.");
    GlobalConfig next = global_config;
    for (auto& kv : c.obj) {
      const std::string& key = kv.first;
      const Json& v = kv.second;
      if (key == "verbosity") {
        require(v.kind == Json::Number && v.num == std::floor(v.num) && v.num >= 0 && v.num <= 3,
                "verbosity must be in [0, 3].");
        next.verbosity = int(v.num);
      } else if (key == "use_rmm") {
        require(!v.truthy(), "RMM is not used by this build; device memory comes from cudaMalloc.");
        next.use_rmm = false;
      } else if (key == "nthread") {
        require(v.kind == Json::Number && v.num >= 0, "nthread must be a nonnegative integer.");
        next.nthread = (long long)v.num;
      } else {
        throw Error("Unknown global parameter: " + key);
      }
    }
    global_config = next;
  });
}

XGB_DLL int XGBGetGlobalConfig(char const** out) {
  return guarded([&] {
    results.str = "{\"nthread\":" + std::to_string(global_config.nthread) + ",\"use_rmm\":false,\"verbosity\":" +
                  std::to_string(global_config.verbosity) + "}";
    *out = results.str.c_str();
  });
}

// ---------------------------------------------------------------------------
// DMatrix
// ---------------------------------------------------------------------------
XGB_DLL int XGDMatrixCreateFromDense(char const* data, char const* config, DMatrixHandle* out) {
  return guarded([&] {
    ArrayView a = parse_array(data);
    require(a.shape.size() == 2, "Dense input must be 2-dimensional.");
    bool zero_copy = false;
    if (config && *config) {
      Json c = Json::parse(config);
      if (auto* z = c.find("zero_copy")) zero_copy = z->truthy();
    }
    const float missing = config_missing(config);
    const bool contiguous = a.strides.empty() ||
                            (a.strides.size() == 2 && a.strides[1] == 4 && a.strides[0] == int64_t(a.shape[1]) * 4);
    if (zero_copy && a.kind == 'f' && a.itemsize == 4 && contiguous && std::isnan(missing)) {
      *out = borrowed_dmatrix(reinterpret_cast<const float*>(a.ptr), a.shape[0], a.shape[1]);
      return;
    }
    uint64_t rows, cols;
    auto v = to_floats(a, rows, cols);
    *out = new_dmatrix(std::move(v), rows, cols, missing);
  });
}

XGB_DLL int XGDMatrixCreateFromMat(const float* data, bst_ulong nrow, bst_ulong ncol, float missing,
                                   DMatrixHandle* out) {
  return guarded([&] {
    std::vector<float> v(data, data + nrow * ncol);
    *out = new_dmatrix(std::move(v), nrow, ncol, missing);
  });
}

// CSR input is densified: an absent entry is a missing value, exactly as the
// reference's CSR histogram treats it (missing = node total - present bins).
XGB_DLL int XGDMatrixCreateFromCSR(char const* indptr, char const* indices, char const* data,
                                   bst_ulong ncol, char const* config, DMatrixHandle* out) {
  return guarded([&] {
    require(out != nullptr, "Null output handle.");
    uint64_t rows, cols;
    auto dense = csr_dense(indptr, indices, data, ncol, config_missing(config), rows, cols);
    *out = new_dmatrix(std::move(dense), rows, cols, NAN);
  });
}

XGB_DLL int XGDMatrixFree(DMatrixHandle handle) {
  return guarded([&] {
    require(handle != nullptr, "DMatrix handle is null.");
    delete static_cast<DMatrixPtr*>(handle);
  });
}

XGB_DLL int XGDMatrixSetFloatInfo(DMatrixHandle handle, const char* field, const float* array,
                                  bst_ulong len) {
  return guarded([&] { set_info(*dmat(handle), field, std::vector<float>(array, array + len)); });
}

XGB_DLL int XGDMatrixSetInfoFromInterface(DMatrixHandle handle, char const* field, char const* data) {
  return guarded([&] {
    ArrayView a = parse_array(data);
    uint64_t r, c;
    set_info(*dmat(handle), field, to_floats(a, r, c));
  });
}

XGB_DLL int XGDMatrixGetFloatInfo(const DMatrixHandle handle, const char* field, bst_ulong* out_len,
                                  const float** out_dptr) {
  return guarded([&] {
    auto& d = *dmat(handle);
    const std::string f = field;
    const std::vector<float>* v = f == "label" ? &d.labels : f == "weight" ? &d.weights
                                  : f == "base_margin" ? &d.base_margin : nullptr;
    require(v != nullptr, "Unknown metadata field: " + f);
    results.floats = *v;
    *out_len = results.floats.size();
    *out_dptr = results.floats.data();
  });
}

XGB_DLL int XGDMatrixNumRow(DMatrixHandle handle, bst_ulong* out) {
  return guarded([&] { *out = dmat(handle)->rows; });
}
XGB_DLL int XGDMatrixNumCol(DMatrixHandle handle, bst_ulong* out) {
  return guarded([&] { *out = dmat(handle)->cols; });
}
XGB_DLL int XGDMatrixNumNonMissing(DMatrixHandle handle, bst_ulong* out) {
  return guarded([&] {
    uint64_t n = 0;
    auto& d = *dmat(handle);
    for (size_t i = 0; i < size_t(d.rows) * d.cols; ++i) n += !std::isnan(d.host[i]);
    *out = n;
  });
}

XGB_DLL int XGDMatrixCreateFromBufferDescriptor(XGBufferDescriptor const* desc, float missing,
                                                DMatrixHandle* out) {
  return guarded([&] {
    require(out != nullptr, "Null output handle.");
    const DescriptorView v = view_descriptor(desc, true);
    // A float32 C-contiguous buffer offered for zero copy, with NaN as the
    // missing value, is read in place.
    if ((desc->flags & 2u) && descriptor_c_contiguous_f32(v) && std::isnan(missing)) {
      *out = borrowed_dmatrix(static_cast<const float*>(desc->data), v.rows, v.cols);
      return;
    }
    *out = new_dmatrix(descriptor_floats(v), v.rows, v.cols, missing);
  });
}

XGB_DLL int XGDMatrixSetInfoFromBufferDescriptor(DMatrixHandle handle, char const* field,
                                                 XGBufferDescriptor const* desc) {
  return guarded([&] {
    require(field != nullptr, "Null field name.");
    set_info(*dmat(handle), field, descriptor_floats(view_descriptor(desc, false)));
  });
}

// Streaming construction (the reference's from_iterator, src/c_api.cpp:140-157):
// the caller's `next` callback fills the proxy with one batch at a time through
// XGProxyDMatrixSetData* and XGDMatrixSetInfoFromInterface; the batches are
// concatenated on the host into one matrix.
XGB_DLL int XGProxyDMatrixCreate(DMatrixHandle* out) {
  return guarded([&] {
    require(out != nullptr, "Null output handle.");
    *out = new DMatrixPtr(std::make_shared<xgbb::DMatrix>());
  });
}

namespace {
// Replaces the proxy's data and keeps its labels, weights and margins.
void replace_proxy_data(DMatrixHandle proxy, DMatrixHandle fresh) {
  DMatrixPtr& slot = dmat(proxy);
  DMatrixPtr value = dmat(fresh);
  delete static_cast<DMatrixPtr*>(fresh);
  value->labels = std::move(slot->labels);
  value->weights = std::move(slot->weights);
  value->base_margin = std::move(slot->base_margin);
  value->feature_info = std::move(slot->feature_info);
  ++value->generation;
  slot = std::move(value);
}

DMatrixPtr from_iterator(DataIterHandle iter, DMatrixHandle proxy, DataIterResetCallback* reset,
                         XGDMatrixCallbackNext* next, const char* config) {
  require(reset != nullptr && next != nullptr && proxy != nullptr, "Iterator callbacks and proxy must be provided.");
  const float missing = config_missing(config);
  std::vector<float> values, labels, weights, margins;
  uint64_t rows = 0, cols = 0;
  bool first = true;
  int has_labels = -1, has_weights = -1, has_margins = -1;
  std::map<std::string, std::vector<std::string>> feature_info;
  reset(iter);
  while (true) {
    const int status = next(iter);
    require(status >= 0, "Data iterator callback failed.");
    if (!status) break;
    const xgbb::DMatrix& b = *dmat(proxy);
    require(b.host != nullptr || b.rows == 0, "A batch of the iterator has no data.");
    if (first) cols = b.cols;
    require(b.cols == cols, "Every batch must have the same number of features.");
    // Every nonempty batch carries a field or none does.
    auto append = [&](std::vector<float>& dst, int& present, const std::vector<float>& src, const char* name) {
      if (b.rows == 0) return;
      const int has = src.empty() ? 0 : 1;
      if (present < 0) present = has;
      require(present == has, std::string("Batches disagree on whether they carry ") + name + ".");
      dst.insert(dst.end(), src.begin(), src.end());
    };
    append(labels, has_labels, b.labels, "labels");
    append(weights, has_weights, b.weights, "weights");
    append(margins, has_margins, b.base_margin, "base margins");
    feature_info = b.feature_info;
    values.insert(values.end(), b.host, b.host + size_t(b.rows) * b.cols);
    rows += b.rows;
    first = false;
  }
  reset(iter);
  require(cols > 0, "The iterator produced no feature data.");
  DMatrixPtr out = dmat(new_dmatrix(std::move(values), rows, cols, missing));
  if (!labels.empty()) set_info(*out, "label", std::move(labels));
  if (!weights.empty()) set_info(*out, "weight", std::move(weights));
  if (!margins.empty()) set_info(*out, "base_margin", std::move(margins));
  out->feature_info = std::move(feature_info);
  return out;
}
}  // namespace

XGB_DLL int XGProxyDMatrixSetDataDense(DMatrixHandle handle, char const* data) {
  return guarded([&] {
    require(data != nullptr, "Null array interface.");
    ArrayView a = parse_array(data);
    require(a.shape.size() == 2, "Dense input must be 2-dimensional.");
    uint64_t rows, cols;
    auto v = to_floats(a, rows, cols);
    replace_proxy_data(handle, new_dmatrix(std::move(v), rows, cols, NAN));
  });
}

XGB_DLL int XGProxyDMatrixSetDataCSR(DMatrixHandle handle, char const* indptr, char const* indices,
                                     char const* data, bst_ulong ncol) {
  return guarded([&] {
    DMatrixHandle fresh = nullptr;
    require(XGDMatrixCreateFromCSR(indptr, indices, data, ncol, nullptr, &fresh) == 0, last_error);
    replace_proxy_data(handle, fresh);
  });
}

// include/xgboost/c_api.h:601
XGB_DLL int XGProxyDMatrixSetDataColumnar(DMatrixHandle handle, char const* data) {
  return guarded([&] {
    uint64_t rows, cols;
    auto v = columnar_dense(data, rows, cols);
    replace_proxy_data(handle, new_dmatrix(std::move(v), rows, cols, NAN));
  });
}

// include/xgboost/c_api.h:591: device batches are copied to the host.
XGB_DLL int XGProxyDMatrixSetDataCudaArrayInterface(DMatrixHandle handle, const char* data) {
  return guarded([&] {
    uint64_t rows, cols;
    auto v = cuda_dense_values(data, rows, cols);
    replace_proxy_data(handle, new_dmatrix(std::move(v), rows, cols, NAN));
  });
}

// include/xgboost/c_api.h:611
XGB_DLL int XGProxyDMatrixSetDataCudaColumnar(DMatrixHandle handle, const char* data) {
  return guarded([&] {
    uint64_t rows, cols;
    auto v = cuda_columnar_values(data, rows, cols);
    replace_proxy_data(handle, new_dmatrix(std::move(v), rows, cols, NAN));
  });
}

XGB_DLL int XGDMatrixCreateFromCallback(DataIterHandle iter, DMatrixHandle proxy, DataIterResetCallback* reset,
                                        XGDMatrixCallbackNext* next, char const* config, DMatrixHandle* out) {
  return guarded([&] {
    require(out != nullptr, "Null output handle.");
    *out = new DMatrixPtr(from_iterator(iter, proxy, reset, next, config));
  });
}

// include/xgboost/c_api.h:576: external memory is not paged here; the
// batches are concatenated in host memory as for a QuantileDMatrix.
XGB_DLL int XGExtMemQuantileDMatrixCreateFromCallback(DataIterHandle iter, DMatrixHandle proxy,
                                                      DataIterHandle ref, DataIterResetCallback* reset,
                                                      XGDMatrixCallbackNext* next, char const* config,
                                                      DMatrixHandle* out) {
  return XGQuantileDMatrixCreateFromCallback(iter, proxy, ref, reset, next, config, out);
}

// The batches are concatenated, then quantised on the GPU with `ref`'s cuts
// when `ref` (a DMatrix handle) is given (src/c_api.cpp:225-239 in the
// reference). config: {"missing", "max_bin" (default 256)}.
XGB_DLL int XGQuantileDMatrixCreateFromCallback(DataIterHandle iter, DMatrixHandle proxy, DataIterHandle ref,
                                                DataIterResetCallback* reset, XGDMatrixCallbackNext* next,
                                                char const* config, DMatrixHandle* out) {
  return guarded([&] {
    require(out != nullptr, "Null output handle.");
    uint32_t bins = 256;
    if (config && *config) {
      const Json c = Json::parse(config);
      if (const Json* m = c.find("max_bin"); m && m->kind != Json::Null) {
        require(m->kind == Json::Number && m->num == std::floor(m->num), "max_bin must be an integer.");
        require(m->num >= 2 && m->num <= 2147483647.0, "max_bin must be in [2, 2147483647].");
        bins = uint32_t(m->num);
      }
    }
    DMatrixPtr m = from_iterator(iter, proxy, reset, next, config);
    ensure_device();
    xgbb::DMatrix* r = ref ? dmat(ref).get() : nullptr;
    if (r && !r->quantised()) r->quantise(bins, nullptr, nullptr, 0);
    m->quantise(bins, r, nullptr, 0);
    m->quantile = true;
    XGBB_CUDA(cudaStreamSynchronize(nullptr));
    *out = new DMatrixPtr(std::move(m));
  });
}

// ---------------------------------------------------------------------------
// Booster
// ---------------------------------------------------------------------------
XGB_DLL int XGBoosterCreate(const DMatrixHandle dmats[], bst_ulong len, BoosterHandle* out) {
  return guarded([&] {
    std::vector<DMatrixPtr> cache;
    for (bst_ulong i = 0; i < len; ++i) cache.push_back(dmat(dmats[i]));
    *out = new xgbb::Booster(std::move(cache));
  });
}

XGB_DLL int XGBoosterFree(BoosterHandle handle) {
  return guarded([&] {
    require(handle != nullptr, "Booster handle is null.");
    auto* b = static_cast<xgbb::Booster*>(handle);
    // Wait for calls in flight on other threads, then free it unlocked.
    { std::lock_guard<std::recursive_mutex> wait(b->mutex()); }
    delete b;
  });
}

XGB_DLL int XGBoosterSetParam(BoosterHandle handle, const char* name, const char* value) {
  return guarded([&] { booster(handle).set_param(name, value ? value : ""); });
}

XGB_DLL int XGBoosterSetParams(BoosterHandle handle, char const* config) {
  return guarded([&] {
    Json c = Json::parse(config);
    for (auto& kv : c.obj)
      booster(handle).set_param(kv.first, kv.second.kind == Json::String ? kv.second.str : kv.second.dump());
  });
}

XGB_DLL int XGBoosterBoostedRounds(BoosterHandle handle, int* out) {
  return guarded([&] { *out = int(booster(handle).boosted_rounds()); });
}

XGB_DLL int XGBoosterGetNumFeature(BoosterHandle handle, bst_ulong* out) {
  return guarded([&] { *out = booster(handle).num_feature(); });
}

XGB_DLL int XGBoosterEvalOneIter(BoosterHandle handle, int iter, DMatrixHandle dmats[], const char* evnames[],
                                 bst_ulong len, const char** out_result) {
  return guarded([&] {
    std::vector<DMatrixPtr> data;
    std::vector<std::string> names;
    for (bst_ulong i = 0; i < len; ++i) {
      data.push_back(dmat(dmats[i]));
      require(evnames && evnames[i], "Null evaluation name.");
      names.emplace_back(evnames[i]);
    }
    results.str = booster(handle).evaluate(iter, data, names);
    *out_result = results.str.c_str();
  });
}

XGB_DLL int XGBoosterUpdateOneIter(BoosterHandle handle, int iter, DMatrixHandle dtrain) {
  return guarded([&] { booster(handle).update(dmat(dtrain), iter); });
}

// One round from a custom objective's gradients and Hessians: two
// __array_interface__ documents of shape (rows,) or (rows, groups), any
// numeric dtype (src/c_api.cpp:485-487 in the reference).
XGB_DLL int XGBoosterTrainOneIter(BoosterHandle handle, DMatrixHandle dtrain, int iter, char const* grad,
                                  char const* hess) {
  return guarded([&] {
    (void)iter;
    require(grad != nullptr && hess != nullptr, "Null gradient or Hessian.");
    const ArrayView ga = parse_array(grad), ha = parse_array(hess);
    require(ga.shape == ha.shape, "Gradient and Hessian must have the same shape.");
    require(ga.shape.size() == 1 || ga.shape.size() == 2, "Gradient must be one or two dimensional.");
    uint64_t gr, gc, hr, hc;
    const std::vector<float> g = to_floats(ga, gr, gc), h = to_floats(ha, hr, hc);
    auto& d = dmat(dtrain);
    require(gr == d->rows, "Gradient and Hessian must have one row per training sample.");
    booster(handle).update_custom(d, g.data(), h.data(), g.size());
  });
}

// Legacy form: flat float arrays of `len` values (src/c_api.cpp:495-497).
XGB_DLL int XGBoosterBoostOneIter(BoosterHandle handle, DMatrixHandle dtrain, float* grad, float* hess,
                                  bst_ulong len) {
  return guarded([&] {
    require(len == 0 || (grad != nullptr && hess != nullptr), "Null gradient or Hessian.");
    booster(handle).update_custom(dmat(dtrain), grad, hess, size_t(len));
  });
}

namespace {
// Prediction config: {"type": 0 value | 1 margin | 6 leaf ids, "iteration_begin",
// "iteration_end", "training", "strict_shape"} (src/c_api.cpp:507 in the
// reference).
void predict_output(xgbb::Booster& bst, const DMatrixPtr& d, const char* config, bst_ulong const** out_shape,
                    bst_ulong* out_dim, float const** out_result) {
  Json c = Json::parse(config && *config ? config : "{}");
  int type = 0;
  if (auto* t = c.find("type")) type = int(t->num);
  require(type == 0 || type == 1 || type == 6,
          "Only value (type 0), margin (type 1) and leaf (type 6) predictions are implemented.");
  uint32_t begin = 0, end = 0;
  if (auto* b = c.find("iteration_begin")) begin = uint32_t(b->num);
  if (auto* e = c.find("iteration_end")) end = uint32_t(e->num);
  bool training = false;
  if (auto* t = c.find("training")) training = t->truthy();
  bool strict = false;
  if (auto* s = c.find("strict_shape")) strict = s->truthy();
  std::vector<uint64_t> shape;
  if (type == 6) {
    results.floats = bst.predict_leaf(d, begin, end, strict, shape);
  } else {
    results.floats = bst.predict(d, type == 1, begin, end, training, shape);
    if (strict && shape.size() == 1) shape.push_back(1);
  }
  results.shape.assign(shape.begin(), shape.end());
  *out_shape = results.shape.data();
  *out_dim = results.shape.size();
  *out_result = results.floats.data();
}
}  // namespace

XGB_DLL int XGBoosterPredictFromDMatrix(BoosterHandle handle, DMatrixHandle dm, char const* config,
                                        bst_ulong const** out_shape, bst_ulong* out_dim,
                                        float const** out_result) {
  return guarded([&] { predict_output(booster(handle), dmat(dm), config, out_shape, out_dim, out_result); });
}

namespace {
// In-place prediction: a temporary matrix of `values`, with base margins from
// the proxy `m` when given (the reference's copy_proxy_metadata).
void predict_values(BoosterHandle handle, std::vector<float>&& values, uint64_t rows, uint64_t cols,
                    float missing, const char* config, DMatrixHandle m, bst_ulong const** out_shape,
                    bst_ulong* out_dim, const float** out_result) {
  auto* handle_d = static_cast<DMatrixPtr*>(new_dmatrix(std::move(values), rows, cols, missing));
  DMatrixPtr d = std::move(*handle_d);
  delete handle_d;
  if (m) d->base_margin = dmat(m)->base_margin;
  predict_output(booster(handle), d, config, out_shape, out_dim, out_result);
}
}  // namespace

// In-place prediction from a dense __array_interface__ (src/c_api.cpp:510-512
// in the reference): config adds "missing"; base margins come from the proxy
// `m` when it is given.
XGB_DLL int XGBoosterPredictFromDense(BoosterHandle handle, char const* values, char const* config,
                                      DMatrixHandle m, bst_ulong const** out_shape, bst_ulong* out_dim,
                                      const float** out_result) {
  return guarded([&] {
    require(values != nullptr, "Null array interface.");
    ArrayView a = parse_array(values);
    require(a.shape.size() == 2, "Dense input must be 2-dimensional.");
    uint64_t rows, cols;
    auto v = to_floats(a, rows, cols);
    predict_values(handle, std::move(v), rows, cols, config_missing(config), config, m, out_shape, out_dim,
                   out_result);
  });
}

// include/xgboost/c_api.h:1289 (src/c_api.cpp:516-518).
XGB_DLL int XGBoosterPredictFromCSR(BoosterHandle handle, char const* indptr, char const* indices,
                                    char const* values, bst_ulong ncol, char const* config, DMatrixHandle m,
                                    bst_ulong const** out_shape, bst_ulong* out_dim, const float** out_result) {
  return guarded([&] {
    uint64_t rows, cols;
    auto v = csr_dense(indptr, indices, values, ncol, config_missing(config), rows, cols);
    predict_values(handle, std::move(v), rows, cols, NAN, config, m, out_shape, out_dim, out_result);
  });
}

// include/xgboost/c_api.h:1261 (src/c_api.cpp:513-515).
XGB_DLL int XGBoosterPredictFromColumnar(BoosterHandle handle, char const* values, char const* config,
                                         DMatrixHandle m, bst_ulong const** out_shape, bst_ulong* out_dim,
                                         const float** out_result) {
  return guarded([&] {
    uint64_t rows, cols;
    auto v = columnar_dense(values, rows, cols);
    predict_values(handle, std::move(v), rows, cols, config_missing(config), config, m, out_shape, out_dim,
                   out_result);
  });
}

// include/xgboost/c_api.h:1313, 1337: device inputs are copied to the host.
XGB_DLL int XGBoosterPredictFromCudaArray(BoosterHandle handle, char const* values, char const* config,
                                          DMatrixHandle proxy, bst_ulong const** out_shape, bst_ulong* out_dim,
                                          const float** out_result) {
  return guarded([&] {
    uint64_t rows, cols;
    auto v = cuda_dense_values(values, rows, cols);
    predict_values(handle, std::move(v), rows, cols, config_missing(config), config, proxy, out_shape, out_dim,
                   out_result);
  });
}

XGB_DLL int XGBoosterPredictFromCudaColumnar(BoosterHandle handle, char const* data, char const* config,
                                             DMatrixHandle proxy, bst_ulong const** out_shape, bst_ulong* out_dim,
                                             const float** out_result) {
  return guarded([&] {
    uint64_t rows, cols;
    auto v = cuda_columnar_values(data, rows, cols);
    predict_values(handle, std::move(v), rows, cols, config_missing(config), config, proxy, out_shape, out_dim,
                   out_result);
  });
}

// include/xgboost/c_api.h:1887: a 2-D buffer descriptor; config as
// XGBoosterPredictFromDMatrix plus "missing".
XGB_DLL int XGBoosterPredictFromBufferDescriptor(BoosterHandle handle, XGBufferDescriptor const* desc,
                                                 char const* config, DMatrixHandle proxy,
                                                 bst_ulong const** out_shape, bst_ulong* out_dim,
                                                 float const** out_result) {
  return guarded([&] {
    const DescriptorView v = view_descriptor(desc, true);
    predict_values(handle, descriptor_floats(v), v.rows, v.cols, config_missing(config), config, proxy, out_shape,
                   out_dim, out_result);
  });
}

// include/xgboost/c_api.h:1891 (src/c_api.cpp:1000-1016): predictions of a
// matrix written into the caller's buffer of out_capacity floats.
XGB_DLL int XGBoosterPredictToBuffer(BoosterHandle handle, DMatrixHandle dm, char const* config, float* out_buffer,
                                     bst_ulong out_capacity, bst_ulong const** out_shape, bst_ulong* out_dim) {
  return guarded([&] {
    const float* values = nullptr;
    predict_output(booster(handle), dmat(dm), config, out_shape, out_dim, &values);
    bst_ulong elems = 1;
    for (bst_ulong i = 0; i < *out_dim; ++i) elems *= (*out_shape)[i];
    require(elems <= out_capacity, "Output buffer capacity (" + std::to_string(out_capacity) +
                                       ") is smaller than prediction size (" + std::to_string(elems) + ").");
    if (elems > 0) {
      require(out_buffer != nullptr, "Null output buffer for nonempty prediction.");
      std::memcpy(out_buffer, values, elems * sizeof(float));
    }
  });
}

// Split and value gradients train vector-leaf trees (multi_strategy =
// multi_output_tree), which this build does not grow.
XGB_DLL int XGBoosterTrainOneIterWithSplitGrad(BoosterHandle handle, DMatrixHandle dtrain, int iter,
                                               char const* grad, char const* hess, char const* value_grad,
                                               char const* value_hess) {
  (void)dtrain, (void)iter, (void)grad, (void)hess, (void)value_grad, (void)value_hess;
  return guarded([&] {
    booster(handle);
    throw Error("Reduced gradients need multi_strategy='multi_output_tree', which the CUDA backend does "
                "not implement.");
  });
}

// Legacy upstream predict entry (older include/xgboost/c_api.h; absent from the
// reference's header, whose predict entries are c_api.h:1207-1339): bit 0 of
// option_mask selects margins; ntree_limit counts rounds (0 = all).
XGB_DLL int XGBoosterPredict(BoosterHandle handle, DMatrixHandle dm, int option_mask,
                             unsigned ntree_limit, int training, bst_ulong* out_len,
                             const float** out_result) {
  return guarded([&] {
    std::vector<uint64_t> shape;
    results.floats = booster(handle).predict(dmat(dm), (option_mask & 1) != 0, 0, ntree_limit,
                                             training != 0, shape);
    *out_len = results.floats.size();
    *out_result = results.floats.data();
  });
}

XGB_DLL int XGBoosterSetAttr(BoosterHandle handle, const char* key, const char* value) {
  return guarded([&] {
    auto& b = booster(handle);
    if (value) b.attrs[key] = value;
    else b.attrs.erase(key);
  });
}

XGB_DLL int XGBoosterGetAttr(BoosterHandle handle, const char* key, const char** out, int* success) {
  return guarded([&] {
    auto& b = booster(handle);
    auto it = b.attrs.find(key);
    *success = it != b.attrs.end();
    if (*success) {
      results.str = it->second;
      *out = results.str.c_str();
    } else {
      *out = nullptr;
    }
  });
}

XGB_DLL int XGBoosterGetAttrNames(BoosterHandle handle, bst_ulong* out_len, const char*** out) {
  return guarded([&] {
    auto& b = booster(handle);
    results.strings.clear();
    for (auto& kv : b.attrs) results.strings.push_back(kv.first);
    results.ptrs.clear();
    for (auto& s : results.strings) results.ptrs.push_back(s.c_str());
    *out_len = results.ptrs.size();
    *out = results.ptrs.data();
  });
}

XGB_DLL int XGBoosterSetStrFeatureInfo(BoosterHandle handle, const char* field,
                                       const char** features, const bst_ulong size) {
  return guarded([&] {
    const std::string f = field ? field : "";
    require(f == "feature_name" || f == "feature_type", "Unknown feature info field: " + f);
    std::vector<std::string> v;
    for (bst_ulong i = 0; i < size; ++i) {
      require(features && features[i], "Null feature metadata.");
      v.emplace_back(features[i]);
      if (f == "feature_type")
        require(v.back() == "q" || v.back() == "c" || v.back() == "int" || v.back() == "float" || v.back() == "i",
                "Invalid feature type: " + v.back());
    }
    auto& b = booster(handle);
    // A model that knows its width checks the list against it
    // (src/c_api.cpp:119-128 in the reference).
    require(v.empty() || b.num_feature() == 0 || v.size() == b.num_feature(),
            "Feature metadata length must match the number of features.");
    b.feature_info[f] = std::move(v);
  });
}

XGB_DLL int XGBoosterGetStrFeatureInfo(BoosterHandle handle, const char* field, bst_ulong* len,
                                       const char*** out_features) {
  return guarded([&] {
    auto& fi = booster(handle).feature_info;
    auto it = fi.find(field);
    results.strings = it == fi.end() ? std::vector<std::string>{} : it->second;
    results.ptrs.clear();
    for (auto& s : results.strings) results.ptrs.push_back(s.c_str());
    *len = results.ptrs.size();
    *out_features = results.ptrs.data();
  });
}

// Model files (src/c_api.cpp:521-538 in the reference): JSON text, or
// Universal Binary JSON, the same document in binary form.
namespace {
std::string model_bytes(xgbb::Booster& b, const std::string& format) {
  xgbb::require(format == "json" || format == "ubj", "Model format must be 'json' or 'ubj': " + format);
  std::string text = b.save_json();
  return format == "json" ? text : xgbb::Json::parse(text).dump_ubj();
}
void load_model_bytes(xgbb::Booster& b, const void* data, size_t size) {
  const char* p = static_cast<const char*>(data);
  size_t i = 0;
  while (i < size && std::isspace(static_cast<unsigned char>(p[i]))) ++i;
  xgbb::require(i < size, "The model buffer is empty.");
  // Both open with '{': JSON text continues with a quote, blank or '}', a
  // UBJSON object with the marker of its first key's length.
  const char next = i + 1 < size ? p[i + 1] : '}';
  const bool text = p[i] == '{' && (next == '"' || next == '}' || std::isspace(static_cast<unsigned char>(next)));
  if (text) b.load_json(std::string(p, size));
  else b.load_json(xgbb::Json::parse_ubj(p, size).dump());
}
}  // namespace

XGB_DLL int XGBoosterSaveModel(BoosterHandle handle, const char* fname) {
  return guarded([&] {
    const std::string path = fname ? fname : "";
    const bool json = path.size() >= 5 && path.compare(path.size() - 5, 5, ".json") == 0;
    const std::string bytes = model_bytes(booster(handle), json ? "json" : "ubj");
    std::FILE* f = std::fopen(path.c_str(), "wb");
    xgbb::require(f != nullptr, "Cannot write model: " + path);
    const size_t wrote = std::fwrite(bytes.data(), 1, bytes.size(), f);
    const bool closed = std::fclose(f) == 0;
    xgbb::require(wrote == bytes.size() && closed, "Failed to write model: " + path);
  });
}

XGB_DLL int XGBoosterLoadModel(BoosterHandle handle, const char* fname) {
  return guarded([&] {
    const std::string path = fname ? fname : "";
    std::FILE* f = std::fopen(path.c_str(), "rb");
    xgbb::require(f != nullptr, "Cannot read model file: " + path);
    std::string bytes;
    char buf[1 << 16];
    size_t n;
    while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) bytes.append(buf, n);
    std::fclose(f);
    load_model_bytes(booster(handle), bytes.data(), bytes.size());
  });
}

XGB_DLL int XGBoosterSaveModelToBuffer(BoosterHandle handle, char const* config, bst_ulong* out_len,
                                       char const** out_dptr) {
  return guarded([&] {
    std::string format = "ubj";
    if (config && *config) {
      Json c = Json::parse(config);
      if (auto* f = c.find("format")) format = f->str;
    }
    results.str = model_bytes(booster(handle), format);
    *out_len = results.str.size();
    *out_dptr = results.str.data();
  });
}

XGB_DLL int XGBoosterLoadModelFromBuffer(BoosterHandle handle, const void* buf, bst_ulong len) {
  return guarded([&] { load_model_bytes(booster(handle), buf, size_t(len)); });
}

XGB_DLL int XGBoosterSaveJsonConfig(BoosterHandle handle, bst_ulong* out_len, char const** out_str) {
  return guarded([&] {
    results.str = booster(handle).config_json();
    *out_len = results.str.size();
    *out_str = results.str.c_str();
  });
}

XGB_DLL int XGBoosterLoadJsonConfig(BoosterHandle handle, char const* config) {
  return guarded([&] {
    require(config != nullptr, "Null configuration.");
    booster(handle).load_config(config);
  });
}

// The whole booster for pickling: {"Config": ..., "Model": ...} as UBJSON
// (src/c_api.cpp:541-546 in the reference).
XGB_DLL int XGBoosterSerializeToBuffer(BoosterHandle handle, bst_ulong* out_len, char const** out_dptr) {
  return guarded([&] {
    auto& b = booster(handle);
    Json state;
    state.kind = Json::Object;
    state.obj.emplace_back("Config", Json::parse(b.config_json()));
    state.obj.emplace_back("Model", Json::parse(b.save_json()));
    results.str = state.dump_ubj();
    *out_len = results.str.size();
    *out_dptr = results.str.data();
  });
}

XGB_DLL int XGBoosterUnserializeFromBuffer(BoosterHandle handle, const void* buf, bst_ulong len) {
  return guarded([&] {
    require(buf != nullptr || len == 0, "Null buffer.");
    const Json state = Json::parse_ubj(buf, size_t(len));
    auto& b = booster(handle);
    b.load_json(state.at("Model").dump());
    b.load_config(state.at("Config").dump());
  });
}

XGB_DLL int XGBoosterReset(BoosterHandle handle) {
  return guarded([&] { booster(handle).reset_training(); });
}

// -2 marks an out-of-range layer index (src/c_api.cpp:503-506 in the reference).
XGB_DLL int XGBoosterSlice(BoosterHandle handle, int begin_layer, int end_layer, int step,
                           BoosterHandle* out) {
  const int status = guarded([&] {
    require(out != nullptr, "Null output handle.");
    *out = booster(handle).slice(begin_layer, end_layer, step).release();
  });
  return status != 0 && last_error.find("out of range") != std::string::npos ? -2 : status;
}

namespace {
std::vector<std::string> feature_field(xgbb::Booster& b, const char* field) {
  auto it = b.feature_info.find(field);
  return it == b.feature_info.end() ? std::vector<std::string>{} : it->second;
}

std::vector<std::string> checked_features(const char** values, bst_ulong len, uint32_t cols, bool types) {
  require(len == 0 || cols == 0 || len == cols, "Feature metadata length must match the number of features.");
  std::vector<std::string> out;
  for (bst_ulong i = 0; i < len; ++i) {
    require(values && values[i], "Null feature metadata.");
    std::string v = values[i];
    if (types)
      require(v == "q" || v == "c" || v == "int" || v == "float" || v == "i", "Invalid feature type: " + v);
    out.push_back(std::move(v));
  }
  return out;
}
}  // namespace

XGB_DLL int XGBoosterDumpModelEx(BoosterHandle handle, const char* fmap, int with_stats, const char* format,
                                 bst_ulong* out_len, const char*** out_dump_array) {
  return guarded([&] {
    require(!fmap || !*fmap, "Feature-map files have not been implemented yet.");
    auto& b = booster(handle);
    const auto& trees = b.trees();
    string_output(xgbb::dump_trees(trees, feature_field(b, "feature_name"), feature_field(b, "feature_type"),
                                   format ? format : "text", with_stats != 0),
                  out_len, out_dump_array);
  });
}

XGB_DLL int XGBoosterDumpModel(BoosterHandle handle, const char* fmap, int with_stats, bst_ulong* out_len,
                               const char*** out_dump_array) {
  return XGBoosterDumpModelEx(handle, fmap, with_stats, "text", out_len, out_dump_array);
}

XGB_DLL int XGBoosterDumpModelExWithFeatures(BoosterHandle handle, int fnum, const char** fname,
                                             const char** ftype, int with_stats, const char* format,
                                             bst_ulong* out_len, const char*** out_models) {
  return guarded([&] {
    auto& b = booster(handle);
    require(fnum >= 0, "Negative feature count.");
    const auto& trees = b.trees();
    const auto names = checked_features(fname, bst_ulong(fnum), b.num_feature(), false);
    const auto types = checked_features(ftype, bst_ulong(fnum), b.num_feature(), true);
    string_output(xgbb::dump_trees(trees, names, types, format ? format : "text", with_stats != 0), out_len,
                  out_models);
  });
}

XGB_DLL int XGBoosterDumpModelWithFeatures(BoosterHandle handle, int fnum, const char** fname,
                                           const char** ftype, int with_stats, bst_ulong* out_len,
                                           const char*** out_models) {
  return XGBoosterDumpModelExWithFeatures(handle, fnum, fname, ftype, with_stats, "text", out_len, out_models);
}

// config: {"importance_type": "weight" | "gain" | "cover" | "total_gain" |
// "total_cover", "feature_names": [...] or null}. Only features used by a split
// are listed; scores have shape [n_features].
XGB_DLL int XGBoosterFeatureScore(BoosterHandle handle, const char* config, bst_ulong* out_n_features,
                                  char const*** out_features, bst_ulong* out_dim,
                                  bst_ulong const** out_shape, float const** out_scores) {
  return guarded([&] {
    auto& b = booster(handle);
    const Json c = Json::parse(config && *config ? config : "{}");
    std::string kind = "weight";
    if (const Json* k = c.find("importance_type"); k && k->kind == Json::String) kind = k->str;
    std::vector<std::string> names = feature_field(b, "feature_name");
    if (const Json* f = c.find("feature_names"); f && f->kind == Json::Array) {
      names.clear();
      for (const Json& x : f->arr) names.push_back(x.str);
    }
    const auto& trees = b.trees();
    xgbb::FeatureScores s = xgbb::feature_scores(trees, b.num_feature(), names, kind);
    results.floats = std::move(s.scores);
    string_output(std::move(s.names), out_n_features, out_features);
    results.shape.assign(1, *out_n_features);
    *out_dim = 1;
    *out_shape = results.shape.data();
    *out_scores = results.floats.data();
  });
}

// ---------------------------------------------------------------------------
// Collective (row-sharded training over NCCL)
// ---------------------------------------------------------------------------
XGB_DLL int XGCommunicatorInit(char const* config) {
  return guarded([&] {
    Json c = Json::parse(config && *config ? config : "{}");
    int rank = 0, world = 1, device = 0;
    if (auto* r = c.find("rank")) rank = int(r->num);
    if (auto* w = c.find("world_size")) world = int(w->num);
    if (auto* d = c.find("device")) device = int(d->num);
    std::string id;
    if (auto* i = c.find("nccl_unique_id")) id = i->str;
    // Seconds a collective may wait for the other ranks before the
    // communicator is aborted and the waiting call fails.
    if (auto* t = c.find("timeout")) xgbb::Comm::get().set_timeout(t->num);
    xgbb::Comm::get().init(rank, world, id, device);
  });
}

XGB_DLL int XGCommunicatorFinalize(void) {
  return guarded([&] { xgbb::Comm::get().finalize(); });
}

XGB_DLL int XGCommunicatorGetRank(void) { return xgbb::Comm::get().rank(); }
XGB_DLL int XGCommunicatorGetWorldSize(void) { return xgbb::Comm::get().world(); }

// ---------------------------------------------------------------------------
// B200 extensions (include/xgb_b200.h)
// ---------------------------------------------------------------------------
XGB_DLL int XGBBNcclUniqueId(char const** out) {
  return guarded([&] {
    results.str = xgbb::nccl_unique_id_hex();
    *out = results.str.c_str();
  });
}

XGB_DLL int XGBBSetDevice(int device) {
  return guarded([&] { XGBB_CUDA(cudaSetDevice(device)); });
}

XGB_DLL int XGBBSynchronize(void) {
  return guarded([&] { xgbb::Comm::get().wait_device("device synchronisation"); });
}

XGB_DLL int XGDMatrixQuantise(DMatrixHandle handle, int max_bin, DMatrixHandle ref) {
  return guarded([&] {
    xgbb::Trace trace("XGDMatrixQuantise");
    ensure_device();
    trace.mark("device", nullptr);
    auto& d = *dmat(handle);
    const xgbb::DMatrix* r = ref ? dmat(ref).get() : nullptr;
    d.quantise(uint32_t(max_bin), r, nullptr, 0);
    d.quantile = true;
    XGBB_CUDA(cudaStreamSynchronize(nullptr));
    trace.mark("quantise", nullptr);
  });
}

XGB_DLL int XGBoosterGetCudaProfile(BoosterHandle handle, char const** out) {
  return guarded([&] {
    booster(handle).finish_pending();  // the last round's profile figures
    auto& p = booster(handle).profile;
    results.str = "{\"hist_ms\":" + std::to_string(p.hist_ms) +
                  ",\"hist_bytes\":" + std::to_string(p.hist_bytes) +
                  ",\"hist_launches\":" + std::to_string(p.hist_launches) +
                  ",\"rounds\":" + std::to_string(p.rounds) + ",\"csr\":" + (p.csr ? "true" : "false") +
                  ",\"levels\":[";
    for (uint32_t d = 0; d < xgbb::kMaxDepth; ++d) {
      if (d) results.str += ",";
      results.str += "[" + std::to_string(p.level_ms[d]) + "," + std::to_string(p.level_rows[d]) + "," +
                     std::to_string(p.level_nodes[d]) + "]";
    }
    // cuda_profile=2: milliseconds per phase, in total and per level.
    static const char* const kNames[xgbb::kPhases] = {"hist", "reduce_scatter", "eval", "best_gather",
                                                      "partition", "counts"};
    results.str += "],\"phases\":{";
    for (uint32_t k = 0; k < xgbb::kPhases; ++k)
      results.str += std::string(k ? "," : "") + "\"" + kNames[k] + "\":" + std::to_string(p.phase_ms[k]);
    results.str += "},\"level_phases\":[";
    for (uint32_t d = 0; d < xgbb::kMaxDepth; ++d) {
      results.str += d ? ",[" : "[";
      for (uint32_t k = 0; k < xgbb::kPhases; ++k)
        results.str += std::string(k ? "," : "") + std::to_string(p.level_phase_ms[d][k]);
      results.str += "]";
    }
    results.str += "]}";
    *out = results.str.c_str();
  });
}

XGB_DLL int XGBoosterRecordEvent(BoosterHandle handle, int slot) {
  return guarded([&] { booster(handle).record_event(slot); });
}

XGB_DLL int XGBoosterEventElapsed(BoosterHandle handle, int a, int b, float* ms) {
  return guarded([&] { *ms = booster(handle).elapsed_ms(a, b); });
}

XGB_DLL int XGBoosterCaptureLevelHistograms(BoosterHandle handle, int depth) {
  return guarded([&] {
    auto& b = booster(handle);
    xgbb::require(depth >= -1 && depth < int(xgbb::kMaxDepth), "capture depth out of range");
    b.capture = xgbb::Booster::LevelCapture{};
    b.capture.depth = depth;
  });
}

XGB_DLL int XGBoosterGetLevelHistograms(BoosterHandle handle, char const** meta, int64_t const** hist,
                                        uint32_t const** node_ids) {
  return guarded([&] {
    auto& b = booster(handle);
    b.sync();
    const auto& c = b.capture;
    xgbb::require(c.ready, "no level histograms were captured (request one, then train a round)");
    results.str = "{\"depth\":" + std::to_string(c.depth) + ",\"pairs\":" + std::to_string(c.pairs) +
                  ",\"f_lo\":" + std::to_string(c.f_lo) + ",\"f_hi\":" + std::to_string(c.f_hi) +
                  ",\"bins1\":" + std::to_string(c.bins1) + "}";
    *meta = results.str.c_str();
    *hist = reinterpret_cast<const int64_t*>(c.hist.data());
    *node_ids = c.node_ids.data();
  });
}

XGB_DLL int XGBoosterResetCudaProfile(BoosterHandle handle) {
  return guarded([&] {
    booster(handle).finish_pending();  // a pending round belongs to the counts being cleared
    booster(handle).profile = xgbb::Profile{};
  });
}

// Test entry: product cuts (host sketch) and GPU bins, decoded to row-major
// uint32 with 0xffffffff for missing. cuts must hold cols * min(max_bin, rows).
XGB_DLL int XGBBQuantizeHost(const float* X, bst_ulong rows, bst_ulong cols, uint32_t max_bin,
                             float* cuts, uint32_t* counts, float* minima, uint32_t* bins) {
  return guarded([&] {
    ensure_device();
    auto h = new_dmatrix(std::vector<float>(X, X + rows * cols), rows, cols, NAN);
    std::unique_ptr<DMatrixPtr> owner(static_cast<DMatrixPtr*>(h));
    auto& d = **owner;
    d.quantise(max_bin, nullptr, nullptr, 0);
    XGBB_CUDA(cudaDeviceSynchronize());
    const auto& c = *d.cuts;
    std::memcpy(cuts, c.values.data(), c.values.size() * 4);
    std::memcpy(counts, c.counts.data(), c.counts.size() * 4);
    std::memcpy(minima, c.minima.data(), c.minima.size() * 4);
    const size_t n = size_t(rows) * d.ell.stride;
    std::vector<uint8_t> raw(n * d.ell.bytes_per_code);
    if (n) XGBB_CUDA(cudaMemcpy(raw.data(), d.codes.get(), raw.size(), cudaMemcpyDeviceToHost));
    for (uint64_t r = 0; r < rows; ++r)
      for (uint64_t f = 0; f < cols; ++f) {
        const size_t i = size_t(r) * d.ell.stride + f;
        const uint32_t code = d.ell.bytes_per_code == 1 ? raw[i] : reinterpret_cast<uint16_t*>(raw.data())[i];
        bins[size_t(r) * cols + f] = code == d.ell.missing ? 0xffffffffu : code;
      }
  });
}

// Test entries: an evaluation metric over host predictions, its per-row
// (loss, weight) sums, and the metric from sums gathered over workers (no
// device needed).
XGB_DLL int XGBBMetricHost(char const* name, const float* pred, bst_ulong rows, uint32_t groups,
                           const float* labels, const float* weights, int multiclass, double* out) {
  return guarded([&] {
    require(name != nullptr && out != nullptr, "Null argument.");
    require(rows == 0 || (pred != nullptr && labels != nullptr), "Null predictions or labels.");
    require(rows < (1ull << 32) && groups >= 1, "Invalid shape.");
    *out = xgbb::eval_metric(name, pred, uint32_t(rows), groups, labels, weights, multiclass != 0);
  });
}

XGB_DLL int XGBBMetricSumsHost(char const* name, const float* pred, bst_ulong rows, uint32_t groups,
                               const float* labels, const float* weights, int multiclass, double* sums) {
  return guarded([&] {
    require(name != nullptr && sums != nullptr, "Null argument.");
    require(rows == 0 || (pred != nullptr && labels != nullptr), "Null predictions or labels.");
    require(rows < (1ull << 32) && groups >= 1, "Invalid shape.");
    require(!xgbb::metric_needs_all_rows(name), std::string(name) + " is not a sum over rows.");
    xgbb::metric_sums(name, pred, uint32_t(rows), groups, labels, weights, multiclass != 0, &sums[0], &sums[1]);
  });
}

XGB_DLL int XGBBMetricFromSums(char const* name, double loss_sum, double weight_sum, double* out) {
  return guarded([&] {
    require(name != nullptr && out != nullptr, "Null argument.");
    require(!xgbb::metric_needs_all_rows(name), std::string(name) + " is not a sum over rows.");
    *out = xgbb::metric_from_sums(name, loss_sum, weight_sum);
  });
}

// Test entry: the quantile sketch on the GPU (sketch_gpu.cu) over a host
// matrix copied in; cuts [cols][min(max_bin, rows)], counts and minima as
// XGBBSketchHost returns them.
XGB_DLL int XGBBSketchDevice(const float* X, bst_ulong rows, bst_ulong cols, const float* weights,
                             uint32_t max_bin, float* cuts, uint32_t* counts, float* minima) {
  return guarded([&] {
    ensure_device();
    require(rows < (1ull << 32) && cols < (1ull << 32), "Matrix too large.");
    require(max_bin >= 2, "max_bin must be at least 2.");
    require(rows == 0 || cols == 0 || X != nullptr, "Null matrix.");
    xgbb::DeviceBuffer dx(std::max<size_t>(size_t(rows) * cols * 4, 4)), dw;
    if (rows && cols) XGBB_CUDA(cudaMemcpy(dx.get(), X, size_t(rows) * cols * 4, cudaMemcpyHostToDevice));
    if (weights) {
      dw.resize(std::max<size_t>(size_t(rows) * 4, 4));
      if (rows) XGBB_CUDA(cudaMemcpy(dw.get(), weights, size_t(rows) * 4, cudaMemcpyHostToDevice));
    }
    cudaStream_t s;
    XGBB_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    try {
      xgbb::sketch_cuts_device(dx.as<float>(), uint32_t(rows), uint32_t(cols), weights ? dw.as<float>() : nullptr,
                               max_bin, cuts, counts, minima, s);
    } catch (...) {
      cudaStreamSynchronize(s);
      cudaStreamDestroy(s);
      throw;
    }
    cudaStreamDestroy(s);
  });
}

// Measurement entry: SM cycles per warp-level shared instruction of a probe
// variant (probe.cu), for sizing the histogram kernels' limb scheme.
XGB_DLL int XGBBProbeSharedPipe(int variant, uint32_t warps, uint32_t iters, double* cycles) {
  return guarded([&] {
    ensure_device();
    xgbb::require(cycles != nullptr, "Null output.");
    *cycles = xgbb::probe_shared_pipe(variant, warps, iters);
  });
}

// Test entry: the host quantile sketch on its own (no device needed).
XGB_DLL int XGBBSketchHost(const float* X, bst_ulong rows, bst_ulong cols, const float* weights,
                           uint32_t max_bin, int threads, float* cuts, uint32_t* counts, float* minima) {
  return guarded([&] {
    xgbb::require(rows < (1ull << 32) && cols < (1ull << 32), "matrix too large");
    xgbb::require(max_bin >= 2 && max_bin <= xgbb::kMaxBins, "max_bin must be in [2, 256]");
    xgbb::sketch_cuts(X, uint32_t(rows), uint32_t(cols), weights, max_bin, cuts, counts, minima, threads);
  });
}

// Test entry: gradient pairs [groups][rows] and scales [groups][2] for margins
// [rows][groups] through the product's gradient and exact-scale kernels.
XGB_DLL int XGBBGradientsHost(int objective, const float* margins, const float* labels,
                              const float* weights, bst_ulong rows, uint32_t groups,
                              float scale_pos_weight, float* pairs, float* scales) {
  return guarded([&] {
    ensure_device();
    xgbb::DeviceBuffer dm(std::max<size_t>(rows * groups, 1) * 4), dl(std::max<size_t>(rows, 1) * 4),
        dw(weights ? rows * 4 : 0), dp(std::max<size_t>(rows * groups, 1) * 8),
        mass(xgbb::mass_bytes(groups)), ds(groups * 8);
    XGBB_CUDA(cudaMemcpy(dm.get(), margins, rows * groups * 4, cudaMemcpyHostToDevice));
    XGBB_CUDA(cudaMemcpy(dl.get(), labels, rows * 4, cudaMemcpyHostToDevice));
    if (weights) XGBB_CUDA(cudaMemcpy(dw.get(), weights, rows * 4, cudaMemcpyHostToDevice));
    XGBB_CUDA(cudaMemset(mass.get(), 0, mass.size()));
    const xgbb::MassAccum m = xgbb::mass_view(mass.get(), groups);
    auto* p = dp.as<float2>();
    xgbb::launch_gradients(objective, dm.as<float>(), dl.as<float>(), weights ? dw.as<float>() : nullptr,
                           uint32_t(rows), groups, scale_pos_weight, p, m, nullptr);
    xgbb::launch_mass_window(p, uint32_t(rows), groups, m, nullptr);
    xgbb::launch_scales(p, uint32_t(rows), groups, m, ds.as<float2>(), rows, true, nullptr);
    xgbb::launch_mass_exact(p, uint32_t(rows), groups, m, nullptr);
    xgbb::launch_scales_exact(groups, m, ds.as<float2>(), nullptr);
    XGBB_CUDA(cudaDeviceSynchronize());
    XGBB_CUDA(cudaMemcpy(pairs, dp.get(), rows * groups * 8, cudaMemcpyDeviceToHost));
    XGBB_CUDA(cudaMemcpy(scales, ds.get(), groups * 8, cudaMemcpyDeviceToHost));
  });
}

// Device-pointer variant of XGBBGradientsHost that allocates nothing: the
// scale accumulators live in a fixed device array (at most 64 groups) and
// everything is enqueued on `stream` without waiting for it.
XGB_DLL int XGBBGradientsDeviceNoAlloc(int objective, const float* margins, const float* labels,
                                       const float* weights, bst_ulong rows, uint32_t groups,
                                       float scale_pos_weight, float* pairs, float* scales,
                                       void* stream) {
  return guarded([&] {
    xgbb::gradients_no_alloc(objective, margins, labels, weights, rows, groups, scale_pos_weight,
                             reinterpret_cast<float2*>(pairs), reinterpret_cast<float2*>(scales),
                             static_cast<cudaStream_t>(stream));
  });
}

// Test entry: a whole training run through DMatrix + Booster, with the trees
// written back to back as DevNode records (48 bytes each).
XGB_DLL int XGBBTrainHost(const float* X, bst_ulong rows, bst_ulong cols, const float* labels,
                          const float* weights, char const* params_json, uint32_t rounds,
                          void* nodes, bst_ulong node_capacity, uint32_t* tree_sizes,
                          float* margins) {
  return guarded([&] {
    ensure_device();
    auto h = new_dmatrix(std::vector<float>(X, X + rows * cols), rows, cols, NAN);
    std::unique_ptr<DMatrixPtr> owner(static_cast<DMatrixPtr*>(h));
    DMatrixPtr d = *owner;
    set_info(*d, "label", std::vector<float>(labels, labels + rows));
    if (weights) set_info(*d, "weight", std::vector<float>(weights, weights + rows));
    xgbb::Booster b({d});
    Json p = Json::parse(params_json && *params_json ? params_json : "{}");
    for (auto& kv : p.obj) b.set_param(kv.first, kv.second.kind == Json::String ? kv.second.str : kv.second.dump());
    for (uint32_t r = 0; r < rounds; ++r) b.update(d, int(r));
    const auto& trees = b.trees();
    size_t used = 0;
    for (size_t t = 0; t < trees.size(); ++t) {
      require(used + trees[t].nodes.size() <= node_capacity, "node buffer too small");
      std::memcpy(static_cast<xgbb::DevNode*>(nodes) + used, trees[t].nodes.data(),
                  trees[t].nodes.size() * sizeof(xgbb::DevNode));
      tree_sizes[t] = uint32_t(trees[t].nodes.size());
      used += trees[t].nodes.size();
    }
    std::vector<uint64_t> shape;
    auto m = b.predict(d, true, 0, 0, true, shape);
    std::memcpy(margins, m.data(), m.size() * 4);
  });
}
