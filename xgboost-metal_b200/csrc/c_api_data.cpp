// DMatrix entry points beyond dense host arrays: sparse (CSR, CSC, COO) and
// columnar inputs, device arrays (CUDA array interface, DLPack), text files,
// row slices, metadata and feature names, data and quantile-cut export, and
// cross-validation folds. Every matrix is densified on the host (absent
// entries are missing), as the rest of the C ABI expects.
#include <cuda_runtime.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <numeric>
#include <random>
#include <sstream>
#include <string>
#include <vector>

#include "c_api_common.h"
#include "xgboost/c_api.h"

using namespace xgbb::capi;
using xgbb::Error;
using xgbb::Json;
using xgbb::require;

namespace {

// Integer index arrays (row pointers, indices) read exactly.
std::vector<uint64_t> to_indices(const ArrayView& a, const char* what) {
  require(a.shape.size() == 1, std::string(what) + " must be one dimensional.");
  require(a.kind == 'i' || a.kind == 'u', std::string(what) + " must have an integer dtype.");
  const uint64_t n = a.shape[0];
  const int64_t stride = a.strides.empty() ? a.itemsize : a.strides[0];
  std::vector<uint64_t> out(n);
  for (uint64_t i = 0; i < n; ++i) {
    const double v = read_element(a, a.ptr + int64_t(i) * stride);
    require(v >= 0, std::string(what) + " must be nonnegative.");
    out[i] = uint64_t(v);
  }
  return out;
}

std::vector<float> to_values(const ArrayView& a) {
  uint64_t r, c;
  require(a.shape.size() == 1, "Sparse values must be one dimensional.");
  return to_floats(a, r, c);
}

// Dense row-major values from compressed rows (csc = false) or columns.
// Entries equal to `missing` and absent entries are missing.
std::vector<float> densify_compressed(const std::vector<uint64_t>& ptr, const std::vector<uint64_t>& idx,
                                      const std::vector<float>& val, uint64_t minor_hint, bool csc,
                                      float missing, uint64_t& rows, uint64_t& cols) {
  require(!ptr.empty(), "The pointer array needs at least one entry.");
  require(idx.size() == val.size(), "Indices and values must have the same length.");
  require(ptr.front() == 0 && ptr.back() == idx.size(), "The pointer array must span the entries.");
  for (size_t i = 0; i + 1 < ptr.size(); ++i) require(ptr[i] <= ptr[i + 1], "The pointer array must be nondecreasing.");
  const uint64_t major = ptr.size() - 1;
  uint64_t minor = minor_hint;
  for (uint64_t k : idx) minor = std::max<uint64_t>(minor, k + 1);
  rows = csc ? minor : major;
  cols = csc ? major : minor;
  require(rows < (1ull << 32) && cols < (1ull << 31), "Matrix exceeds the 32-bit index range.");
  std::vector<float> dense(size_t(rows) * cols, NAN);
  const bool nan_missing = std::isnan(missing);
  for (uint64_t m = 0; m < major; ++m)
    for (uint64_t k = ptr[m]; k < ptr[m + 1]; ++k) {
      const uint64_t r = csc ? idx[k] : m, c = csc ? m : idx[k];
      const float x = val[k];
      dense[size_t(r) * cols + c] = (!nan_missing && x == missing) ? NAN : x;
    }
  return dense;
}

// A validity mask of a column (arrow bitmap '<t1' or bytes) from an
// array-interface "mask" member; empty when absent.
std::vector<uint8_t> column_validity(const Json& col, uint64_t rows) {
  const Json* m = col.find("mask");
  if (!m || m->kind != Json::Object) return {};
  const ArrayView mv = parse_array(m->dump());
  std::vector<uint8_t> valid(rows, 1);
  if (mv.kind == 't') {
    const auto* bits = reinterpret_cast<const uint8_t*>(mv.ptr);
    for (uint64_t r = 0; r < rows; ++r) valid[r] = (bits[r >> 3] >> (r & 7)) & 1u;
  } else {
    for (uint64_t r = 0; r < rows; ++r) valid[r] = read_element(mv, mv.ptr + int64_t(r) * mv.itemsize) != 0;
  }
  return valid;
}

// Columnar input: a JSON list of 1-D array interfaces, one per feature.
std::vector<float> columnar_values(const char* data, uint64_t& rows, uint64_t& cols) {
  require(data != nullptr, "Null columnar input.");
  const Json cols_json = Json::parse(data);
  require(cols_json.kind == Json::Array && !cols_json.arr.empty(), "Expected a list of column array interfaces.");
  cols = cols_json.arr.size();
  rows = 0;
  std::vector<float> out;
  for (uint64_t c = 0; c < cols; ++c) {
    const Json& col = cols_json.arr[c];
    const ArrayView a = parse_array(col.dump());
    require(a.shape.size() == 1 || (a.shape.size() == 2 && a.shape[1] == 1), "Each column must be one dimensional.");
    uint64_t r, one;
    std::vector<float> v = to_floats(a, r, one);
    if (c == 0) {
      rows = r;
      out.assign(size_t(rows) * cols, NAN);
    }
    require(r == rows, "All feature columns must have the same length.");
    const std::vector<uint8_t> valid = column_validity(col, rows);
    for (uint64_t i = 0; i < rows; ++i)
      out[size_t(i) * cols + c] = valid.empty() || valid[i] ? v[i] : NAN;
  }
  return out;
}

// A host copy of the bytes a strided device array spans; `a.ptr` is moved
// into the copy. `stream` (CUDA array interface v3) is waited for first:
// 1 = legacy default stream, 2 = per-thread default stream.
std::vector<char> copy_device_array(ArrayView& a, long long stream) {
  const int64_t item = a.itemsize;
  int64_t lo = 0, hi = item;
  uint64_t n = 1;
  for (size_t d = 0; d < a.shape.size(); ++d) n *= a.shape[d];
  std::vector<int64_t> strides = a.strides;
  if (strides.empty()) {
    strides.assign(a.shape.size(), item);
    for (size_t d = a.shape.size(); d-- > 1;) strides[d - 1] = strides[d] * int64_t(a.shape[d]);
  }
  if (n == 0) return {};
  for (size_t d = 0; d < a.shape.size(); ++d) {
    const int64_t span = int64_t(a.shape[d] - 1) * strides[d];
    if (span < 0) lo += span;
    else hi += span;
  }
  require(a.ptr != nullptr, "Null device pointer for a nonempty array.");
  if (stream == 1) XGBB_CUDA(cudaStreamSynchronize(cudaStreamLegacy));
  else if (stream == 2) XGBB_CUDA(cudaStreamSynchronize(cudaStreamPerThread));
  else if (stream > 2) XGBB_CUDA(cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)));
  else XGBB_CUDA(cudaDeviceSynchronize());
  std::vector<char> host(size_t(hi - lo));
  XGBB_CUDA(cudaMemcpy(host.data(), a.ptr + lo, host.size(), cudaMemcpyDeviceToHost));
  a.ptr = host.data() - lo;
  a.strides = strides;
  return host;
}

long long interface_stream(const std::string& text) {
  Json j = Json::parse(text);
  if (j.kind == Json::Array && !j.arr.empty()) j = j.arr[0];
  const Json* s = j.find("stream");
  return s && s->kind == Json::Number ? s->as_i64() : 0;
}

// Dense float32 values of a CUDA array interface (2-D) on the host.
std::vector<float> cuda_dense(const char* data, uint64_t& rows, uint64_t& cols) {
  require(data != nullptr, "Null CUDA array interface.");
  ensure_device();
  ArrayView a = parse_array(data);
  require(a.shape.size() == 2, "Dense input must be 2-dimensional.");
  const std::vector<char> host = copy_device_array(a, interface_stream(data));
  return to_floats(a, rows, cols);
}

// CUDA columnar input: a JSON list of 1-D CUDA array interfaces.
std::vector<float> cuda_columnar(const char* data, uint64_t& rows, uint64_t& cols) {
  require(data != nullptr, "Null CUDA columnar input.");
  ensure_device();
  const Json cols_json = Json::parse(data);
  require(cols_json.kind == Json::Array && !cols_json.arr.empty(), "Expected a list of column array interfaces.");
  cols = cols_json.arr.size();
  std::vector<float> out;
  for (uint64_t c = 0; c < cols; ++c) {
    const std::string text = cols_json.arr[c].dump();
    ArrayView a = parse_array(text);
    require(a.shape.size() == 1, "Each column must be one dimensional.");
    const std::vector<char> host = copy_device_array(a, interface_stream(text));
    uint64_t r, one;
    std::vector<float> v = to_floats(a, r, one);
    if (c == 0) {
      rows = r;
      out.assign(size_t(rows) * cols, NAN);
    }
    require(r == rows, "All feature columns must have the same length.");
    for (uint64_t i = 0; i < rows; ++i) out[size_t(i) * cols + c] = v[i];
  }
  return out;
}

}  // namespace

namespace xgbb::capi {
// Shared with the booster's in-place prediction entry points.
std::vector<float> csr_dense(const char* indptr, const char* indices, const char* data, uint64_t ncol,
                             float missing, uint64_t& rows, uint64_t& cols) {
  require(indptr && indices && data, "Null CSR input.");
  const auto ptr = to_indices(parse_array(indptr), "indptr");
  const auto idx = to_indices(parse_array(indices), "indices");
  const auto val = to_values(parse_array(data));
  return densify_compressed(ptr, idx, val, ncol, false, missing, rows, cols);
}
std::vector<float> columnar_dense(const char* data, uint64_t& rows, uint64_t& cols) {
  return columnar_values(data, rows, cols);
}
std::vector<float> cuda_dense_values(const char* data, uint64_t& rows, uint64_t& cols) {
  return cuda_dense(data, rows, cols);
}
std::vector<float> cuda_columnar_values(const char* data, uint64_t& rows, uint64_t& cols) {
  return cuda_columnar(data, rows, cols);
}
}  // namespace xgbb::capi

// ---------------------------------------------------------------------------
// Construction
// ---------------------------------------------------------------------------
// include/xgboost/c_api.h:254 (src/c_api.cpp:201-203): nrow 0 = from indices.
XGB_DLL int XGDMatrixCreateFromCSC(char const* indptr, char const* indices, char const* data, bst_ulong nrow,
                                   char const* config, DMatrixHandle* out) {
  return guarded([&] {
    require(indptr && indices && data && out, "Null CSC input.");
    const auto ptr = to_indices(parse_array(indptr), "indptr");
    const auto idx = to_indices(parse_array(indices), "indices");
    const auto val = to_values(parse_array(data));
    uint64_t rows, cols;
    auto dense = densify_compressed(ptr, idx, val, nrow, true, config_missing(config), rows, cols);
    *out = new_dmatrix(std::move(dense), rows, cols, NAN);
  });
}

// include/xgboost/c_api.h:260 (src/c_api.cpp:204-206): duplicate coordinates
// keep the last entry.
XGB_DLL int XGDMatrixCreateFromCOO(char const* row_idx, char const* col_idx, char const* data, bst_ulong nrow,
                                   bst_ulong ncol, char const* config, DMatrixHandle* out) {
  return guarded([&] {
    require(row_idx && col_idx && data && out, "Null COO input.");
    const auto ri = to_indices(parse_array(row_idx), "row indices");
    const auto ci = to_indices(parse_array(col_idx), "column indices");
    const auto val = to_values(parse_array(data));
    require(ri.size() == ci.size() && ci.size() == val.size(), "COO arrays must have the same length.");
    uint64_t rows = nrow, cols = ncol;
    for (size_t k = 0; k < ri.size(); ++k) {
      rows = std::max<uint64_t>(rows, ri[k] + 1);
      cols = std::max<uint64_t>(cols, ci[k] + 1);
    }
    require(rows < (1ull << 32) && cols < (1ull << 31), "Matrix exceeds the 32-bit index range.");
    const float missing = config_missing(config);
    std::vector<float> dense(size_t(rows) * cols, NAN);
    for (size_t k = 0; k < ri.size(); ++k)
      dense[size_t(ri[k]) * cols + ci[k]] = (!std::isnan(missing) && val[k] == missing) ? NAN : val[k];
    *out = new_dmatrix(std::move(dense), rows, cols, NAN);
  });
}

// include/xgboost/c_api.h:205 (src/c_api.cpp:195-197): a list of column
// array interfaces (optional validity masks).
XGB_DLL int XGDMatrixCreateFromColumnar(char const* data, char const* config, DMatrixHandle* out) {
  return guarded([&] {
    require(out != nullptr, "Null output handle.");
    uint64_t rows, cols;
    auto v = columnar_values(data, rows, cols);
    *out = new_dmatrix(std::move(v), rows, cols, config_missing(config));
  });
}

// include/xgboost/c_api.h:1879 (src/c_api.cpp:846-862): one descriptor per column.
XGB_DLL int XGDMatrixCreateFromColumnarBuffers(XGBufferDescriptor const* columns, bst_ulong ncol, float missing,
                                               DMatrixHandle* out) {
  return guarded([&] {
    require(columns && out && ncol > 0, "Expected at least one feature column.");
    require(ncol < (1ull << 31), "Columnar input exceeds dimension limits.");
    uint64_t rows = 0;
    std::vector<float> dense;
    for (bst_ulong c = 0; c < ncol; ++c) {
      const DescriptorView v = view_descriptor(&columns[c], false);
      require(v.cols == 1, "Each column buffer must contain one value per row.");
      if (c == 0) {
        rows = v.rows;
        dense.assign(size_t(rows) * ncol, NAN);
      }
      require(v.rows == rows, "All feature columns must have the same length.");
      const auto col = descriptor_floats(v);
      for (uint64_t r = 0; r < rows; ++r) dense[size_t(r) * ncol + c] = col[r];
    }
    *out = new_dmatrix(std::move(dense), rows, ncol, missing);
  });
}

// include/xgboost/c_api.h:285: the thread count is not needed.
XGB_DLL int XGDMatrixCreateFromMat_omp(const float* data, bst_ulong nrow, bst_ulong ncol, float missing,
                                       DMatrixHandle* out, int nthread) {
  (void)nthread;
  return XGDMatrixCreateFromMat(data, nrow, ncol, missing, out);
}

// Device arrays are copied to the host and ingested like host arrays
// (include/xgboost/c_api.h:300-314).
XGB_DLL int XGDMatrixCreateFromCudaArrayInterface(char const* data, char const* config, DMatrixHandle* out) {
  return guarded([&] {
    require(out != nullptr, "Null output handle.");
    uint64_t rows, cols;
    auto v = cuda_dense(data, rows, cols);
    *out = new_dmatrix(std::move(v), rows, cols, config_missing(config));
  });
}

XGB_DLL int XGDMatrixCreateFromCudaColumnar(char const* data, char const* config, DMatrixHandle* out) {
  return guarded([&] {
    require(out != nullptr, "Null output handle.");
    uint64_t rows, cols;
    auto v = cuda_columnar(data, rows, cols);
    *out = new_dmatrix(std::move(v), rows, cols, config_missing(config));
  });
}

namespace {
// DLPack ABI (dlpack.h v0.8 / v1.x): tensors on the host or a CUDA device.
struct DLDeviceABI {
  int32_t device_type, device_id;
};
struct DLDataTypeABI {
  uint8_t code, bits;
  uint16_t lanes;
};
struct DLTensorABI {
  void* data;
  DLDeviceABI device;
  int32_t ndim;
  DLDataTypeABI dtype;
  int64_t* shape;
  int64_t* strides;  // in elements; NULL = C-contiguous
  uint64_t byte_offset;
};
struct DLManagedTensorABI {
  DLTensorABI dl_tensor;
  void* manager_ctx;
  void (*deleter)(DLManagedTensorABI*);
};
struct DLManagedTensorVersionedABI {
  uint32_t major, minor;
  void* manager_ctx;
  void (*deleter)(DLManagedTensorVersionedABI*);
  uint64_t flags;
  DLTensorABI dl_tensor;
};
}  // namespace

// include/xgboost/c_api.h:1883 (src/c_api.cpp:872-930): a 2-D DLPack tensor on
// the host (kDLCPU, kDLCUDAHost) or a CUDA device (kDLCUDA, kDLCUDAManaged);
// the tensor's deleter runs before the call returns.
XGB_DLL int XGDMatrixCreateFromDLPack(void* dl_managed_tensor, int is_versioned, float missing,
                                      DMatrixHandle* out) {
  return guarded([&] {
    require(dl_managed_tensor && out, "Null DLPack tensor or output handle.");
    struct DeleterGuard {
      void* p;
      int versioned;
      ~DeleterGuard() {
        if (versioned) {
          auto* v = static_cast<DLManagedTensorVersionedABI*>(p);
          if (v->deleter) v->deleter(v);
        } else {
          auto* u = static_cast<DLManagedTensorABI*>(p);
          if (u->deleter) u->deleter(u);
        }
      }
    } guard{dl_managed_tensor, is_versioned};
    const DLTensorABI& t = is_versioned
                               ? static_cast<DLManagedTensorVersionedABI*>(dl_managed_tensor)->dl_tensor
                               : static_cast<DLManagedTensorABI*>(dl_managed_tensor)->dl_tensor;
    const int dev = t.device.device_type;
    require(dev == 1 || dev == 2 || dev == 3 || dev == 13,
            "DLPack tensor must reside in host memory or on a CUDA device.");
    require(t.ndim == 2 && t.shape != nullptr, "Feature data must be two dimensional.");
    require(t.shape[0] >= 0 && t.shape[1] >= 0, "Invalid DLPack shape.");
    require(t.dtype.lanes == 1, "Vector DLPack dtypes are not supported.");
    ArrayView a;
    const uint8_t code = t.dtype.code, bits = t.dtype.bits;
    a.kind = code == 0 ? 'i' : code == 1 ? 'u' : code == 2 ? 'f' : code == 4 ? 'B' : code == 6 ? 'b' : '?';
    a.itemsize = bits / 8;
    require(a.kind != '?' && bits % 8 == 0 && a.itemsize >= 1 && a.itemsize <= 8, "Unsupported DLPack dtype.");
    a.shape = {uint64_t(t.shape[0]), uint64_t(t.shape[1])};
    if (t.strides) a.strides = {t.strides[0] * a.itemsize, t.strides[1] * a.itemsize};
    a.ptr = static_cast<const char*>(t.data) + t.byte_offset;
    std::vector<char> host;
    if (dev == 2 || dev == 13) {
      ensure_device();
      host = copy_device_array(a, 0);
    } else {
      require(t.data != nullptr || a.shape[0] * a.shape[1] == 0, "Null DLPack data pointer for nonempty tensor.");
    }
    uint64_t rows, cols;
    auto v = to_floats(a, rows, cols);
    *out = new_dmatrix(std::move(v), rows, cols, missing);
  });
}

// include/xgboost/c_api.h:149 (src/c_api.cpp:364-438): "path?format=csv" (with
// "label_column=K") or "path?format=libsvm". Query ids are not supported.
XGB_DLL int XGDMatrixCreateFromURI(char const* config, DMatrixHandle* out) {
  return guarded([&] {
    require(config && out, "Null configuration or output handle.");
    const Json c = Json::parse(config);
    const std::string uri = c.at("uri").str;
    require(uri.find('#') == std::string::npos, "External memory training with text input has been removed.");
    const size_t q = uri.find('?');
    require(q != std::string::npos, "URI requires an explicit format, such as ?format=libsvm.");
    const std::string path = uri.substr(0, q), options = uri.substr(q + 1);
    std::ifstream file(path);
    require(file.good(), "Cannot open data file: " + path);
    const bool csv = options.find("format=csv") != std::string::npos;
    require(csv || options.find("format=libsvm") != std::string::npos, "Unknown data file format.");
    int label_column = -1;
    if (size_t pos = options.find("label_column="); pos != std::string::npos)
      label_column = std::stoi(options.substr(pos + 13));
    std::vector<float> labels;
    std::vector<uint64_t> ptr{0}, idx;
    std::vector<float> val;
    uint64_t cols = 0;
    std::string line;
    while (std::getline(file, line)) {
      if (!line.empty() && line.back() == '\r') line.pop_back();
      if (line.empty()) continue;
      std::istringstream input(line);
      if (csv) {
        std::string cell;
        int index = 0;
        uint64_t feature = 0;
        while (std::getline(input, cell, ',')) {
          const float x = cell.empty() ? NAN : std::stof(cell);
          if (index++ == label_column) {
            labels.push_back(x);
          } else {
            idx.push_back(feature++);
            val.push_back(x);
          }
        }
        cols = std::max(cols, feature);
      } else {
        float y;
        require(static_cast<bool>(input >> y), "Invalid libsvm label.");
        labels.push_back(y);
        std::string token;
        while (input >> token) {
          if (token[0] == '#') break;
          const size_t pos = token.find(':');
          require(pos != std::string::npos, "Invalid libsvm feature.");
          require(token.compare(0, 4, "qid:") != 0, "Ranking groups (qid) are not implemented.");
          const uint64_t f = std::stoull(token.substr(0, pos));
          idx.push_back(f);
          val.push_back(std::stof(token.substr(pos + 1)));
          cols = std::max<uint64_t>(cols, f + 1);
        }
      }
      ptr.push_back(idx.size());
    }
    uint64_t rows, ncols;
    auto dense = densify_compressed(ptr, idx, val, cols, false, NAN, rows, ncols);
    *out = new_dmatrix(std::move(dense), rows, ncols, NAN);
    if (!labels.empty()) set_info(*dmat(*out), "label", std::move(labels));
  });
}

XGB_DLL int XGDMatrixSaveBinary(DMatrixHandle handle, const char* fname, int silent) {
  (void)handle, (void)fname, (void)silent;
  return guarded([&] {
    throw Error("DMatrix binary files are not implemented by the CUDA backend; save the arrays instead.");
  });
}

// ---------------------------------------------------------------------------
// Metadata and feature names
// ---------------------------------------------------------------------------
// include/xgboost/c_api.h:849: type 1 float32, 2 float64, 3 uint32, 4 uint64.
XGB_DLL int XGDMatrixSetDenseInfo(DMatrixHandle handle, const char* field, void const* data, bst_ulong size,
                                  int type) {
  return guarded([&] {
    require(field != nullptr, "Null field name.");
    require(type >= 1 && type <= 4, "Invalid metadata type.");
    require(data != nullptr || size == 0, "Null metadata input.");
    ArrayView a;
    a.ptr = static_cast<const char*>(data);
    a.shape = {size};
    a.kind = type <= 2 ? 'f' : 'u';
    a.itemsize = type == 1 || type == 3 ? 4 : 8;
    uint64_t r, c;
    set_info(*dmat(handle), field, to_floats(a, r, c));
  });
}

// include/xgboost/c_api.h:710: integer fields ("group", "qid") are ranking
// metadata, which this build does not train on.
XGB_DLL int XGDMatrixSetUIntInfo(DMatrixHandle handle, const char* field, const unsigned* array, bst_ulong len) {
  return guarded([&] {
    require(field != nullptr, "Null field name.");
    require(array != nullptr || len == 0, "Null metadata input.");
    std::vector<float> v(array, array + len);
    set_info(*dmat(handle), field, std::move(v));
  });
}

// include/xgboost/c_api.h:892: "group_ptr" (always empty: no query groups).
XGB_DLL int XGDMatrixGetUIntInfo(const DMatrixHandle handle, const char* field, bst_ulong* out_len,
                                 const unsigned** out_dptr) {
  return guarded([&] {
    dmat(handle);
    require(field != nullptr && std::string(field) == "group_ptr", "Unknown integer metadata field.");
    *out_len = 0;
    *out_dptr = nullptr;
  });
}

namespace {
std::string interface_json(const void* ptr, std::vector<uint64_t> shape, const char* typestr) {
  std::string s = "{\"data\":[" + std::to_string(reinterpret_cast<uintptr_t>(ptr)) + ",true],\"shape\":[";
  for (size_t i = 0; i < shape.size(); ++i) s += (i ? "," : "") + std::to_string(shape[i]);
  return s + "],\"strides\":null,\"typestr\":\"" + typestr + "\",\"version\":3}";
}
}  // namespace

// include/xgboost/c_api.h:868 (src/c_api.cpp:255-268): an array interface of
// the matrix's own storage; base margins of several groups are [rows, groups].
XGB_DLL int XGDMatrixGetInfoRef(DMatrixHandle handle, char const* field, char const** out_array) {
  return guarded([&] {
    require(field != nullptr && out_array != nullptr, "Null argument.");
    auto& d = *dmat(handle);
    const std::string f = field;
    if (f == "group_ptr") {
      results.str = interface_json(nullptr, {0}, "<u4");
    } else {
      const std::vector<float>* v = f == "label" ? &d.labels : f == "weight" ? &d.weights
                                  : f == "base_margin" ? &d.base_margin : nullptr;
      require(v != nullptr, "Unknown or unsupported metadata field: " + f);
      std::vector<uint64_t> shape{v->size()};
      if (f == "base_margin" && d.rows && v->size() > d.rows && v->size() % d.rows == 0)
        shape = {d.rows, v->size() / d.rows};
      results.str = interface_json(v->empty() ? nullptr : v->data(), shape, "<f4");
    }
    *out_array = results.str.c_str();
  });
}

// include/xgboost/c_api.h:739 (src/c_api.cpp:298-306).
XGB_DLL int XGDMatrixSetStrFeatureInfo(DMatrixHandle handle, const char* field, const char** features,
                                       const bst_ulong size) {
  return guarded([&] {
    const std::string f = field ? field : "";
    require(f == "feature_name" || f == "feature_type", "Unknown feature info field.");
    auto& d = *dmat(handle);
    require(size == 0 || size == d.cols, "Feature metadata length must match the number of features.");
    std::vector<std::string> v;
    for (bst_ulong i = 0; i < size; ++i) {
      require(features && features[i], "Null feature metadata.");
      v.emplace_back(features[i]);
      if (f == "feature_type")
        require(v.back() == "q" || v.back() == "c" || v.back() == "int" || v.back() == "float" || v.back() == "i",
                "Invalid feature type.");
    }
    d.feature_info[f] = std::move(v);
  });
}

// include/xgboost/c_api.h:777
XGB_DLL int XGDMatrixGetStrFeatureInfo(DMatrixHandle handle, const char* field, bst_ulong* size,
                                       const char*** out_features) {
  return guarded([&] {
    const std::string f = field ? field : "";
    require(f == "feature_name" || f == "feature_type", "Unknown feature info field.");
    auto& fi = dmat(handle)->feature_info;
    auto it = fi.find(f);
    string_output(it == fi.end() ? std::vector<std::string>{} : it->second, size, out_features);
  });
}

// include/xgboost/c_api.h:929: rows are the only split.
XGB_DLL int XGDMatrixDataSplitMode(DMatrixHandle handle, bst_ulong* out) {
  return guarded([&] {
    dmat(handle);
    *out = 0;
  });
}

// include/xgboost/c_api.h:1897: 1 when the matrix reads the caller's buffer.
XGB_DLL int XGDMatrixWasZeroCopied(DMatrixHandle handle, int* out) {
  return guarded([&] {
    require(out != nullptr, "Null output pointer.");
    auto& d = *dmat(handle);
    *out = d.host != nullptr && d.host != d.owned.data() ? 1 : 0;
  });
}

// ---------------------------------------------------------------------------
// Export, slices, folds
// ---------------------------------------------------------------------------
// include/xgboost/c_api.h:951 (src/c_api.cpp:313-357): present entries of each
// row; out_indptr has rows + 1 entries, the others XGDMatrixNumNonMissing.
XGB_DLL int XGDMatrixGetDataAsCSR(DMatrixHandle const handle, char const* config, bst_ulong* out_indptr,
                                  unsigned* out_indices, float* out_data) {
  return guarded([&] {
    (void)config;
    auto& d = *dmat(handle);
    require(out_indptr && out_indices && out_data, "Null output array.");
    require(d.host != nullptr || d.rows == 0, "The matrix holds no host data.");
    bst_ulong count = 0;
    out_indptr[0] = 0;
    for (uint32_t r = 0; r < d.rows; ++r) {
      for (uint32_t c = 0; c < d.cols; ++c) {
        const float x = d.host[size_t(r) * d.cols + c];
        if (!std::isnan(x)) {
          out_indices[count] = c;
          out_data[count++] = x;
        }
      }
      out_indptr[r + 1] = count;
    }
  });
}

// include/xgboost/c_api.h:969 (src/c_api.cpp:358-360, src/data.cpp:1441-1449):
// per feature -inf and then its cut values, with uint64 feature offsets.
XGB_DLL int XGDMatrixGetQuantileCut(DMatrixHandle const handle, char const* config, char const** out_indptr,
                                    char const** out_data) {
  return guarded([&] {
    (void)config;
    auto& d = *dmat(handle);
    require(d.cuts != nullptr, "Quantile cuts are not available before quantization.");
    const xgbb::Cuts& c = *d.cuts;
    results.shape.assign(1, 0);
    results.floats.clear();
    for (uint32_t f = 0; f < c.cols; ++f) {
      results.floats.push_back(-INFINITY);
      const float* v = c.values.data() + size_t(f) * c.stride;
      results.floats.insert(results.floats.end(), v, v + c.counts[f]);
      results.shape.push_back(results.floats.size());
    }
    results.str = interface_json(results.shape.data(), {results.shape.size()}, "<u8");
    results.str2 = interface_json(results.floats.data(), {results.floats.size()}, "<f4");
    *out_indptr = results.str.c_str();
    *out_data = results.str2.c_str();
  });
}

namespace {
// Rows `idx` of `d` (labels, weights, margins and names follow).
DMatrixPtr slice_rows(const xgbb::DMatrix& d, const std::vector<uint64_t>& idx) {
  require(!d.quantile, "Slicing a QuantileDMatrix is not supported.");
  require(d.host != nullptr || d.rows == 0, "The matrix holds no host data.");
  std::vector<float> values(idx.size() * d.cols);
  for (size_t i = 0; i < idx.size(); ++i) {
    require(idx[i] < d.rows, "DMatrix slice index out of bounds.");
    std::copy_n(d.host + size_t(idx[i]) * d.cols, d.cols, values.data() + i * d.cols);
  }
  auto* h = static_cast<DMatrixPtr*>(new_dmatrix(std::move(values), idx.size(), d.cols, NAN));
  DMatrixPtr out = std::move(*h);
  delete h;
  auto pick = [&](const std::vector<float>& src, std::vector<float>& dst) {
    if (src.empty() || d.rows == 0) return;
    const size_t width = src.size() / d.rows;
    for (uint64_t r : idx) dst.insert(dst.end(), src.begin() + r * width, src.begin() + (r + 1) * width);
  };
  pick(d.labels, out->labels);
  pick(d.weights, out->weights);
  pick(d.base_margin, out->base_margin);
  out->feature_info = d.feature_info;
  return out;
}
}  // namespace

// include/xgboost/c_api.h:659 (src/c_api.cpp:294-297, src/data.cpp:1451+).
XGB_DLL int XGDMatrixSliceDMatrixEx(DMatrixHandle handle, const int* idxset, bst_ulong len, DMatrixHandle* out,
                                    int allow_groups) {
  return guarded([&] {
    (void)allow_groups;
    require(idxset || !len, "Null slice indices.");
    require(out != nullptr, "Null output handle.");
    std::vector<uint64_t> idx(len);
    for (bst_ulong i = 0; i < len; ++i) {
      require(idxset[i] >= 0, "DMatrix slice index out of bounds.");
      idx[i] = uint64_t(idxset[i]);
    }
    *out = new DMatrixPtr(slice_rows(*dmat(handle), idx));
  });
}

// include/xgboost/c_api.h:648
XGB_DLL int XGDMatrixSliceDMatrix(DMatrixHandle handle, const int* idxset, bst_ulong len, DMatrixHandle* out) {
  return XGDMatrixSliceDMatrixEx(handle, idxset, len, out, 0);
}

// Train/test folds for cross-validation (the reference's extension,
// src/c_api.cpp:1017-1117): rows shuffled with mt19937(seed) when asked, then
// dealt in contiguous chunks, or (stratified) sorted stably by label and dealt
// round robin.
XGB_DLL int XGDMatrixBuildCVFolds(DMatrixHandle handle, int nfold, unsigned seed, int shuffle, int stratified,
                                  DMatrixHandle* out_train, DMatrixHandle* out_test) {
  return guarded([&] {
    require(out_train && out_test, "Null CV fold output arrays.");
    require(nfold >= 2, "nfold must be at least 2.");
    const auto& d = *dmat(handle);
    const uint32_t n = d.rows;
    require(uint32_t(nfold) <= n, "Number of folds cannot exceed number of rows.");
    std::mt19937 rng(seed);
    std::vector<int> fold(n, 0);
    std::vector<uint32_t> order(n);
    std::iota(order.begin(), order.end(), 0u);
    if (shuffle) std::shuffle(order.begin(), order.end(), rng);
    if (stratified) {
      require(d.labels.size() == n, "Stratified CV requires 1D labels matching the number of rows.");
      std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) { return d.labels[a] < d.labels[b]; });
      for (uint32_t pos = 0; pos < n; ++pos) fold[order[pos]] = int(pos % uint32_t(nfold));
    } else {
      uint32_t pos = 0;
      for (int k = 0; k < nfold; ++k) {
        const uint32_t chunk = n / uint32_t(nfold) + (uint32_t(k) < n % uint32_t(nfold) ? 1u : 0u);
        for (uint32_t j = 0; j < chunk; ++j) fold[order[pos++]] = k;
      }
    }
    std::vector<DMatrixPtr> train(nfold), test(nfold);
    for (int k = 0; k < nfold; ++k) {
      std::vector<uint64_t> tr, te;
      for (uint32_t r = 0; r < n; ++r) (fold[r] == k ? te : tr).push_back(r);
      train[k] = slice_rows(d, tr);
      test[k] = slice_rows(d, te);
    }
    for (int k = 0; k < nfold; ++k) {
      out_train[k] = new DMatrixPtr(std::move(train[k]));
      out_test[k] = new DMatrixPtr(std::move(test[k]));
    }
  });
}

// ---------------------------------------------------------------------------
// Categories: this build trains numerical splits only, so a matrix or model
// never holds category dictionaries and the handle is NULL, as the reference
// returns for matrices without categories (src/c_api.cpp:157-166, 307-312).
// ---------------------------------------------------------------------------
XGB_DLL int XGDMatrixGetCategories(DMatrixHandle handle, char const* config, CategoriesHandle* out) {
  return guarded([&] {
    (void)config;
    dmat(handle);
    *out = nullptr;
  });
}

XGB_DLL int XGDMatrixGetCategoriesExportToArrow(DMatrixHandle handle, char const* config, CategoriesHandle* out,
                                                char const** export_out) {
  return guarded([&] {
    (void)config;
    dmat(handle);
    *out = nullptr;
    if (export_out) *export_out = nullptr;
  });
}

XGB_DLL int XGBoosterGetCategories(BoosterHandle handle, char const* config, CategoriesHandle* out) {
  return guarded([&] {
    (void)config;
    booster(handle);
    *out = nullptr;
  });
}

XGB_DLL int XGBoosterGetCategoriesExportToArrow(BoosterHandle handle, char const* config, CategoriesHandle* out,
                                                char const** export_out) {
  return guarded([&] {
    (void)config;
    booster(handle);
    *out = nullptr;
    if (export_out) *export_out = nullptr;
  });
}

XGB_DLL int XGBCategoriesFree(CategoriesHandle handle) {
  return guarded([&] { require(handle == nullptr, "Unknown categories handle."); });
}

// ---------------------------------------------------------------------------
// Arrow C data interface and the legacy batch iterator
// ---------------------------------------------------------------------------
namespace {
// The Arrow C data interface structs (arrow/c/abi.h).
struct ArrowSchemaABI {
  const char* format;
  const char* name;
  const char* metadata;
  int64_t flags;
  int64_t n_children;
  ArrowSchemaABI** children;
  ArrowSchemaABI* dictionary;
  void (*release)(ArrowSchemaABI*);
  void* private_data;
};
struct ArrowArrayABI {
  int64_t length;
  int64_t null_count;
  int64_t offset;
  int64_t n_buffers;
  int64_t n_children;
  const void** buffers;
  ArrowArrayABI** children;
  ArrowArrayABI* dictionary;
  void (*release)(ArrowArrayABI*);
  void* private_data;
};

// One primitive Arrow column as float32 (nulls missing), with its feature
// type (the reference's arrow_column_to_spec, src/c_api.cpp:784-840).
std::vector<float> arrow_column(const ArrowSchemaABI* cs, const ArrowArrayABI* ca, int64_t parent_offset,
                                uint64_t rows, std::string& ftype) {
  require(cs && ca && cs->format, "Invalid null Arrow column schema or array.");
  require(!cs->dictionary && !ca->dictionary, "Dictionary-encoded (categorical) Arrow columns are not supported.");
  require(ca->length >= 0 && uint64_t(ca->length) == rows, "All Arrow columns must have the same row count.");
  const std::string fmt = cs->format;
  static const std::pair<const char*, uint32_t> codes[] = {
      {"c", 5}, {"C", 9}, {"s", 6}, {"S", 10}, {"i", 7}, {"I", 11}, {"l", 8}, {"L", 12},
      {"e", 3}, {"f", 1}, {"g", 2}, {"b", 14}};
  uint32_t code = 0;
  for (auto& c : codes)
    if (fmt == c.first) code = c.second;
  require(code != 0, "Unsupported Arrow column format: " + fmt);
  ftype = code == 14 ? "i" : (code >= 1 && code <= 3) ? "float" : "int";
  if (rows == 0) return {};
  require(ca->n_buffers >= 2 && ca->buffers != nullptr, "Arrow primitive array requires at least 2 buffers.");
  const int64_t offset = parent_offset + ca->offset;
  require(offset >= 0, "Invalid negative Arrow array offset.");
  require(ca->buffers[1] != nullptr, "Null Arrow data buffer for nonempty column.");
  static const int widths[] = {0, 4, 8, 2, 2, 1, 2, 4, 8, 1, 2, 4, 8, 1, 0};
  XGBufferDescriptor d{};
  d.ndim = 1;
  d.shape[0] = rows;
  d.dtype_code = code;
  d.flags = 1;
  if (code == 14) {
    d.data = ca->buffers[1];
    d.flags = 4;
    d.strides[0] = offset;
  } else {
    d.data = static_cast<const char*>(ca->buffers[1]) + offset * widths[code];
  }
  if (ca->buffers[0] != nullptr && ca->null_count != 0) {
    d.mask_mode = 1;
    d.mask_data = ca->buffers[0];
    d.mask_bit_offset = offset;
  }
  return descriptor_floats(view_descriptor(&d, false));
}
}  // namespace

// include/xgboost/c_api.h:1885 (src/c_api.cpp:930-983): a struct (record
// batch) of primitive columns, or a single column; both structures are
// released before the call returns. Column names and types become the
// matrix's feature names and types.
XGB_DLL int XGDMatrixCreateFromArrow(void const* arrow_schema, void const* arrow_array, float missing,
                                     DMatrixHandle* out) {
  return guarded([&] {
    require(arrow_schema && arrow_array && out, "Null Arrow schema, array, or output handle.");
    auto* sch = const_cast<ArrowSchemaABI*>(static_cast<const ArrowSchemaABI*>(arrow_schema));
    auto* arr = const_cast<ArrowArrayABI*>(static_cast<const ArrowArrayABI*>(arrow_array));
    struct Guard {
      ArrowSchemaABI* s;
      ArrowArrayABI* a;
      ~Guard() {
        if (a && a->release) a->release(a);
        if (s && s->release) s->release(s);
      }
    } guard{sch, arr};
    require(sch->format != nullptr, "Released or invalid Arrow schema.");
    require(arr->length >= 0 && uint64_t(arr->length) < (1ull << 32), "Arrow array length exceeds 32-bit row limit.");
    const uint64_t rows = uint64_t(arr->length);
    std::vector<std::vector<float>> columns;
    std::vector<std::string> names, types;
    bool all_named = true;
    if (std::string(sch->format) == "+s") {
      require(sch->n_children > 0 && sch->n_children == arr->n_children && sch->children && arr->children,
              "Arrow RecordBatch/Struct must have at least one column.");
      for (int64_t c = 0; c < sch->n_children; ++c) {
        std::string t;
        columns.push_back(arrow_column(sch->children[c], arr->children[c], arr->offset, rows, t));
        types.push_back(t);
        if (sch->children[c]->name && *sch->children[c]->name) names.emplace_back(sch->children[c]->name);
        else all_named = false;
      }
    } else {
      std::string t;
      columns.push_back(arrow_column(sch, arr, 0, rows, t));
      types.push_back(t);
      if (sch->name && *sch->name) names.emplace_back(sch->name);
      else all_named = false;
    }
    const uint64_t cols = columns.size();
    std::vector<float> dense(size_t(rows) * cols);
    for (uint64_t c = 0; c < cols; ++c)
      for (uint64_t r = 0; r < rows; ++r) dense[size_t(r) * cols + c] = columns[c][r];
    DMatrixHandle h = new_dmatrix(std::move(dense), rows, cols, missing);
    auto& d = *dmat(h);
    if (all_named) d.feature_info["feature_name"] = names;
    d.feature_info["feature_type"] = types;
    *out = h;
  });
}

namespace {
// Rows appended by the legacy iterator's batches (CSR, labels, weights).
struct BatchSink {
  std::vector<uint64_t> ptr{0}, idx;
  std::vector<float> val, labels, weights;
  uint64_t cols = 0;
  bool weighted = false;
  std::string error;
};

int sink_batch(DataHolderHandle handle, XGBoostBatchCSR batch) {
  auto* sink = static_cast<BatchSink*>(handle);
  try {
    require(batch.offset != nullptr || batch.size == 0, "Null batch offsets.");
    const int64_t base = batch.size ? batch.offset[0] : 0;
    for (size_t r = 0; r < batch.size; ++r) {
      require(batch.offset[r] <= batch.offset[r + 1], "Batch offsets must be nondecreasing.");
      for (int64_t k = batch.offset[r]; k < batch.offset[r + 1]; ++k) {
        require(batch.index[k - base] >= 0, "Negative feature index.");
        sink->idx.push_back(uint64_t(batch.index[k - base]));
        sink->val.push_back(batch.value[k - base]);
        sink->cols = std::max<uint64_t>(sink->cols, uint64_t(batch.index[k - base]) + 1);
      }
      sink->ptr.push_back(sink->idx.size());
      if (batch.label) sink->labels.push_back(batch.label[r]);
      if (batch.weight) {
        sink->weighted = true;
        sink->weights.push_back(batch.weight[r]);
      }
    }
    sink->cols = std::max<uint64_t>(sink->cols, batch.columns);
    return 0;
  } catch (const std::exception& e) {
    sink->error = e.what();
    return -1;
  }
}
}  // namespace

// include/xgboost/c_api.h:431: the JVM packages' iterator, whose next()
// hands CSR batches to the set function until it returns 0.
XGB_DLL int XGDMatrixCreateFromDataIter(DataIterHandle data_handle, XGBCallbackDataIterNext* callback,
                                        const char* cache_info, float missing, DMatrixHandle* out) {
  return guarded([&] {
    (void)cache_info;
    require(callback && out, "Null iterator callback or output handle.");
    BatchSink sink;
    while (callback(data_handle, &sink_batch, &sink) != 0) require(sink.error.empty(), sink.error);
    require(sink.error.empty(), sink.error);
    uint64_t rows, cols;
    auto dense = densify_compressed(sink.ptr, sink.idx, sink.val, sink.cols, false, missing, rows, cols);
    DMatrixHandle h = new_dmatrix(std::move(dense), rows, cols, NAN);
    if (sink.labels.size() == rows && rows) set_info(*dmat(h), "label", std::move(sink.labels));
    if (sink.weighted) set_info(*dmat(h), "weight", std::move(sink.weights));
    *out = h;
  });
}
