// Shared pieces of the C ABI translation units: the thread-local results and
// error message of the upstream conventions (0 / -1, XGBGetLastError, output
// pointers valid until the next call on the same thread; the reference's
// src/c_api.cpp:16-40), handle access, and host ingestion of array
// interfaces and buffer descriptors into matrices.
#pragma once
#include <cstdint>
#include <exception>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "common.h"
#include "json.h"
#include "learner.h"
#include "xgboost/c_api.h"

namespace xgbb::capi {

struct Results {
  std::string str, str2;
  std::vector<float> floats;
  std::vector<bst_ulong> shape;
  std::vector<std::string> strings;
  std::vector<const char*> ptrs;
};
extern thread_local Results results;
extern thread_local std::string last_error;
// Booster locks taken during the current C call (booster() takes them;
// guarded() releases them when the call returns).
extern thread_local std::vector<std::unique_lock<std::recursive_mutex>> held_locks;

template <class F>
int guarded(F&& f) noexcept {
  struct Release {
    size_t n;
    ~Release() {
      while (held_locks.size() > n) held_locks.pop_back();
    }
  } release{held_locks.size()};
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    last_error = e.what();
  } catch (...) {
    last_error = "unknown error";
  }
  return -1;
}

using DMatrixPtr = std::shared_ptr<DMatrix>;
DMatrixPtr& dmat(DMatrixHandle h);
// The booster of a handle, locked until the enclosing guarded() call returns.
Booster& booster(BoosterHandle h);
void ensure_device();

// A message to the log callback of XGBRegisterLogCallback, else stderr.
void log_message(const char* text);

// Strings handed out through `results` (valid until the next call).
void string_output(std::vector<std::string> strings, bst_ulong* len, char const*** out);

// A NumPy __array_interface__ (or its JSON encoding): pointer, shape, dtype.
struct ArrayView {
  const char* ptr = nullptr;
  std::vector<uint64_t> shape;
  std::vector<int64_t> strides;  // bytes; empty = C contiguous
  char kind = 'f';               // f i u b, or B for bfloat16
  int itemsize = 4;
};
ArrayView parse_array(const std::string& text);
// One element as binary64 (exact for every supported dtype but 64-bit ints).
double read_element(const ArrayView& a, const char* p);
// A 1-D or 2-D array as float32, row-major.
std::vector<float> to_floats(const ArrayView& a, uint64_t& rows, uint64_t& cols);
// Missing sentinel -> NaN; any other infinity is an error.
void normalise(std::vector<float>& v, float missing, bool& has_missing);
// config {"missing": number | null}; NaN when absent.
float config_missing(const char* config);
// A new matrix owning `values` (normalised with `missing`).
DMatrixHandle new_dmatrix(std::vector<float>&& values, uint64_t rows, uint64_t cols, float missing);
// A matrix reading the caller's float32 C-contiguous buffer in place.
DMatrixHandle borrowed_dmatrix(const float* data, uint64_t rows, uint64_t cols);
// "label", "weight" or "base_margin".
void set_info(DMatrix& d, const std::string& field, std::vector<float> v);

// XGBufferDescriptor (include/xgboost/c_api.h): a strided 1-D or 2-D buffer
// of dtype_code 1 f32, 2 f64, 3 f16, 4 bf16, 5-8 i8..i64, 9-12 u8..u64,
// 13 bool bytes, 14 LSB-first bits; flags bit 0 = C-contiguous (strides
// ignored), bit 1 = zero copy preferred, bit 2 = strides[0] is the bit offset
// of a bit buffer; an optional per-row validity mask (mask_mode 1 LSB-first
// bits, 2 nonzero bytes = valid, 3 nonzero bytes = invalid). Rows masked
// invalid read as missing. The reference's spec_from_descriptor and
// ingest_strided_typed (src/c_api.cpp:657-690, kernels/boost.metal:256-306).
struct DescriptorView {
  const XGBufferDescriptor* d;
  uint64_t rows = 0, cols = 0;
  int64_t stride_r = 0, stride_c = 0, bit0 = 0;
  ArrayView elem;
};
DescriptorView view_descriptor(const XGBufferDescriptor* d, bool two_d);
bool descriptor_c_contiguous_f32(const DescriptorView& v);
std::vector<float> descriptor_floats(const DescriptorView& v);

// Dense row-major values from other layouts (c_api_data.cpp): CSR triplets,
// a list of column array interfaces, and CUDA array interfaces (copied to the
// host).
std::vector<float> csr_dense(const char* indptr, const char* indices, const char* data, uint64_t ncol,
                             float missing, uint64_t& rows, uint64_t& cols);
std::vector<float> columnar_dense(const char* data, uint64_t& rows, uint64_t& cols);
std::vector<float> cuda_dense_values(const char* data, uint64_t& rows, uint64_t& cols);
std::vector<float> cuda_columnar_values(const char* data, uint64_t& rows, uint64_t& cols);

}  // namespace xgbb::capi
