// Shared pieces of the C ABI: thread-local results, handle access, and host
// ingestion of array interfaces and buffer descriptors.
#include "c_api_common.h"

#include <cuda_runtime.h>

#include <cmath>
#include <cstring>

namespace xgbb::capi {

thread_local std::string last_error;
thread_local Results results;

DMatrixPtr& dmat(DMatrixHandle h) {
  require(h != nullptr, "DMatrix handle is null.");
  return *static_cast<DMatrixPtr*>(h);
}
thread_local std::vector<std::unique_lock<std::recursive_mutex>> held_locks;

xgbb::Booster& booster(BoosterHandle h) {
  require(h != nullptr, "Booster handle is null.");
  auto* b = static_cast<xgbb::Booster*>(h);
  held_locks.emplace_back(b->mutex());
  return *b;
}

void ensure_device() {
  int n = 0;
  const cudaError_t e = cudaGetDeviceCount(&n);
  require(e == cudaSuccess && n > 0, "No CUDA device is available; this library trains on CUDA GPUs only.");
}


ArrayView parse_array(const std::string& text) {
  Json j = Json::parse(text);
  if (j.kind == Json::Array) {
    require(j.arr.size() == 1, "Only one array per interface is supported.");
    j = j.arr[0];
  }
  ArrayView a;
  const Json& data = j.at("data");
  require(data.kind == Json::Array && !data.arr.empty(), "array interface 'data' must be [ptr, readonly]");
  a.ptr = reinterpret_cast<const char*>(uintptr_t(data.arr[0].as_u64()));
  for (auto& s : j.at("shape").arr) a.shape.push_back(s.as_u64());
  const std::string type = j.at("typestr").str;
  require(type.size() >= 3, "bad typestr");
  require(type[0] != '>', "Big-endian arrays are not supported.");
  a.kind = type[1];
  a.itemsize = std::stoi(type.substr(2));
  if (auto* st = j.find("strides"); st && st->kind == Json::Array)
    for (auto& s : st->arr) a.strides.push_back(s.as_i64());
  return a;
}

double read_element(const ArrayView& a, const char* p) {
  switch (a.kind) {
    case 'f':
      if (a.itemsize == 4) { float v; std::memcpy(&v, p, 4); return v; }
      if (a.itemsize == 8) { double v; std::memcpy(&v, p, 8); return v; }
      if (a.itemsize == 2) {
        uint16_t h; std::memcpy(&h, p, 2);
        const uint32_t sign = uint32_t(h & 0x8000u) << 16, e = (h >> 10) & 31, m = h & 0x3ffu;
        uint32_t out;
        if (e == 31) out = sign | 0x7f800000u | (m << 13);
        else if (e) out = sign | ((e + 112) << 23) | (m << 13);
        else if (!m) out = sign;
        else { int sh = __builtin_clz(m) - 21; out = sign | (uint32_t(113 - sh) << 23) | (((m << sh) & 0x3ffu) << 13); }
        float v; std::memcpy(&v, &out, 4); return v;
      }
      break;
    case 'i':
      if (a.itemsize == 1) return *reinterpret_cast<const int8_t*>(p);
      if (a.itemsize == 2) { int16_t v; std::memcpy(&v, p, 2); return v; }
      if (a.itemsize == 4) { int32_t v; std::memcpy(&v, p, 4); return v; }
      if (a.itemsize == 8) { int64_t v; std::memcpy(&v, p, 8); return double(v); }
      break;
    case 'u':
      if (a.itemsize == 1) return *reinterpret_cast<const uint8_t*>(p);
      if (a.itemsize == 2) { uint16_t v; std::memcpy(&v, p, 2); return v; }
      if (a.itemsize == 4) { uint32_t v; std::memcpy(&v, p, 4); return v; }
      if (a.itemsize == 8) { uint64_t v; std::memcpy(&v, p, 8); return double(v); }
      break;
    case 'b':
      return *reinterpret_cast<const uint8_t*>(p) ? 1.0 : 0.0;
    case 'B': {  // bfloat16: the upper half of a float32
      uint16_t h; std::memcpy(&h, p, 2);
      const uint32_t bits = uint32_t(h) << 16;
      float v; std::memcpy(&v, &bits, 4); return v;
    }
  }
  throw Error("Unsupported array dtype.");
}

// Copies a 1-D or 2-D array to float32, row-major.
std::vector<float> to_floats(const ArrayView& a, uint64_t& rows, uint64_t& cols) {
  rows = a.shape.empty() ? 0 : a.shape[0];
  cols = a.shape.size() > 1 ? a.shape[1] : 1;
  std::vector<float> out(size_t(rows) * cols);
  const int64_t s0 = a.strides.size() > 0 ? a.strides[0] : int64_t(cols) * a.itemsize;
  const int64_t s1 = a.strides.size() > 1 ? a.strides[1] : a.itemsize;
  if (a.kind == 'f' && a.itemsize == 4 && s1 == 4 && s0 == int64_t(cols) * 4) {
    if (!out.empty()) std::memcpy(out.data(), a.ptr, out.size() * 4);
    return out;
  }
  for (uint64_t r = 0; r < rows; ++r)
    for (uint64_t c = 0; c < cols; ++c)
      out[size_t(r) * cols + c] = float(read_element(a, a.ptr + int64_t(r) * s0 + int64_t(c) * s1));
  return out;
}

// Missing sentinel -> NaN; any other infinity is an error (src/data.cpp:433).
void normalise(std::vector<float>& v, float missing, bool& has_missing) {
  has_missing = false;
  const bool nan_missing = std::isnan(missing);
  for (float& x : v) {
    if (nan_missing ? std::isnan(x) : (x == missing)) {
      x = NAN;
      has_missing = true;
    } else if (std::isnan(x)) {
      has_missing = true;
    } else {
      require(!std::isinf(x), "Input data contains infinity or a value too large for float32.");
    }
  }
}

float config_missing(const char* config) {
  if (!config || !*config) return NAN;
  Json c = Json::parse(config);
  if (auto* m = c.find("missing"); m && m->kind == Json::Number) return float(m->num);
  return NAN;
}

DMatrixHandle new_dmatrix(std::vector<float>&& values, uint64_t rows, uint64_t cols, float missing) {
  require(rows < (1ull << 32) && cols < (1ull << 31), "Matrix exceeds the 32-bit row index range.");
  auto d = std::make_shared<xgbb::DMatrix>();
  d->rows = uint32_t(rows);
  d->cols = uint32_t(cols);
  d->owned = std::move(values);
  normalise(d->owned, missing, d->has_missing);
  d->host = d->owned.data();
  d->validated = true;
  return new DMatrixPtr(std::move(d));
}

// Zero-copy: the matrix reads the caller's float32 C-contiguous buffer, which
// must stay alive and unchanged while the matrix exists (the reference wraps
// caller memory the same way, src/runtime.mm:100-130). Validation (NaN = missing,
// no infinities) happens on the GPU when the data is first uploaded.
DMatrixHandle borrowed_dmatrix(const float* data, uint64_t rows, uint64_t cols) {
  require(rows < (1ull << 32) && cols < (1ull << 31), "Matrix exceeds the 32-bit row index range.");
  auto d = std::make_shared<xgbb::DMatrix>();
  d->rows = uint32_t(rows);
  d->cols = uint32_t(cols);
  d->host = data;
  d->validated = false;
  return new DMatrixPtr(std::move(d));
}

DescriptorView view_descriptor(const XGBufferDescriptor* d, bool two_d) {
  require(d != nullptr, "Null buffer descriptor.");
  if (two_d) require(d->ndim == 2, "Feature data must be two dimensional.");
  else require(d->ndim == 1 || d->ndim == 2, "Buffer descriptor must be 1D or 2D.");
  require(d->shape[0] <= 0xffffffffull && (d->ndim == 1 || d->shape[1] <= 0xffffffffull),
          "Matrix dimension exceeds the 32-bit row or feature index range.");
  require(d->dtype_code >= 1 && d->dtype_code <= 14, "Unsupported buffer dtype code.");
  require(d->mask_mode <= 3, "Invalid buffer mask mode.");
  static const char kinds[] = {0, 'f', 'f', 'f', 'B', 'i', 'i', 'i', 'i', 'u', 'u', 'u', 'u', 'b', 't'};
  static const int widths[] = {0, 4, 8, 2, 2, 1, 2, 4, 8, 1, 2, 4, 8, 1, 0};
  DescriptorView v{d};
  v.rows = d->shape[0];
  v.cols = d->ndim == 2 ? d->shape[1] : 1;
  v.elem.kind = kinds[d->dtype_code];
  v.elem.itemsize = widths[d->dtype_code];
  const int64_t w = v.elem.itemsize;
  if (d->dtype_code == 14) {
    require(v.cols == 1, "Bit-packed boolean buffers must be 1D or single-column.");
    v.bit0 = (d->flags & 4u) ? d->strides[0] : 0;
    require(v.bit0 >= 0, "Invalid negative bit offset.");
  } else if (d->flags & 1u) {
    v.stride_c = d->ndim == 2 ? w : 0;
    v.stride_r = d->ndim == 2 ? int64_t(v.cols) * w : w;
  } else {
    v.stride_r = d->strides[0];
    v.stride_c = d->ndim == 2 ? d->strides[1] : 0;
  }
  if (v.rows * v.cols > 0) {
    require(d->data != nullptr, "Null data pointer for a nonempty buffer.");
    if (d->mask_mode != 0) {
      require(d->mask_data != nullptr, "Null validity mask for a nonempty buffer.");
      require(d->mask_bit_offset >= 0, "Invalid negative mask offset.");
    }
  }
  return v;
}

bool descriptor_c_contiguous_f32(const DescriptorView& v) {
  return v.d->dtype_code == 1 && v.d->mask_mode == 0 &&
         (v.cols == 1 || v.stride_c == 4) && (v.rows <= 1 || v.stride_r == int64_t(v.cols) * 4);
}

std::vector<float> descriptor_floats(const DescriptorView& v) {
  std::vector<float> out(size_t(v.rows * v.cols));
  const char* base = static_cast<const char*>(v.d->data);
  const auto* mask = static_cast<const uint8_t*>(v.d->mask_data);
  const uint64_t moff = uint64_t(v.d->mask_bit_offset);
  for (uint64_t r = 0; r < v.rows; ++r) {
    bool valid = true;
    if (v.d->mask_mode == 1) valid = (mask[(r + moff) >> 3] >> ((r + moff) & 7)) & 1u;
    else if (v.d->mask_mode == 2) valid = mask[r + moff] != 0;
    else if (v.d->mask_mode == 3) valid = mask[r + moff] == 0;
    for (uint64_t c = 0; c < v.cols; ++c) {
      float x = NAN;
      if (valid) {
        if (v.elem.kind == 't') {
          const uint64_t bit = uint64_t(v.bit0) + r;
          x = float((reinterpret_cast<const uint8_t*>(base)[bit >> 3] >> (bit & 7)) & 1u);
        } else {
          x = float(read_element(v.elem, base + int64_t(r) * v.stride_r + int64_t(c) * v.stride_c));
        }
      }
      out[size_t(r * v.cols + c)] = x;
    }
  }
  return out;
}

void set_info(xgbb::DMatrix& d, const std::string& field, std::vector<float> v) {
  if (field == "label") {
    for (float x : v) require(std::isfinite(x), "Label contains NaN, infinity or a value too large.");
    d.labels = std::move(v);
  } else if (field == "weight") {
    for (float x : v) require(std::isfinite(x) && x >= 0, "Weights must be finite and nonnegative.");
    d.weights = std::move(v);
  } else if (field == "base_margin") {
    d.base_margin = std::move(v);
  } else {
    throw Error("Unknown or unsupported metadata field: " + field);
  }
  ++d.generation;
}

void string_output(std::vector<std::string> strings, bst_ulong* len, char const*** out) {
  results.strings = std::move(strings);
  results.ptrs.clear();
  for (auto& s : results.strings) results.ptrs.push_back(s.c_str());
  *len = results.ptrs.size();
  *out = results.ptrs.data();
}

}  // namespace xgbb::capi
