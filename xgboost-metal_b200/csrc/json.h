// Minimal JSON reader/writer for the C ABI's configuration strings, array
// interfaces and model files.
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.h"

namespace xgbb {

struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0;
  std::string str;  // for numbers: the literal text (keeps 64-bit integers exact)
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;

  const Json* find(const std::string& key) const {
    for (auto& kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
  const Json& at(const std::string& key) const {
    auto* p = find(key);
    require(p != nullptr, "JSON key not found: " + key);
    return *p;
  }
  uint64_t as_u64() const {
    require(kind == Number, "JSON value is not a number");
    return std::stoull(str);
  }
  int64_t as_i64() const {
    require(kind == Number, "JSON value is not a number");
    return std::stoll(str);
  }
  double as_double() const {
    require(kind == Number, "JSON value is not a number");
    return num;
  }
  bool truthy() const { return kind == Bool ? b : (kind == Number ? num != 0 : false); }

  static Json parse(const std::string& text);
  std::string dump() const;
  // Universal Binary JSON (the binary model format of upstream XGBoost):
  // numeric arrays are written as typed arrays (float32 when any element is
  // fractional, else int32/int64); typed and untyped containers are read.
  std::string dump_ubj() const;
  static Json parse_ubj(const void* data, size_t size);
};

}  // namespace xgbb
