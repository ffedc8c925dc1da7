#include "json.h"

#include <cctype>
#include <climits>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>

namespace xgbb {
namespace {

struct Parser {
  const std::string& s;
  size_t i = 0;
  explicit Parser(const std::string& t) : s(t) {}

  void ws() {
    while (i < s.size() && std::isspace(static_cast<unsigned char>(s[i]))) ++i;
  }
  char peek() {
    ws();
    require(i < s.size(), "unexpected end of JSON");
    return s[i];
  }
  void expect(char c) {
    require(peek() == c, std::string("JSON: expected '") + c + "'");
    ++i;
  }
  std::string string_lit() {
    expect('"');
    std::string out;
    while (true) {
      require(i < s.size(), "unterminated JSON string");
      char c = s[i++];
      if (c == '"') break;
      if (c == '\\') {
        require(i < s.size(), "bad JSON escape");
        char e = s[i++];
        switch (e) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            require(i + 4 <= s.size(), "bad JSON unicode escape");
            unsigned code = std::strtoul(s.substr(i, 4).c_str(), nullptr, 16);
            i += 4;
            if (code < 0x80) out += char(code);
            else if (code < 0x800) {
              out += char(0xc0 | (code >> 6));
              out += char(0x80 | (code & 0x3f));
            } else {
              out += char(0xe0 | (code >> 12));
              out += char(0x80 | ((code >> 6) & 0x3f));
              out += char(0x80 | (code & 0x3f));
            }
            break;
          }
          default: out += e;
        }
      } else {
        out += c;
      }
    }
    return out;
  }
  Json value() {
    Json v;
    char c = peek();
    if (c == '{') {
      ++i;
      v.kind = Json::Object;
      if (peek() == '}') {
        ++i;
        return v;
      }
      while (true) {
        std::string k = string_lit();
        expect(':');
        v.obj.emplace_back(k, value());
        if (peek() == ',') {
          ++i;
          continue;
        }
        expect('}');
        break;
      }
    } else if (c == '[') {
      ++i;
      v.kind = Json::Array;
      if (peek() == ']') {
        ++i;
        return v;
      }
      while (true) {
        v.arr.push_back(value());
        if (peek() == ',') {
          ++i;
          continue;
        }
        expect(']');
        break;
      }
    } else if (c == '"') {
      v.kind = Json::String;
      v.str = string_lit();
    } else if (s.compare(i, 4, "true") == 0) {
      i += 4;
      v.kind = Json::Bool;
      v.b = true;
    } else if (s.compare(i, 5, "false") == 0) {
      i += 5;
      v.kind = Json::Bool;
    } else if (s.compare(i, 4, "null") == 0) {
      i += 4;
    } else {
      size_t j = i;
      while (j < s.size() && (std::isdigit(static_cast<unsigned char>(s[j])) || s[j] == '-' ||
                              s[j] == '+' || s[j] == '.' || s[j] == 'e' || s[j] == 'E' ||
                              s[j] == 'I' || s[j] == 'n' || s[j] == 'f' || s[j] == 'i' ||
                              s[j] == 't' || s[j] == 'y' || s[j] == 'N' || s[j] == 'a'))
        ++j;
      require(j > i, "bad JSON value");
      v.kind = Json::Number;
      v.str = s.substr(i, j - i);
      v.num = std::strtod(v.str.c_str(), nullptr);
      i = j;
    }
    return v;
  }
};

void dump_string(const std::string& s, std::string& out) {
  out += '"';
  for (char c : s) {
    if (c == '"' || c == '\\') {
      out += '\\';
      out += c;
    } else if (c == '\n') {
      out += "\\n";
    } else {
      out += c;
    }
  }
  out += '"';
}

void dump_value(const Json& v, std::string& out) {
  switch (v.kind) {
    case Json::Null: out += "null"; break;
    case Json::Bool: out += v.b ? "true" : "false"; break;
    case Json::Number: out += v.str.empty() ? std::to_string(v.num) : v.str; break;
    case Json::String: dump_string(v.str, out); break;
    case Json::Array:
      out += '[';
      for (size_t k = 0; k < v.arr.size(); ++k) {
        if (k) out += ',';
        dump_value(v.arr[k], out);
      }
      out += ']';
      break;
    case Json::Object:
      out += '{';
      for (size_t k = 0; k < v.obj.size(); ++k) {
        if (k) out += ',';
        dump_string(v.obj[k].first, out);
        out += ':';
        dump_value(v.obj[k].second, out);
      }
      out += '}';
      break;
  }
}

}  // namespace

Json Json::parse(const std::string& text) {
  Parser p(text);
  Json v = p.value();
  return v;
}

std::string Json::dump() const {
  std::string out;
  dump_value(*this, out);
  return out;
}


// ---------------------------------------------------------------------------
// Universal Binary JSON
// ---------------------------------------------------------------------------
namespace {
bool integral_text(const std::string& t) {
  if (t.empty()) return false;
  for (size_t i = 0; i < t.size(); ++i) {
    const char c = t[i];
    if (!(std::isdigit(static_cast<unsigned char>(c)) || (i == 0 && c == '-'))) return false;
  }
  return true;
}
template <typename T>
void put_be(std::string& out, T v) {
  unsigned char b[sizeof(T)];
  std::memcpy(b, &v, sizeof(T));
  for (size_t i = 0; i < sizeof(T); ++i) out += char(b[sizeof(T) - 1 - i]);
}
void put_len(std::string& out, size_t n) {
  out += 'L';
  put_be<int64_t>(out, int64_t(n));
}
void ubj_value(const Json& v, std::string& out) {
  switch (v.kind) {
    case Json::Null: out += 'Z'; break;
    case Json::Bool: out += v.b ? 'T' : 'F'; break;
    case Json::Number:
      if (integral_text(v.str)) {
        out += 'L';
        put_be<int64_t>(out, std::stoll(v.str));
      } else {
        out += 'd';
        put_be<float>(out, std::strtof(v.str.c_str(), nullptr));
      }
      break;
    case Json::String:
      out += 'S';
      put_len(out, v.str.size());
      out += v.str;
      break;
    case Json::Array: {
      bool numeric = !v.arr.empty(), fractional = false, wide = false;
      for (const Json& e : v.arr) {
        if (e.kind != Json::Number) {
          numeric = false;
          break;
        }
        if (!integral_text(e.str)) {
          fractional = true;
        } else {
          const long long x = std::stoll(e.str);
          if (x < INT32_MIN || x > INT32_MAX) wide = true;
        }
      }
      out += '[';
      if (numeric) {
        out += '$';
        out += fractional ? 'd' : (wide ? 'L' : 'l');
        out += '#';
        put_len(out, v.arr.size());
        for (const Json& e : v.arr) {
          if (fractional) put_be<float>(out, std::strtof(e.str.c_str(), nullptr));
          else if (wide) put_be<int64_t>(out, std::stoll(e.str));
          else put_be<int32_t>(out, int32_t(std::stoll(e.str)));
        }
      } else {
        for (const Json& e : v.arr) ubj_value(e, out);
        out += ']';
      }
      break;
    }
    case Json::Object:
      out += '{';
      for (const auto& kv : v.obj) {
        put_len(out, kv.first.size());
        out += kv.first;
        ubj_value(kv.second, out);
      }
      out += '}';
      break;
  }
}

struct UbjReader {
  const unsigned char* p;
  const unsigned char* end;
  unsigned char byte() {
    require(p < end, "Truncated UBJSON model.");
    return *p++;
  }
  template <typename T>
  T be() {
    require(size_t(end - p) >= sizeof(T), "Truncated UBJSON model.");
    unsigned char b[sizeof(T)];
    for (size_t i = 0; i < sizeof(T); ++i) b[sizeof(T) - 1 - i] = p[i];
    p += sizeof(T);
    T v;
    std::memcpy(&v, b, sizeof(T));
    return v;
  }
  int64_t integer(unsigned char m) {
    switch (m) {
      case 'i': return be<int8_t>();
      case 'U': return be<uint8_t>();
      case 'I': return be<int16_t>();
      case 'l': return be<int32_t>();
      case 'L': return be<int64_t>();
      default: require(false, "Invalid UBJSON integer marker."); return 0;
    }
  }
  size_t length() {
    const int64_t n = integer(byte());
    require(n >= 0 && uint64_t(n) <= uint64_t(end - p) * 8 + 64, "Invalid UBJSON length.");
    return size_t(n);
  }
  std::string text(size_t n) {
    require(size_t(end - p) >= n, "Truncated UBJSON model.");
    std::string s(reinterpret_cast<const char*>(p), n);
    p += n;
    return s;
  }
  static Json number_text(std::string t) {
    Json v;
    v.kind = Json::Number;
    v.num = std::strtod(t.c_str(), nullptr);
    v.str = std::move(t);
    return v;
  }
  Json typed(unsigned char m) {
    char buf[40];
    switch (m) {
      case 'Z': return Json{};
      case 'T': { Json v; v.kind = Json::Bool; v.b = true; return v; }
      case 'F': { Json v; v.kind = Json::Bool; return v; }
      case 'i': case 'U': case 'I': case 'l': case 'L': return number_text(std::to_string(integer(m)));
      case 'd': {
        const float x = be<float>();
        for (int digits = 6; digits <= 9; ++digits) {  // shortest text that reads back as x
          std::snprintf(buf, sizeof buf, "%.*g", digits, double(x));
          if (std::strtof(buf, nullptr) == x) break;
        }
        return number_text(buf);
      }
      case 'D': std::snprintf(buf, sizeof buf, "%.17g", be<double>()); return number_text(buf);
      case 'C': return number_text(std::to_string(int(byte())));
      case 'S': case 'H': { Json v; v.kind = Json::String; v.str = text(length()); return v; }
      case '[': return container(false);
      case '{': return container(true);
      default: require(false, "Invalid UBJSON marker."); return Json{};
    }
  }
  Json container(bool object) {
    Json v;
    v.kind = object ? Json::Object : Json::Array;
    unsigned char type = 0;
    int64_t count = -1;
    if (p < end && *p == '$') {
      ++p;
      type = byte();
      require(p < end && *p == '#', "UBJSON typed container without a count.");
    }
    if (p < end && *p == '#') {
      ++p;
      count = int64_t(length());
    }
    for (int64_t k = 0; count < 0 || k < count; ++k) {
      if (count < 0 && p < end && *p == (object ? '}' : ']')) {
        ++p;
        break;
      }
      std::string key;
      if (object) key = text(length());
      Json e = type ? typed(type) : typed(byte());
      if (object) v.obj.emplace_back(std::move(key), std::move(e));
      else v.arr.push_back(std::move(e));
    }
    return v;
  }
};
}  // namespace

std::string Json::dump_ubj() const {
  std::string out;
  ubj_value(*this, out);
  return out;
}

Json Json::parse_ubj(const void* data, size_t size) {
  UbjReader r{static_cast<const unsigned char*>(data), static_cast<const unsigned char*>(data) + size};
  return r.typed(r.byte());
}

}  // namespace xgbb
