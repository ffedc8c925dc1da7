#include "json.h"

#include <cctype>
#include <cstdio>
#include <cstdlib>

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

}  // namespace xgbb
