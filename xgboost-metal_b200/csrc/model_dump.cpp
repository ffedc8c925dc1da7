// Tree dumps (text, JSON, Graphviz dot) and feature importance, computed on
// the host from the forest the booster keeps after every round.
#include "model_dump.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "common.h"

namespace xgbb {
namespace {

// Text and dot dumps print values with nine significant digits, as an
// ostream with setprecision(9) does (src/model.cpp:355, 386).
std::string g9(double v) {
  char buf[64];
  std::snprintf(buf, sizeof buf, "%.9g", v);
  return buf;
}

// JSON dumps print each binary64 value with the fewest digits that read back
// to the same value, in the layout of the reference's JSON library: plain
// decimals while the decimal point sits within 15 digits, "0.000ddd" down to
// 1e-4, otherwise d.ddde±XX; integral values keep a ".0"; non-finite values
// are written nan / inf / -inf (src/data.cpp:67-93, tree dumps).
std::string json_double(double v) {
  if (std::isnan(v)) return "nan";
  if (std::isinf(v)) return v < 0 ? "-inf" : "inf";
  std::string out;
  if (std::signbit(v)) {
    out += '-';
    v = -v;
  }
  if (v == 0) return out + "0.0";
  char buf[64];
  int p = 1;
  for (; p <= 17; ++p) {
    std::snprintf(buf, sizeof buf, "%.*e", p - 1, v);
    if (std::strtod(buf, nullptr) == v) break;
  }
  // buf = d[.ddd]e±XX: digits and the position of the decimal point.
  std::string digits;
  const char* c = buf;
  for (; *c && *c != 'e'; ++c)
    if (*c != '.') digits += *c;
  const int exp10 = std::atoi(c + 1);
  while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
  const int k = int(digits.size());
  const int n = exp10 + 1;
  if (k <= n && n <= 15) return out + digits + std::string(size_t(n - k), '0') + ".0";
  if (0 < n && n <= 15) return out + digits.substr(0, size_t(n)) + "." + digits.substr(size_t(n));
  if (-4 < n && n <= 0) return out + "0." + std::string(size_t(-n), '0') + digits;
  std::string mant = digits.substr(0, 1);
  if (k > 1) mant += "." + digits.substr(1);
  const int e = n - 1;
  char ebuf[16];
  std::snprintf(ebuf, sizeof ebuf, "e%c%02d", e < 0 ? '-' : '+', e < 0 ? -e : e);
  return out + mant + ebuf;
}

std::string json_string(const std::string& s) {
  std::string out = "\"";
  for (unsigned char ch : s) {
    switch (ch) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\b': out += "\\b"; break;
      case '\f': out += "\\f"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      default:
        if (ch < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof buf, "\\u%04x", ch);
          out += buf;
        } else {
          out += char(ch);
        }
    }
  }
  return out + "\"";
}

struct Dumper {
  const HostTree& tree;
  const std::vector<std::string>& names;
  const std::vector<std::string>& types;
  bool stats;
  std::string out;

  const DevNode& node(int32_t id) const {
    require(id >= 0 && size_t(id) < tree.nodes.size(), "Tree node index out of range.");
    return tree.nodes[size_t(id)];
  }

  std::string feature_name(const DevNode& n) const {
    std::string name;
    if (names.empty()) {
      name = "f" + std::to_string(n.feature);
    } else {
      require(n.feature >= 0 && size_t(n.feature) < names.size(), "Feature name list is shorter than the model's features.");
      name = names[size_t(n.feature)];
    }
    if (n.feature >= 0 && size_t(n.feature) < types.size() && types[size_t(n.feature)] == "c")
      throw Error(name + " in feature map is categorical but the tree node is numerical.");
    return name;
  }

  // "<tabs>id:[fK<t] yes=L,no=R,missing=M[,gain=G,cover=C]" or
  // "<tabs>id:leaf=v[,cover=C]" (src/model.cpp:410-419).
  void text(int32_t id, uint32_t depth) {
    const DevNode& n = node(id);
    out.append(depth, '\t');
    out += std::to_string(id) + ":";
    if (n.left < 0) {
      out += "leaf=" + g9(n.leaf);
    } else {
      out += "[" + feature_name(n) + "<" + g9(n.threshold) + "] yes=" + std::to_string(n.left) +
             ",no=" + std::to_string(n.right) + ",missing=" + std::to_string(n.default_left ? n.left : n.right);
    }
    if (stats) {
      if (n.left >= 0) out += ",gain=" + g9(n.gain);
      out += ",cover=" + g9(n.cover);
    }
    out += '\n';
    if (n.left >= 0) {
      text(n.left, depth + 1);
      text(n.right, depth + 1);
    }
  }

  // Graphviz: one labelled vertex per node, yes/no edges marked with the
  // missing-value direction (src/model.cpp:398-409).
  void dot(int32_t id) {
    const DevNode& n = node(id);
    out += "    " + std::to_string(id) + " [ label=\"";
    out += n.left < 0 ? "leaf=" + g9(n.leaf) : feature_name(n) + "<" + g9(n.threshold);
    if (stats) out += "\\ncover=" + g9(n.cover);
    out += "\" ]\n";
    if (n.left >= 0) {
      out += "    " + std::to_string(id) + " -> " + std::to_string(n.left) + " [ label=\"yes" +
             (n.default_left ? ", missing" : "") + "\" ]\n";
      out += "    " + std::to_string(id) + " -> " + std::to_string(n.right) + " [ label=\"no" +
             (!n.default_left ? ", missing" : "") + "\" ]\n";
      dot(n.left);
      dot(n.right);
    }
  }

  // Nested objects with sorted keys, two-space indent (src/model.cpp:383-397).
  void json(int32_t id, uint32_t depth, int indent) {
    const DevNode& n = node(id);
    const std::string pad(size_t(indent + 2), ' '), close(size_t(indent), ' ');
    std::vector<std::pair<const char*, std::string>> fields;
    std::string children;
    if (n.left >= 0) {
      const std::string inner(size_t(indent + 4), ' ');
      children = "[\n" + inner;
      Dumper l{tree, names, types, stats, {}};
      l.json(n.left, depth + 1, indent + 4);
      Dumper r{tree, names, types, stats, {}};
      r.json(n.right, depth + 1, indent + 4);
      children += l.out + ",\n" + inner + r.out + "\n" + pad + "]";
      fields.emplace_back("children", children);
    }
    if (stats) fields.emplace_back("cover", json_double(n.cover));
    if (n.left >= 0) {
      fields.emplace_back("depth", std::to_string(depth));
      if (stats) fields.emplace_back("gain", json_double(n.gain));
    } else {
      fields.emplace_back("leaf", json_double(n.leaf));
    }
    if (n.left >= 0) {
      fields.emplace_back("missing", std::to_string(n.default_left ? n.left : n.right));
      fields.emplace_back("no", std::to_string(n.right));
    }
    fields.emplace_back("nodeid", std::to_string(id));
    if (n.left >= 0) {
      fields.emplace_back("split", json_string(feature_name(n)));
      fields.emplace_back("split_condition", json_double(n.threshold));
      fields.emplace_back("yes", std::to_string(n.left));
    }
    out += "{\n";
    for (size_t i = 0; i < fields.size(); ++i) {
      out += pad + "\"" + fields[i].first + "\": " + fields[i].second;
      out += i + 1 < fields.size() ? ",\n" : "\n";
    }
    out += close + "}";
  }
};

}  // namespace

std::vector<std::string> dump_trees(const std::vector<HostTree>& trees,
                                    const std::vector<std::string>& names,
                                    const std::vector<std::string>& types,
                                    const std::string& format, bool stats) {
  require(format == "text" || format == "json" || format == "dot", "Unknown dump format.");
  std::vector<std::string> result;
  result.reserve(trees.size());
  for (const HostTree& tree : trees) {
    require(!tree.nodes.empty(), "A tree must have a root node.");
    Dumper d{tree, names, types, stats, {}};
    if (format == "json") {
      d.json(0, 0, 0);
    } else if (format == "dot") {
      d.out = "digraph {\n    graph [ rankdir=TB ]\n";
      d.dot(0);
      d.out += "}\n";
    } else {
      d.text(0, 0);
    }
    result.push_back(std::move(d.out));
  }
  return result;
}

FeatureScores feature_scores(const std::vector<HostTree>& trees, uint32_t num_feature,
                             const std::vector<std::string>& names, const std::string& kind) {
  require(kind == "weight" || kind == "gain" || kind == "cover" || kind == "total_gain" || kind == "total_cover",
          "Unknown importance type.");
  require(names.empty() || names.size() == num_feature, "Feature name length is invalid.");
  std::vector<double> total(num_feature, 0.0);
  std::vector<uint32_t> count(num_feature, 0);
  const bool gain = kind == "gain" || kind == "total_gain";
  for (const HostTree& tree : trees)
    for (const DevNode& n : tree.nodes) {
      if (n.left < 0) continue;
      require(n.feature >= 0 && uint32_t(n.feature) < num_feature, "Split feature out of range.");
      ++count[size_t(n.feature)];
      total[size_t(n.feature)] += kind == "weight" ? 1.0 : (gain ? double(n.gain) : double(n.cover));
    }
  const bool average = kind == "gain" || kind == "cover";
  FeatureScores out;
  for (uint32_t f = 0; f < num_feature; ++f) {
    if (!count[f]) continue;
    out.names.push_back(names.empty() ? "f" + std::to_string(f) : names[f]);
    out.scores.push_back(float(total[f] / (average ? count[f] : 1)));
  }
  return out;
}

}  // namespace xgbb
