// Evaluation metrics on the host. Per-row terms follow the reference's
// metric_partial kernel (kernels/boost.metal:2225-2270) in float32; the sums
// are taken in binary64, and a metric is the weighted mean of its terms
// (src/metrics.cpp:148-158). AUC integrates the weighted ROC curve with ties
// as trapezoids, one class against the rest for multiclass models, weighted
// by each class's positive weight (src/metrics.cpp:84-146).
#include "metrics.h"

#include <algorithm>
#include <cmath>
#include <limits>
#include <numeric>
#include <string>
#include <vector>

#include "common.h"

namespace xgbb {
namespace {

constexpr double kNaN = std::numeric_limits<double>::quiet_NaN();

// Area under the ROC curve of `score` for labels in [0, 1] (fractional labels
// count partially on both sides); NaN without positive or negative weight.
double roc_auc(const std::vector<float>& score, const std::vector<float>& label, const float* weights,
               double* positive_weight) {
  const size_t n = score.size();
  std::vector<uint32_t> order(n);
  std::iota(order.begin(), order.end(), 0u);
  std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) { return score[a] > score[b]; });
  double tp = 0, fp = 0, area = 0;
  for (size_t i = 0; i < n;) {
    const double tp0 = tp, fp0 = fp;
    size_t j = i;
    for (; j < n && score[order[j]] == score[order[i]]; ++j) {
      const uint32_t r = order[j];
      const double w = weights ? double(weights[r]) : 1.0;
      tp += w * label[r];
      fp += w * (1.0 - label[r]);
    }
    area += (fp - fp0) * (tp + tp0) / 2.0;
    i = j;
  }
  if (positive_weight) *positive_weight = tp;
  if (!(tp > 0 && fp > 0)) return kNaN;
  return area / (tp * fp);
}

}  // namespace

std::string default_metric(const std::string& objective) {
  if (objective == "binary:logistic" || objective == "binary:logitraw") return "logloss";
  if (objective == "multi:softprob" || objective == "multi:softmax") return "mlogloss";
  return "rmse";
}

bool metric_needs_all_rows(const std::string& name) { return name.substr(0, name.find('@')) == "auc"; }

double eval_metric(const std::string& name, const float* pred, uint32_t rows, uint32_t groups,
                   const float* labels, const float* weights, bool multiclass) {
  const size_t at = name.find('@');
  const std::string base = name.substr(0, at);
  if (base != "auc") {
    double loss_sum = 0, weight_sum = 0;
    metric_sums(name, pred, rows, groups, labels, weights, multiclass, &loss_sum, &weight_sum);
    return metric_from_sums(name, loss_sum, weight_sum);
  }
  {
    if (rows == 0) return kNaN;
    if (!multiclass) {
      for (uint32_t r = 0; r < rows; ++r)
        require(labels[r] >= 0 && labels[r] <= 1, "AUC labels must be in [0,1].");
      return roc_auc(std::vector<float>(pred, pred + rows), std::vector<float>(labels, labels + rows), weights,
                     nullptr);
    }
    double sum = 0, total = 0;
    std::vector<float> score(rows), onehot(rows);
    for (uint32_t k = 0; k < groups; ++k) {
      for (uint32_t r = 0; r < rows; ++r) {
        score[r] = pred[size_t(r) * groups + k];
        onehot[r] = labels[r] == float(k) ? 1.0f : 0.0f;
      }
      double pos = 0;
      const double auc = roc_auc(score, onehot, weights, &pos);
      if (std::isnan(auc)) return kNaN;
      sum += auc * pos;
      total += pos;
    }
    return total > 0 ? sum / total : kNaN;
  }
}

namespace {
int metric_type(const std::string& base) {
  static const char* const kNames[] = {"rmse", "mae", "rmsle", "logloss", "merror", "mlogloss", "error", "mape"};
  for (int i = 0; i < 8; ++i)
    if (base == kNames[i]) return i;
  return -1;
}
}  // namespace

double metric_from_sums(const std::string& name, double loss_sum, double weight_sum) {
  const int type = metric_type(name.substr(0, name.find('@')));
  require(type >= 0, "Metric has not been implemented yet: " + name);
  const double mean = weight_sum > 0 ? loss_sum / weight_sum : kNaN;
  return type == 0 || type == 2 ? std::sqrt(mean) : mean;
}

void metric_sums(const std::string& name, const float* pred, uint32_t rows, uint32_t groups, const float* labels,
                 const float* weights, bool multiclass, double* loss_out, double* weight_out) {
  const size_t at = name.find('@');
  const std::string base = name.substr(0, at);
  const std::string param = at == std::string::npos ? "" : name.substr(at + 1);
  const int type = metric_type(base);
  require(type >= 0, "Metric has not been implemented yet: " + name);
  const bool per_row = type == 4 || type == 5;
  if (per_row || multiclass)
    for (uint32_t r = 0; r < rows; ++r)
      require(labels[r] >= 0 && labels[r] < float(groups) && std::floor(labels[r]) == labels[r],
              "Multiclass evaluation label is out of range.");
  const float threshold = type == 6 && !param.empty() ? std::stof(param) : 0.5f;
  const uint64_t count = uint64_t(rows) * (per_row ? 1 : groups);
  double loss_sum = 0, weight_sum = 0;
  for (uint64_t i = 0; i < count; ++i) {
    const uint32_t row = uint32_t(per_row ? i : i / groups);
    const uint32_t group = per_row ? 0 : uint32_t(i % groups);
    const float w = weights ? weights[row] : 1.0f;
    const float y = labels[row];
    const float p = pred[size_t(row) * groups + group];
    float loss = 0;
    switch (type) {
      case 0: loss = (p - y) * (p - y); break;
      case 1: loss = std::fabs(p - y); break;
      case 2: {
        const float delta = std::log1p(p) - std::log1p(y);
        loss = delta * delta;
        break;
      }
      case 3:
        loss = -y * std::log(std::max(p, 1.0e-16f)) - (1 - y) * std::log(std::max(1 - p, 1.0e-16f));
        break;
      case 4: {
        uint32_t best = 0;
        for (uint32_t k = 1; k < groups; ++k)
          if (pred[size_t(row) * groups + k] > pred[size_t(row) * groups + best]) best = k;
        loss = float(best != uint32_t(y));
        break;
      }
      case 5: loss = -std::log(std::max(pred[size_t(row) * groups + uint32_t(y)], 1.0e-16f)); break;
      case 6: loss = p > threshold ? 1 - y : y; break;  // a fractional label counts partially
      case 7: loss = std::fabs((p - y) / y); break;
    }
    loss_sum += double(w * loss);
    weight_sum += double(w);
  }
  *loss_out = loss_sum;
  *weight_out = weight_sum;
}

}  // namespace xgbb
