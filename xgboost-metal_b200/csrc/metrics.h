// Evaluation metrics on the host (XGBoosterEvalOneIter). They read the
// transformed predictions of a trained booster and the matrix's labels and
// weights; they are not on the training path.
#pragma once
#include <cstdint>
#include <string>

namespace xgbb {

// `name` is a metric with an optional "@parameter" ("error@0.7"); `pred` is
// [rows][groups] of transformed predictions (probabilities for logistic and
// multiclass objectives); `weights` may be null. Multiclass metrics (merror,
// mlogloss) take one label per row with groups columns of probabilities.
double eval_metric(const std::string& name, const float* pred, uint32_t rows, uint32_t groups,
                   const float* labels, const float* weights, bool multiclass);

// The weighted sum of per-row terms and the weight sum of a mean-type metric
// (every metric but auc), and the metric from them: rows split over ranks
// give the metric of all rows once both sums are added up.
bool metric_needs_all_rows(const std::string& name);
void metric_sums(const std::string& name, const float* pred, uint32_t rows, uint32_t groups, const float* labels,
                 const float* weights, bool multiclass, double* loss_sum, double* weight_sum);
double metric_from_sums(const std::string& name, double loss_sum, double weight_sum);

// The metric an objective is evaluated with when none is set
// (src/learner.cpp:1012-1024 in the reference).
std::string default_metric(const std::string& objective);

}  // namespace xgbb
