// Host-side model inspection: tree dumps and feature importance of a trained
// forest. Needs no GPU.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

#include "learner.h"

namespace xgbb {

// One string per tree in "text", "json" or "dot" form (the reference's
// Learner::dump, src/model.cpp:334-429). `names` empty = "f<index>"; a feature
// typed "c" in `types` is rejected, since every split here is numerical.
std::vector<std::string> dump_trees(const std::vector<HostTree>& trees,
                                    const std::vector<std::string>& names,
                                    const std::vector<std::string>& types,
                                    const std::string& format, bool stats);

struct FeatureScores {
  std::vector<std::string> names;
  std::vector<float> scores;
};

// Importance of every feature used by a split ("weight", "gain", "cover",
// "total_gain" or "total_cover"), in feature order (the reference's
// XGBoosterFeatureScore, src/c_api.cpp:590-620).
FeatureScores feature_scores(const std::vector<HostTree>& trees, uint32_t num_feature,
                             const std::vector<std::string>& names, const std::string& kind);

}  // namespace xgbb
