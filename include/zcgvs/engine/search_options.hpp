// Per-request knobs of the engine (the reference's SearchOptions,
// include/zcgvs/engine/search_options.hpp:8-27): fields left at their sentinel fall back to the
// engine configuration.
#pragma once

#include <vector>

#include "zcgvs/core/metric.hpp"
#include "zcgvs/search/search_params.hpp"

namespace zcgvs {

struct SearchOptions {
    int top_k = 0;       // <= 0: the configured default_top_k
    int candidates = 0;  // <= 0: the configured default_candidates
    bool use_config_metric = true;
    Metric metric = Metric::Cosine;
    // Corpus indices the search is restricted to; empty means no restriction.
    std::vector<int> allow;
    int rescore_candidates = -1;  // < 0: the configured rescore_candidates
    float dense_weight = -1.0f;   // < 0: the configured dense_weight
    bool hybrid = false;
    bool rerank = true;
    bool use_config_backend = true;
    SimilarityBackend backend = SimilarityBackend::Custom;
    bool use_config_graphs = true;
    bool use_graph = false;
};

}  // namespace zcgvs
