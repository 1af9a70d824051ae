// JSON engine configs: the C++ form of the reference's python/zcgvs_tools/config.py:54-96
// (config_from_dict / config_from_json), with the same rules:
//   - every key must name an EngineConfig field, else std::invalid_argument
//     ("unknown config field: <key>");
//   - "metric" takes cosine | dot | dotproduct | ip | l2 | euclidean and "similarity_backend"
//     custom | cublas, in any letter case (else std::invalid_argument "unknown metric '<name>'" /
//     "unknown similarity backend '<name>'");
//   - a non-empty path field (embeddings_path, metadata_path, vocab_path,
//     rescore_embeddings_path, lexical_index_path, encoder_model_path, reranker_model_path) is
//     kept when it is absolute or exists relative to the working directory, else resolved
//     against the first search root holding it, else kept as written. configFromJsonFile's roots
//     are the file's directory and its parent (a config under configs/ names repository paths);
//   - a value of the wrong JSON type for its field is std::invalid_argument naming the field.
// Implemented in csrc/config.cpp with a small JSON reader of its own (no dependency).
#pragma once

#include <string>
#include <vector>

#include "zcgvs/engine/engine_config.hpp"
#include "zcgvs/engine/vector_engine.hpp"

namespace zcgvs {

// config.py's metric_from_name: strict (an unknown name throws) and case-insensitive, unlike
// the lenient metricFromName of zcgvs/core/metric.hpp, which maps unknown names to cosine.
Metric configMetricFromName(const std::string& name);
SimilarityBackend similarityBackendFromName(const std::string& name);

// Parses a JSON object of config fields.
EngineConfig configFromJsonText(const std::string& json, const std::vector<std::string>& search_roots = {});

// Reads and parses a config file (std::runtime_error when it cannot be read).
EngineConfig configFromJsonFile(const std::string& path);

// The search-path fields of a configuration.
VectorEngineConfig toVectorEngineConfig(const EngineConfig& config);

}  // namespace zcgvs
