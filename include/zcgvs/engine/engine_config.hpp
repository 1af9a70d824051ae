// The engine configuration of the reference (include/zcgvs/engine/engine_config.hpp:12-63): the
// same fields, names and defaults, so the reference's JSON configs (configs/*.json) describe an
// engine here too. The search-path fields feed VectorEngineConfig (toVectorEngineConfig); the
// text-stage fields (vocabulary, ONNX encoder and reranker) are carried for completeness and are
// not used by this library, which takes query vectors and token ids instead. Loaded from JSON by
// zcgvs/engine/config_loader.hpp.
#pragma once

#include <string>

#include "zcgvs/core/metric.hpp"
#include "zcgvs/search/search_params.hpp"

namespace zcgvs {

enum class RerankerBackend { Onnx };

struct EngineConfig {
    std::string embeddings_path;
    std::string metadata_path;
    std::string vocab_path;
    // Same corpus, same order, higher precision: the coarse scan's candidates are rescored
    // against it.
    std::string rescore_embeddings_path;
    // CSR BM25 index; makes the hybrid stage available.
    std::string lexical_index_path;

    std::string encoder_model_path;
    std::string encoder_output_name = "last_hidden_state";
    int encoder_max_seq_len = 256;

    RerankerBackend reranker_backend = RerankerBackend::Onnx;
    std::string reranker_model_path;  // empty: retrieval only
    std::string reranker_output_name = "logits";
    int reranker_max_seq_len = 256;
    int reranker_batch_size = 32;

    int device_id = 0;
    bool lowercase = true;

    Metric metric = Metric::Cosine;
    SimilarityBackend similarity_backend = SimilarityBackend::Custom;

    int default_top_k = 10;
    int default_candidates = 100;
    int rescore_candidates = 0;  // 0: no rescore stage even with a rescore store
    bool hybrid = false;         // run the BM25 stage by default (needs the index)
    float dense_weight = 0.7f;   // weight of the dense score in the hybrid blend
    int max_query_terms = 64;
    bool use_cuda_graphs = false;
};

}  // namespace zcgvs
