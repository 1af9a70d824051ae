// The request layer above Searcher, for callers that bring their own query vectors and token
// ids: the reference Engine's option resolution, allow-mask upload, lexical term preparation,
// result assembly, timings and stats (src/engine/engine.cpp:87-172, 228-310, 419-446), without
// its text stages (tokenizer, ONNX bi-encoder, cross-encoder, passage store), which are not on
// the search path this library replaces. One VectorEngine per thread / stream / GPU, like the
// reference (its Searcher is not thread-safe).
#pragma once

#include <algorithm>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <unordered_set>
#include <vector>

#include "zcgvs/core/cuda_stream.hpp"
#include "zcgvs/core/device_buffer.hpp"
#include "zcgvs/core/metric.hpp"
#include "zcgvs/data/embedding_store.hpp"
#include "zcgvs/data/lexical_index.hpp"
#include "zcgvs/engine/engine_stats.hpp"
#include "zcgvs/engine/search_hit.hpp"
#include "zcgvs/engine/search_options.hpp"
#include "zcgvs/engine/search_response.hpp"
#include "zcgvs/search/searcher.hpp"

namespace zcgvs {

// The search-path fields of the reference's EngineConfig (include/zcgvs/engine/engine_config.hpp),
// same names and defaults.
struct VectorEngineConfig {
    Metric metric = Metric::Cosine;
    SimilarityBackend similarity_backend = SimilarityBackend::Custom;
    int default_top_k = 10;
    int default_candidates = 100;
    int rescore_candidates = 0;
    bool hybrid = false;
    float dense_weight = 0.7f;
    int max_query_terms = 64;
    bool use_cuda_graphs = false;
    int device_id = 0;
};

// Options after defaults and clamps (the reference's Engine::ResolvedOptions).
struct ResolvedOptions {
    int top_k = 10;
    int candidates = 100;
    Metric metric = Metric::Cosine;
    int rescore_candidates = 0;
    float dense_weight = 1.0f;
    bool hybrid = false;
    bool rerank = false;
    SimilarityBackend backend = SimilarityBackend::Custom;
    bool use_graph = false;
};

// Engine::resolve (src/engine/engine.cpp:87-126): defaults for unset fields, dense_weight clamped
// to [0, 1], candidates >= top_k and <= the corpus, top_k <= candidates, rescore_candidates (only
// with a rescore store, when positive) >= candidates and <= the corpus. No reranker here.
inline ResolvedOptions resolveSearchOptions(const VectorEngineConfig& config, const SearchOptions& options,
                                            std::int64_t corpus_size, bool has_rescore_store,
                                            bool has_lexical_index) {
    ResolvedOptions r;
    r.top_k = options.top_k > 0 ? options.top_k : config.default_top_k;
    r.candidates = options.candidates > 0 ? options.candidates : config.default_candidates;
    r.metric = options.use_config_metric ? config.metric : options.metric;
    r.backend = options.use_config_backend ? config.similarity_backend : options.backend;
    r.use_graph = options.use_config_graphs ? config.use_cuda_graphs : options.use_graph;
    r.rerank = false;
    r.hybrid = options.hybrid && has_lexical_index;
    r.dense_weight = options.dense_weight >= 0.0f ? options.dense_weight : config.dense_weight;
    r.dense_weight = std::min(1.0f, std::max(0.0f, r.dense_weight));
    if (r.top_k <= 0) throw std::invalid_argument("zcgvs: top_k must be positive");
    r.candidates = std::max(r.top_k, r.candidates);
    if (r.candidates > corpus_size) r.candidates = static_cast<int>(corpus_size);
    if (r.top_k > r.candidates) r.top_k = r.candidates;
    if (has_rescore_store) {
        const int requested = options.rescore_candidates >= 0 ? options.rescore_candidates : config.rescore_candidates;
        r.rescore_candidates = std::max(requested, 0);
        if (r.rescore_candidates > 0) {
            r.rescore_candidates = std::max(r.rescore_candidates, r.candidates);
            if (r.rescore_candidates > corpus_size) r.rescore_candidates = static_cast<int>(corpus_size);
        }
    }
    return r;
}

// Engine::lexicalTerms on an encoded query (src/engine/engine.cpp:150-172): the tokenizer's ids
// without the first and last ([CLS] / [SEP]), negative ids dropped, first occurrences kept in
// order, at most max(1, max_terms) of them.
inline std::vector<int> lexicalTermsFromIds(const std::vector<int>& encoded, int max_terms) {
    std::vector<int> terms;
    if (encoded.size() <= 2) return terms;
    std::unordered_set<int> seen;
    const int limit = std::max(1, max_terms);
    for (std::size_t i = 1; i + 1 < encoded.size(); ++i) {
        const int id = encoded[i];
        if (id < 0 || !seen.insert(id).second) continue;
        terms.push_back(id);
        if (static_cast<int>(terms.size()) >= limit) break;
    }
    return terms;
}

// Engine::buildMask's host part (src/engine/engine.cpp:128-146): 1 for every allowed index in
// [0, doc_count), 0 elsewhere; empty when nothing is restricted.
inline std::vector<std::uint8_t> allowMask(const std::vector<int>& allow, std::int64_t doc_count) {
    std::vector<std::uint8_t> mask;
    if (allow.empty()) return mask;
    mask.assign(static_cast<std::size_t>(doc_count), 0);
    for (const int index : allow) {
        if (index >= 0 && index < doc_count) mask[static_cast<std::size_t>(index)] = 1;
    }
    return mask;
}

class VectorEngine {
public:
    // The stores and the index are borrowed and must outlive the engine.
    VectorEngine(const EmbeddingStore& store, const VectorEngineConfig& config,
                 const EmbeddingStore* rescore_store = nullptr, const LexicalIndex* lexical_index = nullptr);
    ~VectorEngine();
    VectorEngine(const VectorEngine&) = delete;
    VectorEngine& operator=(const VectorEngine&) = delete;

    // Options pre-filled from the configuration (Engine::defaultOptions).
    SearchOptions defaultOptions() const;

    // host_queries: [batch, dim] fp32. encoded_terms: per query, the tokenizer's ids of its text
    // ([CLS] ... [SEP]); used when the resolved options are hybrid. Hits per query: at most
    // top_k, best first.
    BatchSearchResponse searchBatch(const float* host_queries, int batch, const SearchOptions& options,
                                    const std::vector<std::vector<int>>& encoded_terms = {}) const;
    SearchResponse searchTimed(const float* host_query, const SearchOptions& options,
                               const std::vector<int>& encoded_terms = {}) const;
    // Dense-only top-k with an optional allow list (Engine::retrieve).
    std::vector<Candidate> retrieve(const float* host_query, int k, Metric metric, const std::vector<int>& allow) const;

    EngineStats stats() const;
    std::int64_t corpusSize() const { return store_.docCount(); }
    int dim() const { return store_.dim(); }
    bool hasLexicalIndex() const { return lexical_index_ != nullptr; }
    bool hasRescoreStore() const { return rescore_store_ != nullptr; }
    const VectorEngineConfig& config() const { return config_; }

private:
    const std::uint8_t* uploadMask(const std::vector<int>& allow) const;

    const EmbeddingStore& store_;
    const EmbeddingStore* rescore_store_;
    const LexicalIndex* lexical_index_;
    VectorEngineConfig config_;
    std::unique_ptr<Searcher> searcher_;
    std::unique_ptr<CudaStream> stream_;
    mutable DeviceBuffer<std::uint8_t> d_mask_;
    mutable std::vector<int> host_terms_;
};

}  // namespace zcgvs
