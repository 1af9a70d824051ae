// VectorEngine (include/zcgvs/engine/vector_engine.hpp): the reference Engine's request path
// (src/engine/engine.cpp:228-310) over this library's Searcher, for query vectors and token ids.
#include "zcgvs/engine/vector_engine.hpp"

#include <cuda_runtime.h>

#include <chrono>
#include <stdexcept>
#include <string>

#include "zcgvs/core/cuda_check.hpp"

namespace zcgvs {

namespace {

using Clock = std::chrono::steady_clock;

double elapsed_ms(Clock::time_point a, Clock::time_point b) {
    return std::chrono::duration<double, std::milli>(b - a).count();
}

}  // namespace

VectorEngine::VectorEngine(const EmbeddingStore& store, const VectorEngineConfig& config,
                           const EmbeddingStore* rescore_store, const LexicalIndex* lexical_index)
    : store_(store), rescore_store_(rescore_store), lexical_index_(lexical_index), config_(config) {
    if (store.docCount() <= 0 || store.dim() <= 0) throw std::invalid_argument("zcgvs: the engine needs a non-empty corpus");
    if (lexical_index != nullptr && lexical_index->docCount() < store.docCount()) {
        throw std::invalid_argument("zcgvs: lexical index holds fewer documents than the corpus");
    }
    ZCGVS_CUDA_CHECK(cudaSetDevice(config.device_id));
    stream_ = std::make_unique<CudaStream>();
    searcher_ = std::make_unique<Searcher>(store_);
    searcher_->setRescoreStore(rescore_store_);
    searcher_->setLexicalIndex(lexical_index_);
}

VectorEngine::~VectorEngine() = default;

SearchOptions VectorEngine::defaultOptions() const {
    SearchOptions options;
    options.top_k = config_.default_top_k;
    options.candidates = config_.default_candidates;
    options.metric = config_.metric;
    options.rescore_candidates = config_.rescore_candidates;
    options.dense_weight = config_.dense_weight;
    options.hybrid = config_.hybrid && lexical_index_ != nullptr;
    options.rerank = false;
    options.use_config_backend = true;
    options.use_config_graphs = true;
    return options;
}

const std::uint8_t* VectorEngine::uploadMask(const std::vector<int>& allow) const {
    if (allow.empty()) return nullptr;
    const std::int64_t n = store_.docCount();
    const std::vector<std::uint8_t> mask = allowMask(allow, n);
    if (d_mask_.size() < static_cast<std::size_t>(n)) d_mask_.allocate(static_cast<std::size_t>(n));
    // Synchronous: the host vector dies with this call.
    ZCGVS_CUDA_CHECK(cudaMemcpyAsync(d_mask_.data(), mask.data(), mask.size(), cudaMemcpyHostToDevice, stream_->get()));
    ZCGVS_CUDA_CHECK(cudaStreamSynchronize(stream_->get()));
    return d_mask_.data();
}

BatchSearchResponse VectorEngine::searchBatch(const float* host_queries, int batch, const SearchOptions& options,
                                              const std::vector<std::vector<int>>& encoded_terms) const {
    if (batch <= 0 || host_queries == nullptr) throw std::invalid_argument("zcgvs: searchBatch requires at least one query");
    const auto t_start = Clock::now();
    const std::int64_t corpus_size = store_.docCount();
    const ResolvedOptions resolved =
        resolveSearchOptions(config_, options, corpus_size, rescore_store_ != nullptr, lexical_index_ != nullptr);

    double tokenize_ms = 0.0;
    int lexical_stride = 0;
    if (resolved.hybrid) {
        const auto t0 = Clock::now();
        if (!encoded_terms.empty() && static_cast<int>(encoded_terms.size()) != batch) {
            throw std::invalid_argument("zcgvs: encoded_terms must hold one list per query");
        }
        std::vector<std::vector<int>> per_query;
        for (int q = 0; q < static_cast<int>(encoded_terms.size()); ++q) {
            per_query.push_back(lexicalTermsFromIds(encoded_terms[static_cast<std::size_t>(q)], config_.max_query_terms));
            lexical_stride = std::max(lexical_stride, static_cast<int>(per_query.back().size()));
        }
        if (lexical_stride > 0) {
            host_terms_.assign(static_cast<std::size_t>(batch) * lexical_stride, -1);
            for (std::size_t q = 0; q < per_query.size(); ++q) {
                std::copy(per_query[q].begin(), per_query[q].end(),
                          host_terms_.begin() + static_cast<std::ptrdiff_t>(q * lexical_stride));
            }
        }
        tokenize_ms = elapsed_ms(t0, Clock::now());
    }

    SearchParams params;
    params.k = resolved.candidates;
    params.metric = resolved.metric;
    params.d_mask = uploadMask(options.allow);
    params.rescore_candidates = resolved.rescore_candidates;
    params.backend = resolved.backend;
    params.use_graph = resolved.use_graph;
    if (resolved.hybrid && lexical_stride > 0) {
        params.host_query_terms = host_terms_.data();
        params.lexical_stride = lexical_stride;
        params.dense_weight = resolved.dense_weight;
    }
    searcher_->search(host_queries, store_.dim(), batch, params, *stream_);
    const auto t_copy = Clock::now();
    const HostTopK selection = searcher_->copyResultToHost(*stream_);
    const auto t_copied = Clock::now();

    // Engine::assemble without passages or a reranker: valid ids in selection order (already
    // best first), truncated to top_k.
    BatchSearchResponse response;
    response.results.resize(static_cast<std::size_t>(batch));
    for (int q = 0; q < batch; ++q) {
        std::vector<SearchHit>& hits = response.results[static_cast<std::size_t>(q)];
        const std::size_t base = selection.offset(q);
        for (int i = 0; i < selection.k && static_cast<int>(hits.size()) < resolved.top_k; ++i) {
            const int index = selection.indices[base + static_cast<std::size_t>(i)];
            if (index < 0 || index >= corpus_size) continue;
            SearchHit hit;
            hit.corpus_index = index;
            hit.similarity = selection.scores[base + static_cast<std::size_t>(i)];
            hit.rerank_score = hit.similarity;
            hits.push_back(std::move(hit));
        }
    }
    response.timing.tokenize_ms = tokenize_ms;
    response.timing.search_gpu_ms = searcher_->lastSearchGpuMs();
    response.timing.copy_ms = elapsed_ms(t_copy, t_copied);
    response.timing.total_ms = elapsed_ms(t_start, Clock::now());
    response.timing.batch = batch;
    response.timing.graph_replay = searcher_->lastSearchUsedGraph();
    return response;
}

SearchResponse VectorEngine::searchTimed(const float* host_query, const SearchOptions& options,
                                         const std::vector<int>& encoded_terms) const {
    std::vector<std::vector<int>> terms;
    if (!encoded_terms.empty()) terms.push_back(encoded_terms);
    BatchSearchResponse batch = searchBatch(host_query, 1, options, terms);
    SearchResponse response;
    response.hits = std::move(batch.results.front());
    response.timing = batch.timing;
    return response;
}

std::vector<Candidate> VectorEngine::retrieve(const float* host_query, int k, Metric metric,
                                              const std::vector<int>& allow) const {
    if (k <= 0) throw std::invalid_argument("zcgvs: retrieve requires k > 0");
    SearchOptions options;
    options.top_k = k;
    options.candidates = k;
    options.use_config_metric = false;
    options.metric = metric;
    options.allow = allow;
    options.rescore_candidates = 0;
    options.hybrid = false;
    const BatchSearchResponse response = searchBatch(host_query, 1, options);
    std::vector<Candidate> out;
    for (const SearchHit& hit : response.results.front()) {
        Candidate c;
        c.corpus_index = hit.corpus_index;
        c.score = hit.similarity;
        out.push_back(c);
    }
    return out;
}

EngineStats VectorEngine::stats() const {
    EngineStats s;
    s.corpus_size = store_.docCount();
    s.dim = store_.dim();
    s.storage_dtype = scalarName(store_.dtype());
    s.corpus_bytes = store_.deviceBytes();
    if (rescore_store_ != nullptr) {
        s.has_rescore_store = true;
        s.rescore_dtype = scalarName(rescore_store_->dtype());
        s.rescore_bytes = rescore_store_->deviceBytes();
    }
    if (lexical_index_ != nullptr) {
        s.has_lexical_index = true;
        s.lexical_postings = lexical_index_->postingCount();
        s.lexical_bytes = lexical_index_->deviceBytes();
    }
    s.has_reranker = false;
    s.graph_captures = searcher_->graphCaptureCount();
    s.graph_launches = searcher_->graphLaunchCount();
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, config_.device_id) == cudaSuccess) {
        s.device_name = prop.name;
        s.device_total_memory = prop.totalGlobalMem;
        s.compute_major = prop.major;
        s.compute_minor = prop.minor;
    }
    return s;
}

}  // namespace zcgvs
