// The search driver (the reference's Searcher, include/zcgvs/search/searcher.hpp:32-63), over the
// fused kernels of this library: one zcgvs_scan_topk (or zcgvs_hybrid_topk with a lexical index)
// per search, followed by zcgvs_rescore_topk when a rescore store is attached. Same public
// interface and exceptions; optional CUDA-graph replay keyed by the launches' own argument list.
// Not thread-safe (one Searcher per thread / stream / GPU), like the reference.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "zcgvs/core/cuda_stream.hpp"
#include "zcgvs/core/device_buffer.hpp"
#include "zcgvs/core/pinned_buffer.hpp"
#include "zcgvs/data/embedding_store.hpp"
#include "zcgvs/data/lexical_index.hpp"
#include "zcgvs/search/search_params.hpp"
#include "zcgvs/search/search_result.hpp"

namespace zcgvs {

class Searcher {
public:
    explicit Searcher(const EmbeddingStore& store);
    ~Searcher();

    Searcher(const Searcher&) = delete;
    Searcher& operator=(const Searcher&) = delete;

    // Higher-precision copy of the corpus (same order) for rescoring; nullptr disables it.
    void setRescoreStore(const EmbeddingStore* store);
    // CSR inverted index enabling the hybrid lexical stage; nullptr disables it.
    void setLexicalIndex(const LexicalIndex* index);

    void search(const float* host_queries, int dim, int batch, const SearchParams& params, const CudaStream& stream);
    // Copies the last search's result to the host (synchronising `stream`). Throws
    // std::runtime_error when the search's kernels left a non-zero device status word (a bounded
    // wait ran out, or a query of the tensor-core path kept more candidates than its buffer
    // holds): the result may be incomplete. The word is cleared first, so the next search runs.
    HostTopK copyResultToHost(const CudaStream& stream);

    int resultK() const { return current_k_; }
    int resultBatch() const { return current_batch_; }
    double lastSearchGpuMs() const { return last_gpu_ms_; }
    bool lastSearchUsedGraph() const { return used_graph_; }
    std::uint64_t graphCaptureCount() const { return graph_captures_; }
    std::uint64_t graphLaunchCount() const { return graph_launches_; }
    bool hasRescoreStore() const { return rescore_store_ != nullptr; }
    bool hasLexicalIndex() const { return lexical_index_ != nullptr; }

private:
    void validate(int dim, int batch, const SearchParams& params, std::int64_t doc_count) const;
    void ensureCapacity(std::int64_t doc_count, int batch, const SearchParams& params);
    // Launches one search on `stream`, or, with `key`, only lists the launches' arguments: the
    // key of its CUDA graph, which replays only for searches with identical launches.
    void recordPipeline(std::int64_t doc_count, int batch, const SearchParams& params, cudaStream_t stream,
                        std::vector<std::uint64_t>* key = nullptr);
    bool lexicalEnabled(const SearchParams& params) const;
    bool rescoreEnabled(const SearchParams& params) const;
    void destroyGraph() noexcept;

    const EmbeddingStore& store_;
    const EmbeddingStore* rescore_store_ = nullptr;
    const LexicalIndex* lexical_index_ = nullptr;
    int dim_ = 0;

    DeviceBuffer<float> d_queries_;
    DeviceBuffer<int> d_query_terms_;
    DeviceBuffer<std::uint8_t> d_workspace_;
    DeviceBuffer<int> d_coarse_indices_;
    DeviceBuffer<float> d_coarse_values_;
    DeviceBuffer<int> d_out_indices_;
    DeviceBuffer<float> d_out_values_;
    PinnedBuffer<float> h_queries_;
    PinnedBuffer<int> h_query_terms_;
    PinnedBuffer<int> h_out_indices_;
    PinnedBuffer<float> h_out_values_;
    PinnedBuffer<std::uint32_t> h_status_;  // the workspace's device status word, read with each result

    cudaEvent_t ev_start_ = nullptr;
    cudaEvent_t ev_end_ = nullptr;
    cudaGraphExec_t graph_exec_ = nullptr;
    std::vector<std::uint64_t> graph_key_;
    bool graph_valid_ = false;
    std::uint64_t graph_captures_ = 0;
    std::uint64_t graph_launches_ = 0;

    // Results of at most kHostResultMax (id, score) pairs are written by the search's last
    // kernel straight into the pinned host buffers (device-accessible under unified addressing),
    // saving the two device-to-host copies; larger ones go through device buffers and copies.
    static constexpr long long kHostResultMax = 16384;
    bool host_out_ = false;
    int current_k_ = 0;
    int current_batch_ = 0;
    double last_gpu_ms_ = 0.0;
    bool used_graph_ = false;
};

}  // namespace zcgvs
