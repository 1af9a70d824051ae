// Row-sharded search across the GPUs of one node (one process per GPU), the multi-GPU form of
// Searcher: the corpus' rows are split evenly over `world` ranks, rank r holds rows
// [shardBegin(), shardEnd()) in its stores, and every search returns the global top-k on every
// rank, identical to a one-GPU Searcher over the whole corpus. No reference counterpart (the
// reference runs on one GPU); the interface follows Searcher's (search, then copyResultToHost).
// Implemented over zcgvs_sharded_* (NCCL all-gathers, device merges, one CUDA graph per search
// shape when params.use_graph is set). Every rank must make the same calls in the same order.
#pragma once

#include <cstdint>
#include <vector>

#include "zcgvs/core/cuda_stream.hpp"
#include "zcgvs/core/device_buffer.hpp"
#include "zcgvs/core/pinned_buffer.hpp"
#include "zcgvs/data/embedding_store.hpp"
#include "zcgvs/search/search_params.hpp"
#include "zcgvs/search/search_result.hpp"

struct zcgvs_sharded;

namespace zcgvs {

class ShardedSearcher {
public:
    // An NCCL unique id, made once by rank 0 and sent to the other ranks by the caller.
    static std::vector<char> uniqueId();
    // Rows [begin, end) of `rank`'s shard of total_rows rows.
    static void shardBounds(std::int64_t total_rows, int world, int rank, std::int64_t* begin, std::int64_t* end);

    // A collective: every rank constructs its searcher with the same id, world and total_rows,
    // with its GPU current.
    ShardedSearcher(const std::vector<char>& nccl_id, int world, int rank, std::int64_t total_rows);
    ~ShardedSearcher();
    ShardedSearcher(const ShardedSearcher&) = delete;
    ShardedSearcher& operator=(const ShardedSearcher&) = delete;

    std::int64_t shardBegin() const { return begin_; }
    std::int64_t shardEnd() const { return end_; }

    // This rank's rows of a higher-precision store for rescoring (same shard); nullptr disables.
    void setRescoreStore(const EmbeddingStore* shard_store);

    // Searches `shard` (this rank's rows; the coarse store when rescoring) with host fp32
    // queries; params as for Searcher (k, metric, d_mask over the shard's rows, rescore
    // candidates, use_graph; no lexical stage). Asynchronous on `stream`.
    void search(const EmbeddingStore& shard, const float* host_queries, int dim, int batch, const SearchParams& params,
                const CudaStream& stream);
    // The global [batch, k] result (synchronises `stream`). Throws std::runtime_error when a
    // kernel left a non-zero device status word or NCCL reported an asynchronous error.
    HostTopK copyResultToHost(const CudaStream& stream);

private:
    zcgvs_sharded* handle_ = nullptr;
    const EmbeddingStore* rescore_store_ = nullptr;
    std::int64_t begin_ = 0;
    std::int64_t end_ = 0;
    DeviceBuffer<float> d_queries_;
    DeviceBuffer<int> d_out_indices_;
    DeviceBuffer<float> d_out_values_;
    PinnedBuffer<float> h_queries_;
    PinnedBuffer<int> h_out_indices_;
    PinnedBuffer<float> h_out_values_;
    int current_k_ = 0;
    int current_batch_ = 0;
};

}  // namespace zcgvs
