// Score-matrix launcher (the reference's include/zcgvs/cuda/similarity.cuh:20-36), implemented
// over zcgvs_similarity. Float storage takes fp32 queries, binary storage packed query words.
// Throws std::invalid_argument on invalid arguments and zcgvs::CudaError on CUDA errors.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "zcgvs/core/metric.hpp"
#include "zcgvs/core/scalar_type.hpp"

namespace zcgvs {
namespace cuda {

void launchSimilarity(const void* d_corpus, ScalarType dtype, float scale, int doc_count, int dim,
                      const void* d_queries, int batch, const std::uint8_t* d_mask, Metric metric,
                      float* d_scores, cudaStream_t stream);

// Queries one launch scores together (8).
int similarityQueryTile();

// Shared memory one launch stages queries in: min(8, batch) queries of dim fp32 values (or packed
// words); throws std::invalid_argument when one query does not fit.
std::size_t similaritySharedBytes(ScalarType dtype, int dim, int batch);

}  // namespace cuda
}  // namespace zcgvs
