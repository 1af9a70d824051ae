// Lexical launchers (the reference's include/zcgvs/cuda/lexical.cuh:20-40), implemented over
// zcgvs_bm25 / zcgvs_max_positive / zcgvs_fuse_scores. launchBm25 sums in (term slot, posting)
// order, deterministically; it needs each term's postings sorted by document.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace zcgvs {
namespace cuda {

void launchBm25(const std::int64_t* d_offsets, const int* d_docs, const float* d_weights, const int* d_query_terms,
                int term_count, int doc_count, float* d_scores, cudaStream_t stream);
void launchMaxPositive(const float* d_values, int count, float* d_max, cudaStream_t stream);
void launchFuseScores(float* d_dense, const float* d_lexical, const float* d_lexical_max, float weight, int count,
                      cudaStream_t stream);

}  // namespace cuda
}  // namespace zcgvs
