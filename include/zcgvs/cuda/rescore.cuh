// Rescore launchers (the reference's include/zcgvs/cuda/rescore.cuh:20-45), implemented over
// zcgvs_gather_rescore / zcgvs_remap_indices. The fused form is zcgvs_rescore_topk.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>

#include "zcgvs/core/metric.hpp"
#include "zcgvs/core/scalar_type.hpp"

namespace zcgvs {
namespace cuda {

void launchGatherRescore(const void* d_corpus, ScalarType dtype, float scale, int doc_count, int dim,
                         const float* d_queries, int batch, const int* d_candidate_indices, int candidate_count,
                         Metric metric, float* d_values, cudaStream_t stream);

void launchRemapIndices(const int* d_candidate_indices, const int* d_local_indices, int candidate_count, int k,
                        int batch, int* d_out_indices, cudaStream_t stream);

std::size_t rescoreSharedBytes(int dim);

}  // namespace cuda
}  // namespace zcgvs
