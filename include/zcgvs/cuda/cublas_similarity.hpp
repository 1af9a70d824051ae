// The vendor-library yardstick of the reference (include/zcgvs/cuda/cublas_similarity.hpp:14-36,
// src/cuda/cublas_similarity.cpp:15-50): the fp32 [batch, doc_count] inner-product score matrix
// as a cuBLAS GEMV (batch 1) or GEMM, for benchmarking the scan kernels against a library
// baseline. It is not on the search path: the Searcher never calls it. It lives in its own
// library, libzcgvs_cublas.so (csrc/yardstick/), so the search library does not depend on
// cuBLAS; a program that uses it links -lzcgvs_cublas -lcublas.
#pragma once

#include <cublas_v2.h>
#include <cuda_runtime.h>

#include "zcgvs/core/metric.hpp"
#include "zcgvs/core/scalar_type.hpp"

namespace zcgvs {

class CublasSimilarity {
public:
    CublasSimilarity();
    ~CublasSimilarity();

    CublasSimilarity(const CublasSimilarity&) = delete;
    CublasSimilarity& operator=(const CublasSimilarity&) = delete;

    // A GEMM scores fp32 rows by inner product (cosine of normalised rows) and has no mask:
    // everything else goes to the library's kernels.
    static bool supports(ScalarType dtype, Metric metric, bool has_mask);

    // scores[q, i] = <queries[q], corpus[i]> for a row-major [doc_count, dim] fp32 corpus and
    // [batch, dim] fp32 queries, on `stream`. Zero-sized problems do nothing.
    void run(const float* d_corpus, int doc_count, int dim, const float* d_queries, int batch, float* d_scores,
             cudaStream_t stream);

private:
    cublasHandle_t handle_ = nullptr;
};

}  // namespace zcgvs
