// CublasSimilarity: the reference's cuBLAS yardstick (src/cuda/cublas_similarity.cpp:15-50),
// built into libzcgvs_cublas.so, apart from the search library.
//
// cuBLAS is column-major. The row-major [doc_count, dim] corpus is the column-major [dim,
// doc_count] matrix C with leading dimension dim, and the queries likewise Q = [dim, batch].
// C^T Q is then the column-major [doc_count, batch] matrix, i.e. the row-major [batch,
// doc_count] score matrix the reference's top-k reads.
#include "zcgvs/cuda/cublas_similarity.hpp"

#include "zcgvs/core/cublas_check.hpp"

namespace zcgvs {

CublasSimilarity::CublasSimilarity() { ZCGVS_CUBLAS_CHECK(cublasCreate(&handle_)); }

CublasSimilarity::~CublasSimilarity() {
    if (handle_ != nullptr) cublasDestroy(handle_);
}

bool CublasSimilarity::supports(ScalarType dtype, Metric metric, bool has_mask) {
    return !has_mask && dtype == ScalarType::Float32 && (metric == Metric::Cosine || metric == Metric::DotProduct);
}

void CublasSimilarity::run(const float* d_corpus, int doc_count, int dim, const float* d_queries, int batch,
                           float* d_scores, cudaStream_t stream) {
    if (doc_count <= 0 || dim <= 0 || batch <= 0) return;
    ZCGVS_CUBLAS_CHECK(cublasSetStream(handle_, stream));
    const float one = 1.0f, zero = 0.0f;
    if (batch == 1) {
        ZCGVS_CUBLAS_CHECK(
            cublasSgemv(handle_, CUBLAS_OP_T, dim, doc_count, &one, d_corpus, dim, d_queries, 1, &zero, d_scores, 1));
    } else {
        ZCGVS_CUBLAS_CHECK(cublasSgemm(handle_, CUBLAS_OP_T, CUBLAS_OP_N, doc_count, batch, dim, &one, d_corpus, dim,
                                       d_queries, dim, &zero, d_scores, doc_count));
    }
}

}  // namespace zcgvs
