// One device-side search request (the reference's SearchParams,
// include/zcgvs/search/search_params.hpp:24-46).
#pragma once

#include <cstdint>

#include "zcgvs/core/metric.hpp"

namespace zcgvs {

// Who computes the scores. Both names are kept for configuration compatibility; this library
// always runs its fused kernels (there is no separate cuBLAS score matrix).
enum class SimilarityBackend : std::int32_t { Custom = 0, Cublas = 1 };

inline const char* similarityBackendName(SimilarityBackend backend) {
    return backend == SimilarityBackend::Cublas ? "cublas" : "custom";
}

struct SearchParams {
    int k = 10;
    Metric metric = Metric::Cosine;
    // Optional [doc_count] uint8 allow-mask on the device; 0 excludes a document.
    const std::uint8_t* d_mask = nullptr;
    // With a rescore store attached: the coarse scan keeps this many candidates and the exact
    // store rescores them to k.
    int rescore_candidates = 0;
    // Flattened [batch, lexical_stride] term ids on the host, -1 padded (lexical index attached).
    const int* host_query_terms = nullptr;
    int lexical_stride = 0;
    // Weight of the dense score in the hybrid blend; 1 is dense only.
    float dense_weight = 1.0f;
    SimilarityBackend backend = SimilarityBackend::Custom;
    bool use_graph = false;
};

}  // namespace zcgvs
