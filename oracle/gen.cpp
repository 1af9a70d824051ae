// gen.cpp - seeded input generators for the oracle and the tests. TEST INFRASTRUCTURE ONLY.
//
// The reference harnesses draw their inputs with std::mt19937 and the standard library
// distributions (e.g. tests/cpp/test_pipeline.cu:20-31, tests/cpp/test_topk.cu:14-20) and
// normalise rows with a sequential fp32 sum (tests/cpp/cpu_reference.hpp:36-49). Using the same
// standard-library engine and distributions here reproduces those inputs bit for bit, so the
// Python tests can run the reference's own cases.
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <random>

#include "oracle.h"

extern "C" void orc_gen_normal_rows(int64_t rows, int dim, uint32_t seed, int normalize, float* out) {
    std::mt19937 rng(seed);
    std::normal_distribution<float> distribution(0.0f, 1.0f);
    for (int64_t r = 0; r < rows; ++r) {
        float* row = out + static_cast<size_t>(r) * static_cast<size_t>(dim);
        for (int j = 0; j < dim; ++j) row[j] = distribution(rng);
        if (!normalize) continue;
        float norm = 0.0f;
        for (int j = 0; j < dim; ++j) norm += row[j] * row[j];
        norm = std::sqrt(norm);
        if (norm <= 0.0f) continue;
        for (int j = 0; j < dim; ++j) row[j] /= norm;
    }
}

extern "C" void orc_gen_uniform(size_t count, uint32_t seed, float lo, float hi, float* out) {
    std::mt19937 rng(seed);
    std::uniform_real_distribution<float> distribution(lo, hi);
    for (size_t i = 0; i < count; ++i) out[i] = distribution(rng);
}

// The synthetic inverted index and query of tests/cpp/test_lexical.cu:31-67: for every term a
// U{0..max_postings} posting count, documents U{0..doc_count-1} (unsorted, repeats possible) and
// weights U[wlo, whi) from std::mt19937(index_seed); then term_count query terms
// U{0..vocab-1} from std::mt19937(query_seed) with the last slot set to -1, followed by
// doc_count dense scores U[-1, 1) from the same engine. Two-phase: call with docs == NULL to
// get the posting count in *nnz, then again with buffers.
extern "C" void orc_gen_lexical_test(uint32_t index_seed, int doc_count, int vocab, int max_postings, float wlo,
                                     float whi, uint32_t query_seed, int term_count, int64_t* offsets, int32_t* docs,
                                     float* weights, int64_t* nnz, int32_t* terms, float* dense) {
    std::mt19937 rng(index_seed);
    std::uniform_int_distribution<int> postings_per_term(0, max_postings);
    std::uniform_int_distribution<int> doc_picker(0, doc_count - 1);
    std::uniform_real_distribution<float> weight_picker(wlo, whi);
    int64_t total = 0;
    if (offsets != nullptr) offsets[0] = 0;
    for (int term = 0; term < vocab; ++term) {
        const int count = postings_per_term(rng);
        for (int i = 0; i < count; ++i) {
            const int doc = doc_picker(rng);
            const float w = weight_picker(rng);
            if (docs != nullptr) {
                docs[total] = doc;
                weights[total] = w;
            }
            ++total;
        }
        if (offsets != nullptr) offsets[term + 1] = total;
    }
    *nnz = total;
    if (terms == nullptr) return;
    std::mt19937 qrng(query_seed);
    std::uniform_int_distribution<int> term_picker(0, vocab - 1);
    std::uniform_real_distribution<float> dense_picker(-1.0f, 1.0f);
    for (int t = 0; t < term_count; ++t) terms[t] = term_picker(qrng);
    terms[term_count - 1] = -1;
    for (int i = 0; i < doc_count; ++i) dense[i] = dense_picker(qrng);
}
