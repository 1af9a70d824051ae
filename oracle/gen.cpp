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
