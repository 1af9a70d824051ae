// ref_cpu_capi.cpp - C entry points over the reference's own CPU search code.
// TEST / BASELINE INFRASTRUCTURE ONLY.
//
// Compiled by oracle/Makefile against the read-only reference header
// tests/cpp/cpu_reference.hpp (found through -I, never copied) into oracle/_ref/. It gives the
// tests the reference's CPU outputs to pin the oracle against, and bench.py the reference CPU
// path (cpuCosineSimilarity + cpuTopKIndices, tests/cpp/cpu_reference.hpp:12-34) to time.
#include <algorithm>
#include <chrono>
#include <cstddef>
#include <cstdint>
#include <thread>
#include <vector>

#include "cpu_reference.hpp"

namespace {

using zcgvs::testing::cpuCosineSimilarity;
using zcgvs::testing::cpuTopKIndices;

}  // namespace

extern "C" {

// Scores of `batch` queries against a float32 corpus: cpuCosineSimilarity per query.
void refcpu_scores(const float* corpus, int doc_count, int dim, const float* queries, int batch,
                   float* out) {
    const std::vector<float> matrix(corpus, corpus + static_cast<size_t>(doc_count) * dim);
    for (int q = 0; q < batch; ++q) {
        const std::vector<float> query(queries + static_cast<size_t>(q) * dim,
                                       queries + static_cast<size_t>(q + 1) * dim);
        const std::vector<float> s = cpuCosineSimilarity(matrix, doc_count, dim, query);
        std::copy(s.begin(), s.end(), out + static_cast<size_t>(q) * doc_count);
    }
}

// Top-k indices of each score row: cpuTopKIndices (stable sort, ties to the lower index).
void refcpu_topk(const float* scores, int doc_count, int batch, int k, int* out) {
    for (int q = 0; q < batch; ++q) {
        const std::vector<float> s(scores + static_cast<size_t>(q) * doc_count,
                                   scores + static_cast<size_t>(q + 1) * doc_count);
        const std::vector<int> idx = cpuTopKIndices(s, k);
        std::copy(idx.begin(), idx.end(), out + static_cast<size_t>(q) * k);
    }
}

void refcpu_quantize_dequantize_i8(const float* values, size_t count, float scale, float* out) {
    const std::vector<float> v(values, values + count);
    const std::vector<float> r = zcgvs::testing::cpuQuantizeDequantizeInt8(v, scale);
    std::copy(r.begin(), r.end(), out);
}

void refcpu_pack_binary(const float* matrix, int rows, int dim, uint32_t* out) {
    const std::vector<float> m(matrix, matrix + static_cast<size_t>(rows) * dim);
    const std::vector<uint32_t> p = zcgvs::testing::cpuPackBinary(m, rows, dim);
    std::copy(p.begin(), p.end(), out);
}

int refcpu_hamming(const uint32_t* a, const uint32_t* b, int words) {
    return zcgvs::testing::cpuHamming(a, b, words);
}

void refcpu_l2_normalize(float* vector, int dim) {
    std::vector<float> v(vector, vector + dim);
    zcgvs::testing::l2Normalize(v, 0, dim);
    std::copy(v.begin(), v.end(), vector);
}

// The reference CPU search path timed by bench.py: for every query, cpuCosineSimilarity over
// the whole float32 corpus and cpuTopKIndices(k). Queries are split across `threads` host
// threads; each query is the reference's sequential code. Writes top-k ids and returns the
// wall time in seconds.
double refcpu_search(const float* corpus, int doc_count, int dim, const float* queries,
                     int batch, int k, int threads, int* out) {
    const std::vector<float> matrix(corpus, corpus + static_cast<size_t>(doc_count) * dim);
    threads = std::max(1, std::min(threads, batch));
    const auto start = std::chrono::steady_clock::now();
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t) {
        pool.emplace_back([&, t]() {
            for (int q = t; q < batch; q += threads) {
                const std::vector<float> query(queries + static_cast<size_t>(q) * dim,
                                               queries + static_cast<size_t>(q + 1) * dim);
                const std::vector<float> s = cpuCosineSimilarity(matrix, doc_count, dim, query);
                const std::vector<int> idx = cpuTopKIndices(s, k);
                std::copy(idx.begin(), idx.end(), out + static_cast<size_t>(q) * k);
            }
        });
    }
    for (std::thread& th : pool) th.join();
    const auto end = std::chrono::steady_clock::now();
    return std::chrono::duration<double>(end - start).count();
}

}  // extern "C"
