// End-to-end query rate through the C++ drop-in layer: the call sequence a reference caller runs
// per query (src/search/searcher.cpp:344-397), Searcher::search on a host query followed by
// Searcher::copyResultToHost, timed on the host clock around `steps` back-to-back queries after
// `warmup` ones. Each search copies the query into the Searcher's pinned staging, uploads it,
// runs the search (a CUDA graph replay once captured, as the reference's Searcher serves) and
// copyResultToHost synchronises and downloads the [1, k] ids and scores.
//
//   searcher_e2e docs=<N> dim=<d> dtype=<0 f32|1 f16|2 i8|4 i8 per row> k=<k> metric=<0|1|2>
//                [queries=<pool size>] [steps=<S>] [warmup=<W>] [seed=<s>] [graph=<0|1>]
//                [vocab=<V> mean_len=<L> terms=<max terms> weight=<w>]   (hybrid: a synthetic
//                 BM25 index, Zipf(1.1) terms over V, L term draws per document)
//
// The corpus and queries are seeded, approximately normal rows normalised to unit length
// (converted to the storage dtype on the device by EmbeddingStore::fromHostMatrix). Prints one
// JSON line.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

#include "zcgvs/core/cuda_stream.hpp"
#include "zcgvs/data/embedding_store.hpp"
#include "zcgvs/data/lexical_index.hpp"
#include "zcgvs/search/searcher.hpp"

namespace {

// splitmix64 stream; normals from the sum of four 16-bit uniforms (Irwin-Hall, variance
// matched): seeded, a few nanoseconds a value, which a gigabyte-sized corpus needs.
struct Rng {
    std::uint64_t s;
    std::uint64_t next() {
        std::uint64_t z = (s += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    }
    double uniform() { return (static_cast<double>(next() >> 11) + 0.5) * (1.0 / 9007199254740992.0); }
    float normal() {
        const std::uint64_t z = next();
        const double sum = static_cast<double>(z & 0xFFFF) + static_cast<double>((z >> 16) & 0xFFFF) +
                           static_cast<double>((z >> 32) & 0xFFFF) + static_cast<double>(z >> 48);
        return static_cast<float>((sum - 2.0 * 65535.0) * (1.0 / 37837.0));  // sd of the sum: 65536 / sqrt(3)
    }
};

void normal_rows(std::vector<float>& out, std::int64_t rows, int dim, std::uint64_t seed) {
    out.resize(static_cast<std::size_t>(rows) * dim);
    Rng rng{seed};
    for (std::int64_t r = 0; r < rows; ++r) {
        float* row = out.data() + static_cast<std::size_t>(r) * dim;
        double ss = 0.0;
        for (int j = 0; j < dim; ++j) {
            row[j] = rng.normal();
            ss += static_cast<double>(row[j]) * row[j];
        }
        const float inv = static_cast<float>(1.0 / std::sqrt(ss));
        for (int j = 0; j < dim; ++j) row[j] *= inv;
    }
}

long arg(const std::map<std::string, std::string>& a, const char* key, long fallback) {
    const auto it = a.find(key);
    return it == a.end() ? fallback : std::stol(it->second);
}

}  // namespace

int main(int argc, char** argv) {
    std::map<std::string, std::string> a;
    for (int i = 1; i < argc; ++i) {
        const std::string s = argv[i];
        const auto eq = s.find('=');
        if (eq != std::string::npos) a[s.substr(0, eq)] = s.substr(eq + 1);
    }
    try {
        const std::int64_t docs = arg(a, "docs", 1000000);
        const int dim = static_cast<int>(arg(a, "dim", 768));
        const auto dtype = static_cast<zcgvs::ScalarType>(arg(a, "dtype", 4));
        const int k = static_cast<int>(arg(a, "k", 100));
        const int metric = static_cast<int>(arg(a, "metric", 0));
        const int pool = static_cast<int>(arg(a, "queries", 256));
        const int steps = static_cast<int>(arg(a, "steps", 1000));
        const int warmup = static_cast<int>(arg(a, "warmup", 20));
        const std::uint64_t seed = static_cast<std::uint64_t>(arg(a, "seed", 7001));
        const long vocab = arg(a, "vocab", 0);

        std::vector<float> host;
        normal_rows(host, docs, dim, seed);
        zcgvs::EmbeddingStore store = zcgvs::EmbeddingStore::fromHostMatrix(host.data(), docs, dim, dtype, 0.0f, true);
        std::vector<float>().swap(host);
        std::vector<float> queries;
        normal_rows(queries, pool, dim, seed + 1);

        zcgvs::Searcher searcher(store);
        zcgvs::SearchParams params;
        params.k = k;
        params.metric = static_cast<zcgvs::Metric>(metric);
        params.use_graph = arg(a, "graph", 1) != 0;

        // Hybrid: a seeded CSR index (Zipf(1.1) term ranks, mean_len term draws per document,
        // sorted postings) and per-query term lists.
        zcgvs::LexicalIndex index;
        std::vector<int> terms;
        int stride = 0;
        if (vocab > 0) {
            const long mean_len = arg(a, "mean_len", 100);
            stride = static_cast<int>(arg(a, "terms", 12));
            std::vector<double> cdf(static_cast<std::size_t>(vocab));
            double acc = 0.0;
            for (long t = 0; t < vocab; ++t) cdf[t] = (acc += std::pow(static_cast<double>(t + 1), -1.1));
            for (double& c : cdf) c /= acc;
            // Inverse CDF tabulated at 2^20 points: one lookup per draw.
            constexpr int kTableBits = 20;
            std::vector<int> table(std::size_t{1} << kTableBits);
            for (std::size_t i = 0; i < table.size(); ++i) {
                const double u = (static_cast<double>(i) + 0.5) / static_cast<double>(table.size());
                table[i] = std::min<int>(static_cast<int>(std::lower_bound(cdf.begin(), cdf.end(), u) - cdf.begin()),
                                         static_cast<int>(vocab - 1));
            }
            Rng rng{seed + 2};
            auto draw = [&]() { return table[rng.next() >> (64 - kTableBits)]; };
            std::vector<std::vector<int>> lists(static_cast<std::size_t>(vocab));
            std::vector<int> seen;
            for (std::int64_t d = 0; d < docs; ++d) {
                seen.clear();
                for (long j = 0; j < mean_len; ++j) seen.push_back(draw());
                std::sort(seen.begin(), seen.end());
                seen.erase(std::unique(seen.begin(), seen.end()), seen.end());
                for (int t : seen) lists[t].push_back(static_cast<int>(d));
            }
            std::vector<std::int64_t> offsets(static_cast<std::size_t>(vocab) + 1, 0);
            std::vector<int> pdocs;
            std::vector<float> weights;
            for (long t = 0; t < vocab; ++t) {
                const double idf = std::log(1.0 + (static_cast<double>(docs) - lists[t].size() + 0.5) /
                                                      (lists[t].size() + 0.5));
                for (int d : lists[t]) {
                    pdocs.push_back(d);
                    weights.push_back(static_cast<float>(idf * (0.5 + rng.uniform())));
                }
                offsets[t + 1] = static_cast<std::int64_t>(pdocs.size());
            }
            index = zcgvs::LexicalIndex::fromHostCsr(offsets.data(), static_cast<int>(vocab), pdocs.data(), weights.data(),
                                                     docs);
            searcher.setLexicalIndex(&index);
            terms.assign(static_cast<std::size_t>(pool) * stride, -1);
            for (int q = 0; q < pool; ++q) {
                const int n = 3 + static_cast<int>(rng.next() % static_cast<std::uint64_t>(std::max(1, stride - 2)));
                for (int j = 0; j < n && j < stride; ++j) terms[static_cast<std::size_t>(q) * stride + j] = draw();
            }
            params.lexical_stride = stride;
            params.dense_weight = static_cast<float>(std::stod(a.count("weight") ? a["weight"] : "0.5"));
        }

        zcgvs::CudaStream stream;
        auto one = [&](int i) {
            const int q = i % pool;
            if (stride > 0) params.host_query_terms = terms.data() + static_cast<std::size_t>(q) * stride;
            searcher.search(queries.data() + static_cast<std::size_t>(q) * dim, dim, 1, params, stream);
            return searcher.copyResultToHost(stream);
        };
        for (int i = 0; i < warmup; ++i) one(i);
        double gpu_ms = 0.0;
        const auto t0 = std::chrono::steady_clock::now();
        for (int i = 0; i < steps; ++i) {
            one(warmup + i);
            gpu_ms += searcher.lastSearchGpuMs();
        }
        const auto t1 = std::chrono::steady_clock::now();
        const double seconds = std::chrono::duration<double>(t1 - t0).count();
        std::printf("{\"queries_per_s\": %.3f, \"ms_per_query\": %.6f, \"steps\": %d, \"warmup\": %d, "
                    "\"graph\": %s, \"search_gpu_ms_mean\": %.6f, \"h2d_bytes_per_step\": %d, "
                    "\"d2h_bytes_per_step\": %d}\n",
                    steps / seconds, seconds * 1e3 / steps, steps, warmup, searcher.lastSearchUsedGraph() ? "true" : "false",
                    gpu_ms / steps, dim * 4 + stride * 4, k * 8);
        return 0;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "searcher_e2e: %s\n", e.what());
        return 1;
    }
}
