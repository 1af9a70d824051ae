// Test driver for zcgvs::VectorEngine (include/zcgvs/engine/vector_engine.hpp): builds the stores
// on the device from a host fp32 matrix, optionally a rescore store and a lexical index from raw
// CSR files, runs searchBatch `repeat` times and writes the last result for the Python test.
//
//   engine_search key=value ...
//     corpus=<raw f32 [n, dim]> n=<rows> dim=<d> dtype=<code> queries=<raw f32 [batch, dim]> batch=<B>
//     [rescore_dtype=<code>] [offsets=<raw i64 [vocab+1]> docs=<raw i32> weights=<raw f32> vocab=<V>
//      terms=<raw i32: per query a count, then that many encoded ids>]
//     [top_k=] [candidates=] [rescore=] [weight=] [hybrid=1] [graph=1] [metric=] [allow=<raw i32 list>
//      allow_n=<count>] [repeat=<searches>] out=<prefix>
//   -> <prefix>.ids / <prefix>.scores: [batch, top_k] (-1 / 0 past a query's hits), and one line
//      of stats on stdout. A thrown exception prints its message and exits 1.
#include <cstdint>
#include <cstdio>
#include <fstream>
#include <iostream>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "zcgvs/engine/vector_engine.hpp"

namespace {

template <typename T>
std::vector<T> read_raw(const std::string& path, std::size_t count) {
    std::ifstream in(path, std::ios::binary);
    std::vector<T> v(count);
    in.read(reinterpret_cast<char*>(v.data()), static_cast<std::streamsize>(count * sizeof(T)));
    if (!in) throw std::runtime_error("cannot read " + path);
    return v;
}

template <typename T>
std::vector<T> read_all(const std::string& path) {
    std::ifstream in(path, std::ios::binary | std::ios::ate);
    if (!in) throw std::runtime_error("cannot read " + path);
    const auto bytes = static_cast<std::size_t>(in.tellg());
    in.seekg(0);
    std::vector<T> v(bytes / sizeof(T));
    in.read(reinterpret_cast<char*>(v.data()), static_cast<std::streamsize>(v.size() * sizeof(T)));
    return v;
}

}  // namespace

int main(int argc, char** argv) {
    std::map<std::string, std::string> a;
    for (int i = 1; i < argc; ++i) {
        const std::string s = argv[i];
        const auto eq = s.find('=');
        if (eq != std::string::npos) a[s.substr(0, eq)] = s.substr(eq + 1);
    }
    auto num = [&](const char* key, long long fallback) { return a.count(key) ? std::stoll(a[key]) : fallback; };
    try {
        const long long n = num("n", 0);
        const int dim = static_cast<int>(num("dim", 0));
        const int batch = static_cast<int>(num("batch", 1));
        const auto host = read_raw<float>(a["corpus"], static_cast<std::size_t>(n) * dim);
        const auto store = zcgvs::EmbeddingStore::fromHostMatrix(host.data(), n, dim,
                                                                 static_cast<zcgvs::ScalarType>(num("dtype", 0)), 0.0f, true);
        std::unique_ptr<zcgvs::EmbeddingStore> rescore;
        if (a.count("rescore_dtype")) {
            rescore = std::make_unique<zcgvs::EmbeddingStore>(zcgvs::EmbeddingStore::fromHostMatrix(
                host.data(), n, dim, static_cast<zcgvs::ScalarType>(num("rescore_dtype", 1)), 0.0f, true));
        }
        std::unique_ptr<zcgvs::LexicalIndex> index;
        std::vector<std::vector<int>> encoded;
        if (a.count("offsets")) {
            const int vocab = static_cast<int>(num("vocab", 0));
            const auto offsets = read_raw<std::int64_t>(a["offsets"], static_cast<std::size_t>(vocab) + 1);
            const auto docs = read_all<int>(a["docs"]);
            const auto weights = read_all<float>(a["weights"]);
            index = std::make_unique<zcgvs::LexicalIndex>(
                zcgvs::LexicalIndex::fromHostCsr(offsets.data(), vocab, docs.data(), weights.data(), n, 0.9f, 0.4f, 200.0f));
            const auto flat = read_all<int>(a["terms"]);
            for (std::size_t i = 0; i < flat.size();) {
                const int count = flat[i++];
                encoded.emplace_back(flat.begin() + static_cast<std::ptrdiff_t>(i),
                                     flat.begin() + static_cast<std::ptrdiff_t>(i + count));
                i += static_cast<std::size_t>(count);
            }
        }
        zcgvs::VectorEngineConfig config;
        config.use_cuda_graphs = num("graph", 0) != 0;
        config.metric = static_cast<zcgvs::Metric>(num("metric", 0));
        zcgvs::VectorEngine engine(store, config, rescore.get(), index.get());
        zcgvs::SearchOptions options = engine.defaultOptions();
        options.top_k = static_cast<int>(num("top_k", 10));
        options.candidates = static_cast<int>(num("candidates", 100));
        options.rescore_candidates = static_cast<int>(num("rescore", 0));
        options.dense_weight = a.count("weight") ? std::stof(a["weight"]) : -1.0f;
        options.hybrid = num("hybrid", 0) != 0;
        if (a.count("allow")) options.allow = read_raw<int>(a["allow"], static_cast<std::size_t>(num("allow_n", 0)));
        const auto queries = read_raw<float>(a["queries"], static_cast<std::size_t>(batch) * dim);
        zcgvs::BatchSearchResponse response;
        for (long long r = 0; r < num("repeat", 1); ++r) response = engine.searchBatch(queries.data(), batch, options, encoded);
        const int top_k = options.top_k;
        std::vector<int> ids(static_cast<std::size_t>(batch) * top_k, -1);
        std::vector<float> scores(static_cast<std::size_t>(batch) * top_k, 0.0f);
        for (int q = 0; q < batch; ++q) {
            const auto& hits = response.results[static_cast<std::size_t>(q)];
            for (std::size_t i = 0; i < hits.size() && static_cast<int>(i) < top_k; ++i) {
                ids[static_cast<std::size_t>(q) * top_k + i] = hits[i].corpus_index;
                scores[static_cast<std::size_t>(q) * top_k + i] = hits[i].similarity;
            }
        }
        std::ofstream(a["out"] + ".ids", std::ios::binary)
            .write(reinterpret_cast<const char*>(ids.data()), static_cast<std::streamsize>(ids.size() * sizeof(int)));
        std::ofstream(a["out"] + ".scores", std::ios::binary)
            .write(reinterpret_cast<const char*>(scores.data()), static_cast<std::streamsize>(scores.size() * sizeof(float)));
        const zcgvs::EngineStats s = engine.stats();
        std::printf("corpus=%lld dim=%d dtype=%s rescore=%s lexical=%lld captures=%llu launches=%llu graph=%d major=%d hits0=%zu\n",
                    static_cast<long long>(s.corpus_size), s.dim, s.storage_dtype.c_str(),
                    s.has_rescore_store ? s.rescore_dtype.c_str() : "-", static_cast<long long>(s.lexical_postings),
                    static_cast<unsigned long long>(s.graph_captures), static_cast<unsigned long long>(s.graph_launches),
                    response.timing.graph_replay ? 1 : 0, s.compute_major, response.results.front().size());
    } catch (const std::exception& e) {
        std::cerr << "engine_search: " << e.what() << "\n";
        return 1;
    }
    return 0;
}
