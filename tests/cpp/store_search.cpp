// Test driver for the C++ drop-in layer's stores (include/zcgvs/): loads or builds an
// EmbeddingStore, optionally a rescore store and a lexical index, runs one Searcher::search and
// writes the [batch, k] ids and scores as raw little-endian arrays for the Python test to check.
//
//   store_search key=value ...
//     corpus=<zcve>              load the corpus with EmbeddingStore::loadFromFile, or
//     host=<raw f32 [n, dim]> n=<rows> dtype=<code> [append=<rows>]
//                                build it with fromHostMatrix from the first n - append rows and
//                                append the rest (exercising growth and per-row scale copies)
//     queries=<raw f32 [batch, dim]> batch=<B> dim=<d> k=<k> metric=<0|1|2>
//     [rescore=<zcve> m=<candidates>] [index=<zcvl> terms=<raw i32 [batch, stride]> stride=<s>
//     weight=<dense weight>] [graph=1]  out=<prefix>  -> <prefix>.ids, <prefix>.scores
//     [cap=<n>]                  lower the tensor-core path's candidate buffer to n entries
//                                (zcgvs_test_set_candidate_cap) for the search; on the
//                                exception it raises, restore the default and search again,
//                                printing "recovered" when the Searcher's next result is clean
// Exit status 0 on success; a thrown exception prints its message and exits 1.
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iostream>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "zcgvs/data/embedding_store.hpp"
#include "zcgvs/data/lexical_index.hpp"
#include "zcgvs/search/searcher.hpp"
#include "zcgvs_sm100.h"

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
void write_raw(const std::string& path, const std::vector<T>& v) {
    std::ofstream out(path, std::ios::binary);
    out.write(reinterpret_cast<const char*>(v.data()), static_cast<std::streamsize>(v.size() * sizeof(T)));
    if (!out) throw std::runtime_error("cannot write " + path);
}

}  // namespace

int main(int argc, char** argv) {
    std::map<std::string, std::string> a;
    for (int i = 1; i < argc; ++i) {
        const std::string s = argv[i];
        const auto eq = s.find('=');
        if (eq != std::string::npos) a[s.substr(0, eq)] = s.substr(eq + 1);
    }
    auto num = [&](const char* key, long long fallback) {
        return a.count(key) ? std::stoll(a[key]) : fallback;
    };
    try {
        const int batch = static_cast<int>(num("batch", 1));
        const int dim = static_cast<int>(num("dim", 0));
        zcgvs::EmbeddingStore store;
        if (a.count("corpus")) {
            store = zcgvs::EmbeddingStore::loadFromFile(a["corpus"]);
        } else {
            const long long n = num("n", 0), extra = num("append", 0);
            const auto host = read_raw<float>(a["host"], static_cast<std::size_t>(n) * dim);
            store = zcgvs::EmbeddingStore::fromHostMatrix(host.data(), n - extra, dim,
                                                          static_cast<zcgvs::ScalarType>(num("dtype", 0)), 0.0f, true);
            if (extra > 0) {
                zcgvs::CudaStream s;
                store.append(host.data() + static_cast<std::size_t>(n - extra) * dim, extra, s.get());
            }
        }
        if (store.dim() != dim) throw std::runtime_error("store dim does not match dim=");
        std::unique_ptr<zcgvs::EmbeddingStore> rescore;
        std::unique_ptr<zcgvs::LexicalIndex> index;
        zcgvs::Searcher searcher(store);
        zcgvs::SearchParams params;
        params.k = static_cast<int>(num("k", 10));
        params.metric = static_cast<zcgvs::Metric>(num("metric", 1));
        params.use_graph = num("graph", 0) != 0;
        if (a.count("rescore")) {
            rescore = std::make_unique<zcgvs::EmbeddingStore>(zcgvs::EmbeddingStore::loadFromFile(a["rescore"]));
            searcher.setRescoreStore(rescore.get());
            params.rescore_candidates = static_cast<int>(num("m", params.k));
        }
        std::vector<int> terms;
        if (a.count("index")) {
            index = std::make_unique<zcgvs::LexicalIndex>(zcgvs::LexicalIndex::loadFromFile(a["index"]));
            searcher.setLexicalIndex(index.get());
            params.lexical_stride = static_cast<int>(num("stride", 0));
            terms = read_raw<int>(a["terms"], static_cast<std::size_t>(batch) * params.lexical_stride);
            params.host_query_terms = terms.data();
            params.dense_weight = std::stof(a.count("weight") ? a["weight"] : "1");
        }
        const auto queries = read_raw<float>(a["queries"], static_cast<std::size_t>(batch) * dim);
        zcgvs::CudaStream stream;
        zcgvs::HostTopK result;
        if (a.count("cap")) {
            if (zcgvs_test_set_candidate_cap(static_cast<int>(num("cap", 0))) != ZCGVS_OK) {
                throw std::runtime_error(zcgvs_last_error_message());
            }
            try {
                searcher.search(queries.data(), dim, batch, params, stream);
                result = searcher.copyResultToHost(stream);
            } catch (const std::runtime_error& e) {
                zcgvs_test_set_candidate_cap(0);
                std::cerr << "store_search: " << e.what() << "\n";
                searcher.search(queries.data(), dim, batch, params, stream);
                result = searcher.copyResultToHost(stream);
                std::printf("recovered\n");
                write_raw(a["out"] + ".ids", result.indices);
                write_raw(a["out"] + ".scores", result.scores);
                return 1;
            }
            zcgvs_test_set_candidate_cap(0);
        }
        for (int pass = 0; pass < (params.use_graph ? 3 : 1); ++pass) {  // capture, then replays
            searcher.search(queries.data(), dim, batch, params, stream);
            result = searcher.copyResultToHost(stream);
        }
        write_raw(a["out"] + ".ids", result.indices);
        write_raw(a["out"] + ".scores", result.scores);
        std::printf("docs=%lld dtype=%d row_scales=%d graph_launches=%llu\n", static_cast<long long>(store.docCount()),
                    static_cast<int>(store.dtype()), store.rowScales() != nullptr ? 1 : 0,
                    static_cast<unsigned long long>(searcher.graphLaunchCount()));
    } catch (const std::exception& e) {
        std::cerr << "store_search: " << e.what() << "\n";
        return 1;
    }
    return 0;
}
