// Test driver for the C++ ShardedSearcher (include/zcgvs/search/sharded_searcher.hpp): one
// process per rank. Rank 0 writes an NCCL id to `id=<file>`, the other ranks wait for it; each
// rank converts its rows of a host fp32 corpus into its shard store (and rescore store), runs
// the search `passes` times (with use_graph, the first captures and the rest replay) and writes
// the global [batch, k] ids and scores of the last pass.
//
//   sharded_search id=<file> world=<P> rank=<r> host=<raw f32 [n, dim]> n=<rows> dim=<d>
//                  dtype=<code> queries=<raw f32 [batch, dim]> batch=<B> k=<k> metric=<m>
//                  [rescore_dtype=<code> m=<candidates>] [graph=1 passes=<n>] out=<prefix>
// Exit status 0 on success; a thrown exception prints its message and exits 1.
#include <chrono>
#include <cstdio>
#include <fstream>
#include <iostream>
#include <iterator>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "zcgvs/core/cuda_context.hpp"
#include "zcgvs/data/embedding_store.hpp"
#include "zcgvs/search/sharded_searcher.hpp"

namespace {

template <typename T>
std::vector<T> read_raw(const std::string& path, std::size_t count, std::size_t offset = 0) {
    std::ifstream in(path, std::ios::binary);
    in.seekg(static_cast<std::streamoff>(offset * sizeof(T)));
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

// Rank 0 writes the id (to a temporary name, then renamed); the others poll for up to a minute.
std::vector<char> exchange_id(const std::string& path, int rank) {
    if (rank == 0) {
        const std::vector<char> id = zcgvs::ShardedSearcher::uniqueId();
        write_raw(path + ".tmp", id);
        if (std::rename((path + ".tmp").c_str(), path.c_str()) != 0) throw std::runtime_error("cannot publish the id");
        return id;
    }
    for (int i = 0; i < 600; ++i) {
        std::ifstream in(path, std::ios::binary);
        if (in) {
            std::vector<char> id((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
            if (!id.empty()) return id;
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(100));
    }
    throw std::runtime_error("rank 0 did not publish the NCCL id");
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
        const int world = static_cast<int>(num("world", 1));
        const int rank = static_cast<int>(num("rank", 0));
        const long long n = num("n", 0);
        const int dim = static_cast<int>(num("dim", 0));
        const int batch = static_cast<int>(num("batch", 1));
        zcgvs::setDevice(static_cast<int>(num("device", rank)));
        const std::vector<char> id = exchange_id(a["id"], rank);
        zcgvs::ShardedSearcher searcher(id, world, rank, n);
        const long long begin = searcher.shardBegin(), rows = searcher.shardEnd() - searcher.shardBegin();
        const auto host = read_raw<float>(a["host"], static_cast<std::size_t>(rows) * dim,
                                          static_cast<std::size_t>(begin) * dim);
        const auto shard = zcgvs::EmbeddingStore::fromHostMatrix(
            host.data(), rows, dim, static_cast<zcgvs::ScalarType>(num("dtype", 0)), 0.0f, true);
        std::unique_ptr<zcgvs::EmbeddingStore> fine;
        zcgvs::SearchParams params;
        params.k = static_cast<int>(num("k", 10));
        params.metric = static_cast<zcgvs::Metric>(num("metric", 1));
        params.use_graph = num("graph", 0) != 0;
        if (a.count("rescore_dtype")) {
            fine = std::make_unique<zcgvs::EmbeddingStore>(zcgvs::EmbeddingStore::fromHostMatrix(
                host.data(), rows, dim, static_cast<zcgvs::ScalarType>(num("rescore_dtype", 1)), 0.0f, true));
            searcher.setRescoreStore(fine.get());
            params.rescore_candidates = static_cast<int>(num("m", params.k));
        }
        const auto queries = read_raw<float>(a["queries"], static_cast<std::size_t>(batch) * dim);
        zcgvs::CudaStream stream;
        zcgvs::HostTopK result;
        for (long long pass = 0; pass < num("passes", 1); ++pass) {
            searcher.search(shard, queries.data(), dim, batch, params, stream);
            result = searcher.copyResultToHost(stream);
        }
        write_raw(a["out"] + ".ids", result.indices);
        write_raw(a["out"] + ".scores", result.scores);
        std::printf("rank=%d shard=[%lld,%lld)\n", rank, begin, begin + rows);
    } catch (const std::exception& e) {
        std::cerr << "sharded_search: " << e.what() << "\n";
        return 1;
    }
    return 0;
}
