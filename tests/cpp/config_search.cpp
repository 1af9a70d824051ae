// Test driver for the JSON config loader (include/zcgvs/engine/config_loader.hpp).
//
//   config_search dump=<json file> [roots=<dir>,<dir>...]
//       parses the file's text (configFromJsonText with those search roots; no roots: paths
//       are kept as written) and prints every field as key=value, one per line;
//   config_search file=<json file>
//       the same through configFromJsonFile (roots: the file's directory and its parent);
//   config_search config=<json file> queries=<raw f32 [batch, dim]> batch=<B> out=<prefix>
//       loads the stores the config names (embeddings_path, optional rescore_embeddings_path),
//       builds a VectorEngine from its search fields and runs searchBatch with the config's
//       default options, writing <prefix>.ids / <prefix>.scores [batch, default_top_k].
// An exception prints "error: <message>" on stderr and exits 2.
#include <cstdio>
#include <fstream>
#include <iostream>
#include <map>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "zcgvs/engine/config_loader.hpp"

namespace {

void dump(const zcgvs::EngineConfig& c) {
    auto s = [](const char* k, const std::string& v) { std::printf("%s=%s\n", k, v.c_str()); };
    auto i = [](const char* k, long long v) { std::printf("%s=%lld\n", k, v); };
    s("embeddings_path", c.embeddings_path);
    s("metadata_path", c.metadata_path);
    s("vocab_path", c.vocab_path);
    s("rescore_embeddings_path", c.rescore_embeddings_path);
    s("lexical_index_path", c.lexical_index_path);
    s("encoder_model_path", c.encoder_model_path);
    s("encoder_output_name", c.encoder_output_name);
    i("encoder_max_seq_len", c.encoder_max_seq_len);
    s("reranker_backend", "onnx");
    s("reranker_model_path", c.reranker_model_path);
    s("reranker_output_name", c.reranker_output_name);
    i("reranker_max_seq_len", c.reranker_max_seq_len);
    i("reranker_batch_size", c.reranker_batch_size);
    i("device_id", c.device_id);
    i("lowercase", c.lowercase);
    s("metric", c.metric == zcgvs::Metric::Cosine ? "Cosine" : c.metric == zcgvs::Metric::DotProduct ? "DotProduct" : "L2");
    s("similarity_backend", c.similarity_backend == zcgvs::SimilarityBackend::Cublas ? "Cublas" : "Custom");
    i("default_top_k", c.default_top_k);
    i("default_candidates", c.default_candidates);
    i("rescore_candidates", c.rescore_candidates);
    i("hybrid", c.hybrid);
    std::printf("dense_weight=%.9g\n", static_cast<double>(c.dense_weight));
    i("max_query_terms", c.max_query_terms);
    i("use_cuda_graphs", c.use_cuda_graphs);
}

std::string slurp(const std::string& path) {
    std::ifstream in(path, std::ios::binary);
    if (!in) throw std::runtime_error("cannot read " + path);
    std::ostringstream text;
    text << in.rdbuf();
    return text.str();
}

}  // namespace

int main(int argc, char** argv) {
    std::map<std::string, std::string> a;
    for (int k = 1; k < argc; ++k) {
        const std::string s = argv[k];
        const auto eq = s.find('=');
        if (eq != std::string::npos) a[s.substr(0, eq)] = s.substr(eq + 1);
    }
    try {
        if (a.count("dump")) {
            std::vector<std::string> roots;
            std::stringstream list(a["roots"]);
            for (std::string r; std::getline(list, r, ',');) {
                if (!r.empty()) roots.push_back(r);
            }
            dump(zcgvs::configFromJsonText(slurp(a["dump"]), roots));
            return 0;
        }
        if (a.count("file")) {
            dump(zcgvs::configFromJsonFile(a["file"]));
            return 0;
        }
        const zcgvs::EngineConfig config = zcgvs::configFromJsonFile(a["config"]);
        const auto store = zcgvs::EmbeddingStore::loadFromFile(config.embeddings_path);
        std::unique_ptr<zcgvs::EmbeddingStore> rescore;
        if (!config.rescore_embeddings_path.empty()) {
            rescore = std::make_unique<zcgvs::EmbeddingStore>(zcgvs::EmbeddingStore::loadFromFile(config.rescore_embeddings_path));
        }
        zcgvs::VectorEngine engine(store, zcgvs::toVectorEngineConfig(config), rescore.get(), nullptr);
        const int batch = std::stoi(a["batch"]);
        const std::string raw = slurp(a["queries"]);
        if (raw.size() != static_cast<std::size_t>(batch) * store.dim() * sizeof(float)) {
            throw std::runtime_error("queries file size does not match batch x dim");
        }
        const auto* queries = reinterpret_cast<const float*>(raw.data());
        const zcgvs::SearchOptions options = engine.defaultOptions();
        const zcgvs::BatchSearchResponse response = engine.searchBatch(queries, batch, options);
        const int top_k = config.default_top_k;
        std::vector<int> ids(static_cast<std::size_t>(batch) * top_k, -1);
        std::vector<float> scores(static_cast<std::size_t>(batch) * top_k, 0.0f);
        for (int q = 0; q < batch; ++q) {
            const auto& hits = response.results[static_cast<std::size_t>(q)];
            for (std::size_t h = 0; h < hits.size() && static_cast<int>(h) < top_k; ++h) {
                ids[static_cast<std::size_t>(q) * top_k + h] = hits[h].corpus_index;
                scores[static_cast<std::size_t>(q) * top_k + h] = hits[h].similarity;
            }
        }
        std::ofstream(a["out"] + ".ids", std::ios::binary)
            .write(reinterpret_cast<const char*>(ids.data()), static_cast<std::streamsize>(ids.size() * sizeof(int)));
        std::ofstream(a["out"] + ".scores", std::ios::binary)
            .write(reinterpret_cast<const char*>(scores.data()), static_cast<std::streamsize>(scores.size() * sizeof(float)));
        std::printf("graph=%d rescore=%d\n", response.timing.graph_replay ? 1 : 0, rescore ? 1 : 0);
    } catch (const std::exception& e) {
        std::cerr << "error: " << e.what() << "\n";
        return 2;
    }
    return 0;
}
