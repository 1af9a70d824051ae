// Prints the request rules of include/zcgvs/engine/vector_engine.hpp (option resolution, lexical
// term preparation, allow masks) for fixed cases, one line each, for tests/test_engine_cpu.py.
// Host code only: no device is touched.
#include <cstdio>
#include <vector>

#include "zcgvs/engine/vector_engine.hpp"

using namespace zcgvs;

static void show(const char* name, const ResolvedOptions& r) {
    std::printf("%s top_k=%d candidates=%d rescore=%d weight=%.3f hybrid=%d graph=%d metric=%d\n", name, r.top_k,
                r.candidates, r.rescore_candidates, r.dense_weight, r.hybrid ? 1 : 0, r.use_graph ? 1 : 0,
                static_cast<int>(r.metric));
}

int main() {
    VectorEngineConfig c;  // top_k 10, candidates 100, rescore 0, weight 0.7, graphs off
    SearchOptions o;
    show("defaults", resolveSearchOptions(c, o, 1000, false, false));
    show("small_corpus", resolveSearchOptions(c, o, 50, false, false));
    SearchOptions a;
    a.top_k = 200;
    a.candidates = 20;
    show("topk_over_candidates", resolveSearchOptions(c, a, 1000, false, false));
    show("topk_over_corpus", resolveSearchOptions(c, a, 150, false, false));
    SearchOptions r;
    r.rescore_candidates = 40;
    show("rescore_below_candidates", resolveSearchOptions(c, r, 1000, true, false));
    show("rescore_without_store", resolveSearchOptions(c, r, 1000, false, false));
    r.rescore_candidates = 5000;
    show("rescore_over_corpus", resolveSearchOptions(c, r, 1000, true, false));
    VectorEngineConfig c2 = c;
    c2.rescore_candidates = 300;
    c2.use_cuda_graphs = true;
    c2.metric = Metric::L2;
    show("config_rescore_graph", resolveSearchOptions(c2, o, 1000, true, false));
    SearchOptions w;
    w.dense_weight = 3.0f;
    w.hybrid = true;
    w.use_config_metric = false;
    w.metric = Metric::DotProduct;
    w.use_config_graphs = false;
    w.use_graph = true;
    show("weight_clamp_hybrid", resolveSearchOptions(c, w, 1000, false, true));
    show("hybrid_without_index", resolveSearchOptions(c, w, 1000, false, false));
    try {
        VectorEngineConfig bad = c;
        bad.default_top_k = 0;
        resolveSearchOptions(bad, o, 1000, false, false);
        std::printf("zero_topk no-throw\n");
    } catch (const std::invalid_argument&) {
        std::printf("zero_topk invalid_argument\n");
    }
    const std::vector<std::vector<int>> enc = {{101, 7, 7, 9, -1, 3, 9, 102}, {101, 102}, {101, 5, 102}, {}};
    for (const auto& e : enc) {
        std::printf("terms");
        for (int t : lexicalTermsFromIds(e, 64)) std::printf(" %d", t);
        std::printf("\n");
    }
    std::printf("terms_capped");
    for (int t : lexicalTermsFromIds({101, 1, 2, 3, 4, 5, 102}, 3)) std::printf(" %d", t);
    std::printf("\n");
    const auto m = allowMask({3, -2, 0, 3, 9, 12}, 10);
    std::printf("mask");
    for (auto b : m) std::printf(" %d", static_cast<int>(b));
    std::printf("\nmask_empty %zu\n", allowMask({}, 10).size());
    return 0;
}
