// One returned document (the reference's SearchHit / Candidate,
// include/zcgvs/engine/search_hit.hpp:7-19). The vector engine has no passage store, so doc_id
// and text stay empty; rerank_score equals similarity (no cross-encoder on this path).
#pragma once

#include <string>

namespace zcgvs {

struct SearchHit {
    std::string doc_id;
    std::string text;
    float similarity = 0.0f;
    float rerank_score = 0.0f;
    int corpus_index = -1;
};

struct Candidate {
    std::string doc_id;
    float score = 0.0f;
    int corpus_index = -1;
};

}  // namespace zcgvs
