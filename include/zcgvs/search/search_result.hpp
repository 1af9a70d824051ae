// Host copy of a [batch, k] selection (the reference's HostTopK,
// include/zcgvs/search/search_result.hpp:10-19).
#pragma once

#include <cstddef>
#include <vector>

namespace zcgvs {

struct HostTopK {
    std::vector<int> indices;
    std::vector<float> scores;
    int batch = 0;
    int k = 0;

    std::size_t offset(int query) const { return static_cast<std::size_t>(query) * static_cast<std::size_t>(k); }
};

}  // namespace zcgvs
