// Host interface of the lexical (BM25) kernel, used by the hybrid search entry point.
#pragma once

#include <cuda_runtime.h>

namespace zc {

// Number of document ranges (CTAs per query) the lexical kernel uses for n documents; also the
// row length of its partial-maximum output.
int lexical_parts(long long n);

// Scores `batch` queries of `stride` term slots each: out[q][d] = init[q][d] (or 0) + the
// posting weights of d under the valid terms of query q, summed in (slot, posting) order;
// part_max[q][i] = max(0, max over range i). `sorted`: posting lists are sorted by document id
// within each term (each range reads only its slice); otherwise every range walks the query's
// whole lists (any order, same sums). Returns a zcgvs status.
int launch_lexical(const long long* offsets, const int* docs, const float* weights, int vocab, const int* terms,
                   int stride, long long n, int batch, const float* init, float* out, float* part_max, bool sorted,
                   cudaStream_t stream);

}  // namespace zc
