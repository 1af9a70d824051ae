// Host interface of the lexical (BM25) kernel, used by the hybrid search entry point.
#pragma once

#include <cuda_runtime.h>

#include "lexical_device.cuh"

namespace zc {

// Number of document ranges (CTAs per query) the lexical kernel uses for n documents; also the
// row length of its partial-maximum output.
int lexical_parts(long long n);

// The index view the kernels read; `vec` (16-byte posting loads) is set when the lists are
// sorted, the vocabulary is bounded (vocab != INT_MAX) and both posting arrays are 16-byte
// aligned.
LexIndex lex_index(const long long* offsets, const int* docs, const float* weights, int vocab, long long n,
                   bool sorted);

// Scores `batch` queries of `stride` term slots each: out[q][d] = init[q][d] (or 0) + the
// posting weights of d under the valid terms of query q, summed in (slot, posting) order;
// part_max[q][i] = max(0, max over range i). `sorted`: posting lists are sorted by document id
// within each term (each range reads only its slice); otherwise every range walks the query's
// whole lists (any order, same sums). Returns a zcgvs status.
int launch_lexical(const long long* offsets, const int* docs, const float* weights, int vocab, const int* terms,
                   int stride, long long n, int batch, const float* init, float* out, float* part_max, bool sorted,
                   cudaStream_t stream);

// Cross-CTA state of the fused hybrid search, zero between calls (the select kernel's last CTA
// clears it): the bits of max(0, max lexical score), raised by the hybrid scan, and the select
// kernel's ticket.
struct HybridSelectState {
    unsigned int peak;
    unsigned int ticket;
};

// Second kernel of the fused hybrid search (hybrid_select.cu): blends dense[n] and lex[n] with
// w and 1 / max (the peak in *state; 0 when not positive), writes the top-k keys of each of
// `grid` contiguous document ranges to cand[grid][k], and the last CTA ranks the keys at or
// above the largest k-th key into out_idx / out_scores. k <= 256.
// Launched as a programmatic dependent of the kernel before it on `stream`.
int launch_hybrid_select(const float* dense, const float* lex, HybridSelectState* state, float weight, long long n,
                         int k, unsigned int id_base, unsigned long long* cand, int* out_idx, float* out_scores,
                         int grid, cudaStream_t stream);

}  // namespace zc
