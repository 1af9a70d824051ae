// BM25 lexical scoring over a CSR inverted index, deterministic and without atomics.
//
// The reference (src/cuda/lexical.cu:17-41) launches a block per query term and scatter-adds
// every posting weight into a [N] score vector with float atomicAdd, so the order of the
// additions (and the low bits of the result) changes from run to run; its own test compares
// with a tolerance (tests/cpp/test_lexical.cu:118-126). Here the document space is cut into
// contiguous ranges, one per CTA, and each CTA walks the query's term slots in order with the
// accumulation of lexical_device.cuh (every document's score is the exact sequential sum in
// (slot, posting) order). Each CTA writes its documents' scores and its max(0, max score) to the
// workspace; the scan kernel reduces those partial maxima (src/cuda/lexical.cu:44-64 does it
// with a float atomicMax) and blends lexical and dense scores before its top-k.
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <climits>
#include <string>

#include "host_common.h"
#include "lexical.h"
#include "lexical_device.cuh"
#include "zcgvs_sm100.h"

namespace zc {

namespace {

constexpr int kLexThreads = 512;
constexpr int kLexWarps = kLexThreads / 32;
constexpr int kLexMaxDocsPerCta = 32768;  // 128 KB accumulator

struct LexParams {
    LexIndex index;
    const int* terms;       // [batch, stride]
    int stride;
    int docs_per_cta;
    const float* init;      // [batch, n] scores to add onto, or nullptr (start at 0)
    float* out;             // [batch, n]
    float* part_max;        // [batch, gridDim.x] or nullptr
};

__global__ void __launch_bounds__(kLexThreads) lexical_kernel(const LexParams p) {
    extern __shared__ __align__(16) float acc[];
    __shared__ long long s_lo[kLexSlots];
    __shared__ long long s_hi[kLexSlots];
    __shared__ float s_max[kLexWarps];

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int q = blockIdx.y;
    const long long n = p.index.n;
    const long long d0 = static_cast<long long>(blockIdx.x) * p.docs_per_cta;
    const int count = static_cast<int>(min(static_cast<long long>(p.docs_per_cta), n - d0));
    const size_t row = static_cast<size_t>(q) * n;
    const int* terms = p.terms + static_cast<size_t>(q) * p.stride;
    // Postings in the index (CSR end): the 16-byte loads never reach past it.
    const long long total = p.index.vec ? __ldg(p.index.offsets + p.index.vocab) : 0;

    for (int i = tid; i < count; i += kLexThreads) acc[i] = p.init != nullptr ? p.init[row + d0 + i] : 0.0f;
    for (int t0 = 0; t0 < p.stride; t0 += kLexSlots) {
        lex_round<kLexThreads, 0>(p.index, terms + t0, min(kLexSlots, p.stride - t0), d0, count, acc, s_lo, s_hi,
                                  total, tid);
    }
    __syncthreads();

    float best = 0.0f;
    for (int i = tid; i < count; i += kLexThreads) {
        const float v = acc[i];
        p.out[row + d0 + i] = v;
        best = fmaxf(best, v);
    }
    if (p.part_max == nullptr) return;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, off));
    if (lane == 0) s_max[warp] = best;
    __syncthreads();
    if (tid == 0) {
        float m = 0.0f;
        for (int w = 0; w < kLexWarps; ++w) m = fmaxf(m, s_max[w]);
        p.part_max[static_cast<size_t>(q) * gridDim.x + blockIdx.x] = m > 0.0f ? m : 0.0f;
    }
}

// max(0, max of values) into *out_max with an unsigned atomicMax on the float's bits (valid
// for non-negative floats), the reference launchMaxPositive contract (src/cuda/lexical.cu:44-64).
__global__ void max_positive_kernel(const float* __restrict__ values, long long count, float* out_max) {
    float best = 0.0f;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        best = fmaxf(best, values[i]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, off));
    if ((threadIdx.x & 31) == 0 && best > 0.0f) {
        atomicMax(reinterpret_cast<unsigned int*>(out_max), __float_as_uint(best));
    }
}

// dense[i] = w * dense[i] + ((1 - w) * lexical[i]) * inv, inv = 1 / *lexical_max or 0
// (src/cuda/lexical.cu:66-72), every operation rounded on its own.
__global__ void fuse_scores_kernel(float* __restrict__ dense, const float* __restrict__ lexical,
                                   const float* __restrict__ lexical_max, float weight, long long count) {
    const float peak = *lexical_max;
    const float inv = peak > 0.0f ? __fdiv_rn(1.0f, peak) : 0.0f;
    const float lw = __fsub_rn(1.0f, weight);
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        dense[i] = __fadd_rn(__fmul_rn(weight, dense[i]), __fmul_rn(__fmul_rn(lw, lexical[i]), inv));
    }
}

}  // namespace

LexIndex lex_index(const long long* offsets, const int* docs, const float* weights, int vocab, long long n,
                   bool sorted) {
    LexIndex x{};
    x.offsets = offsets;
    x.docs = docs;
    x.weights = weights;
    x.vocab = vocab;
    x.n = n;
    x.sorted = sorted ? 1 : 0;
    x.vec = (sorted && vocab != INT_MAX && reinterpret_cast<uintptr_t>(docs) % 16 == 0 &&
             reinterpret_cast<uintptr_t>(weights) % 16 == 0)
                ? 1
                : 0;
    return x;
}

int lexical_parts(long long n) {
    const long long sms = device_sm_count();
    long long per = (n + 2 * sms - 1) / (2 * sms);
    per = std::max<long long>(per, 256);
    per = std::min<long long>(per, kLexMaxDocsPerCta);
    return static_cast<int>((n + per - 1) / per);
}

int launch_lexical(const long long* offsets, const int* docs, const float* weights, int vocab, const int* terms,
                   int stride, long long n, int batch, const float* init, float* out, float* part_max, bool sorted,
                   cudaStream_t stream) {
    const int parts = lexical_parts(n);
    const long long per = (n + parts - 1) / parts;
    LexParams p{};
    p.index = lex_index(offsets, docs, weights, vocab, n, sorted);
    p.terms = terms;
    p.stride = stride;
    p.docs_per_cta = static_cast<int>(per);
    p.init = init;
    p.out = out;
    p.part_max = part_max;
    const size_t smem = static_cast<size_t>(per) * sizeof(float);
    cudaError_t e = ensure_smem_optin(reinterpret_cast<const void*>(lexical_kernel));
    if (e != cudaSuccess) return fail_cuda(e, "cudaFuncSetAttribute(lexical_kernel)");
    constexpr int kMaxY = 65535;
    for (int q0 = 0; q0 < batch; q0 += kMaxY) {
        LexParams pc = p;
        pc.terms += static_cast<size_t>(q0) * stride;
        if (pc.init != nullptr) pc.init += static_cast<size_t>(q0) * n;
        pc.out += static_cast<size_t>(q0) * n;
        if (pc.part_max != nullptr) pc.part_max += static_cast<size_t>(q0) * parts;
        const dim3 grid(static_cast<unsigned>(parts), static_cast<unsigned>(std::min(kMaxY, batch - q0)));
        {
            KernelTimer timer("lexical", stream);
            lexical_kernel<<<grid, kLexThreads, smem, stream>>>(pc);
        }
        e = cudaGetLastError();
        if (e != cudaSuccess) return fail_cuda(e, "lexical_kernel launch");
    }
    return ok();
}

}  // namespace zc

extern "C" {

int zcgvs_bm25(const int64_t* offsets, const int* posting_docs, const float* posting_weights, const int* query_terms,
               int term_count, int doc_count, float* scores, void* stream) {
    using namespace zc;
    if (term_count <= 0 || doc_count <= 0) return ok();
    if (offsets == nullptr || posting_docs == nullptr || posting_weights == nullptr || query_terms == nullptr ||
        scores == nullptr) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_bm25: null pointer");
    }
    return launch_lexical(reinterpret_cast<const long long*>(offsets), posting_docs, posting_weights, INT_MAX,
                          query_terms, term_count, doc_count, 1, scores, scores, nullptr, false,
                          static_cast<cudaStream_t>(stream));
}

int zcgvs_max_positive(const float* values, int count, float* out_max, void* stream) {
    using namespace zc;
    if (count <= 0) return ok();
    if (values == nullptr || out_max == nullptr) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_max_positive: null pointer");
    const int blocks = std::min((count + 255) / 256, 4 * device_sm_count());
    max_positive_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(values, count, out_max);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ok() : fail_cuda(e, "max_positive_kernel launch");
}

int zcgvs_fuse_scores(float* dense, const float* lexical, const float* lexical_max, float weight, int count,
                      void* stream) {
    using namespace zc;
    if (count <= 0) return ok();
    if (dense == nullptr || lexical == nullptr || lexical_max == nullptr) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_fuse_scores: null pointer");
    }
    const int blocks = std::min((count + 255) / 256, 4 * device_sm_count());
    fuse_scores_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(dense, lexical, lexical_max, weight,
                                                                            count);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ok() : fail_cuda(e, "fuse_scores_kernel launch");
}

}  // extern "C"
