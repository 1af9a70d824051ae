// BM25 lexical scoring over a CSR inverted index, deterministic and without atomics.
//
// The reference (src/cuda/lexical.cu:17-41) launches a block per query term and scatter-adds
// every posting weight into a [N] score vector with float atomicAdd, so the order of the
// additions (and the low bits of the result) changes from run to run; its own test compares
// with a tolerance (tests/cpp/test_lexical.cu:118-126). Here the document space is cut into
// contiguous ranges, one per CTA, and each CTA walks the query's term slots in order:
//
//   * For every slot a warp finds the CTA's slice of that term's posting list with a 32-way
//     search (about log32(df) dependent loads instead of log2(df)); posting lists are sorted by
//     document within each term, as the reference builder writes them
//     (python/zcgvs_tools/build_lexical.py:143-162).
//   * The slice is added into a shared-memory accumulator of the CTA's documents. A run of
//     equal document ids (possible in hand-made indexes) is summed by one thread in posting
//     order, and slots are separated by a barrier, so every document's score is the exact
//     sequential sum in (slot, posting) order: the CPU loop of tests/cpp/test_lexical.cu:71-80.
//   * Each CTA writes its documents' scores and its max(0, max score) to the workspace; the
//     scan kernel reduces those partial maxima (src/cuda/lexical.cu:44-64 does it with a float
//     atomicMax) and blends lexical and dense scores before its top-k.
//   * Indexes whose postings are in any order (the reference launcher's contract, used by
//     zcgvs_bm25) take a second path with the same sums: one warp per CTA walks each term's whole
//     list in posting order, grouping equal documents of a 32-posting step (match_any) and adding
//     them in lane order. It reads every posting once per CTA, so it is the slow path.
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <climits>
#include <string>

#include "host_common.h"
#include "lexical.h"
#include "zcgvs_sm100.h"

namespace zc {

namespace {

constexpr int kLexThreads = 512;
constexpr int kLexWarps = kLexThreads / 32;
constexpr int kLexSlots = 128;          // term slots searched per round
constexpr int kLexMaxDocsPerCta = 32768;  // 128 KB accumulator

struct LexParams {
    const long long* offsets;
    const int* docs;
    const float* weights;
    int vocab;
    const int* terms;       // [batch, stride]
    int stride;
    long long n;
    int docs_per_cta;
    const float* init;      // [batch, n] scores to add onto, or nullptr (start at 0)
    float* out;             // [batch, n]
    float* part_max;        // [batch, gridDim.x] or nullptr
    int sorted;             // postings sorted by document within each term (else: any order)
    int vec;                // sorted, docs and weights 16-byte aligned: 16-byte posting loads
};

// First index in [lo, hi) whose document id is >= target (hi if none), for sorted docs[].
// Whole warp; 32 probes per step.
__device__ long long lower_bound_warp(const int* __restrict__ docs, long long lo, long long hi, int target,
                                      int lane) {
    while (hi - lo > 32) {
        const long long step = (hi - lo + 31) / 32;
        const long long pos = lo + lane * step;
        const bool less = pos < hi && __ldg(docs + pos) < target;
        const int c = __popc(__ballot_sync(0xffffffffu, less));
        if (c == 0) return lo;
        const long long next_hi = lo + static_cast<long long>(c) * step;
        lo += static_cast<long long>(c - 1) * step + 1;
        hi = min(hi, next_hi);
    }
    const long long pos = lo + lane;
    const bool less = pos < hi && __ldg(docs + pos) < target;
    return lo + __popc(__ballot_sync(0xffffffffu, less));
}

// lower_bound_warp with a first round of 32 probes `step` apart around `guess` (where the target
// would sit if the list's documents were spread evenly over [0, n)); the answer's side of that
// window is then searched as usual. Exact for any sorted list; for evenly spread lists the
// window holds the answer and about two dependent loads are saved per search.
__device__ long long lower_bound_hint(const int* __restrict__ docs, long long lo, long long hi, int target,
                                      long long guess, long long step, int lane) {
    if (hi - lo > 64) {
        const long long pos = min(max(guess + static_cast<long long>(lane - 16) * step, lo), hi - 1);
        const bool less = __ldg(docs + pos) < target;  // a prefix of the lanes (positions ascend)
        const int c = __popc(__ballot_sync(0xffffffffu, less));
        const long long below = __shfl_sync(0xffffffffu, pos, max(c - 1, 0));
        const long long at = __shfl_sync(0xffffffffu, pos, min(c, 31));
        if (c > 0) lo = below + 1;   // docs[below] < target
        if (c < 32) hi = at + 1;     // docs[at] >= target
    }
    return lower_bound_warp(docs, lo, hi, target, lane);
}

__global__ void __launch_bounds__(kLexThreads) lexical_kernel(const LexParams p) {
    extern __shared__ __align__(16) float acc[];
    __shared__ long long s_lo[kLexSlots];
    __shared__ long long s_hi[kLexSlots];
    __shared__ float s_max[kLexWarps];

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int q = blockIdx.y;
    const long long d0 = static_cast<long long>(blockIdx.x) * p.docs_per_cta;
    const int count = static_cast<int>(min(static_cast<long long>(p.docs_per_cta), p.n - d0));
    const size_t row = static_cast<size_t>(q) * p.n;
    const int* terms = p.terms + static_cast<size_t>(q) * p.stride;
    // Postings in the index (CSR end): the 16-byte loads never reach past it.
    const long long total = p.vec ? __ldg(p.offsets + p.vocab) : 0;

    for (int i = tid; i < count; i += kLexThreads) acc[i] = p.init != nullptr ? p.init[row + d0 + i] : 0.0f;

    for (int t0 = 0; t0 < p.stride; t0 += kLexSlots) {
        const int slots = min(kLexSlots, p.stride - t0);
        __syncthreads();  // the previous round's slices are consumed
        for (int t = warp; t < slots; t += kLexWarps) {
            const int term = __ldg(terms + t0 + t);
            long long lo = 0, hi = 0;
            if (term >= 0 && term < p.vocab) {
                const long long begin = __ldg(p.offsets + term);
                const long long end = __ldg(p.offsets + term + 1);
                if (p.sorted) {
                    // Interpolated first probes: a window of +-16 steps covers about three standard
                    // deviations of a randomly spread list's position (sqrt(df) / 2 at most).
                    const long long df = end - begin;
                    const double per_doc = static_cast<double>(df) / static_cast<double>(p.n);
                    const long long step = 1 + static_cast<long long>(0.1 * sqrt(static_cast<double>(df)));
                    lo = lower_bound_hint(p.docs, begin, end, static_cast<int>(d0),
                                          begin + static_cast<long long>(per_doc * static_cast<double>(d0)), step, lane);
                    hi = lower_bound_hint(p.docs, lo, end, static_cast<int>(d0 + count),
                                          begin + static_cast<long long>(per_doc * static_cast<double>(d0 + count)), step,
                                          lane);
                } else {
                    lo = begin;
                    hi = end;
                }
            }
            if (lane == 0) {
                s_lo[t] = lo;
                s_hi[t] = hi;
            }
        }
        __syncthreads();
        if (!p.sorted) {
            // Any posting order: warp 0 walks each term's whole list in posting order, 32 at a time.
            // Postings of one document inside a step are grouped (match_any) and added in lane
            // order, so every sum keeps the sequential (slot, posting) order.
            if (warp == 0) {
                for (int t = 0; t < slots; ++t) {
                    const long long lo = s_lo[t];
                    const long long hi = s_hi[t];
                    for (long long base = lo; base < hi; base += 32) {
                        const long long i = base + lane;
                        const int doc = i < hi ? __ldg(p.docs + i) : -1;
                        const bool mine = doc >= d0 && doc < d0 + count;
                        const float w = mine ? __ldg(p.weights + i) : 0.0f;
                        const uint32_t peers = __match_any_sync(0xffffffffu, mine ? doc : -1 - lane);
                        const int rank = __popc(peers & ((1u << lane) - 1u));
                        int rounds = mine ? __popc(peers) : 0;
#pragma unroll
                        for (int off = 16; off > 0; off >>= 1) rounds = max(rounds, __shfl_xor_sync(0xffffffffu, rounds, off));
                        for (int r = 0; r < rounds; ++r) {
                            if (mine && rank == r) acc[doc - d0] = __fadd_rn(acc[doc - d0], w);
                            __syncwarp();
                        }
                    }
                }
            }
            __syncthreads();
            continue;
        }
        if (p.vec) {
            // 16-byte posting groups, software-pipelined across slots. A step is one group per
            // thread of one slot (thread tid owns group g0 + tid); the loads of the next two steps
            // are in flight while a step's additions run, across the barrier that closes a slot
            // (loads never touch the accumulator), so a slot's memory latency overlaps the work
            // of the slots before it. Slots without postings here are skipped. A posting is the
            // head of its run unless the posting before it (the same thread's, the previous
            // lane's last one, or for lane 0 a load) holds the same document.
            struct Step {
                int t;
                long long g0;
            };
            struct Group {
                int4 dv;
                float4 wv;
                int before;
            };
            auto g_lo = [&](int t) { return s_lo[t] >> 2; };
            auto g_hi = [&](int t) { return (s_hi[t] + 3) >> 2; };
            auto first_from = [&](int t) {
                while (t < slots && g_lo(t) >= g_hi(t)) ++t;
                return Step{t, t < slots ? g_lo(t) : 0};
            };
            auto advance = [&](Step c) {
                if (c.t >= slots) return c;
                const long long g0 = c.g0 + kLexThreads;
                return g0 < g_hi(c.t) ? Step{c.t, g0} : first_from(c.t + 1);
            };
            auto load = [&](Step c, Group& b) {
                b.dv = make_int4(-1, -1, -1, -1);
                b.wv = make_float4(0.f, 0.f, 0.f, 0.f);
                b.before = -1;
                if (c.t >= slots) return;
                const long long g = c.g0 + tid;
                if (g >= g_hi(c.t)) return;
                if (4 * g + 3 < total) {
                    b.dv = __ldg(reinterpret_cast<const int4*>(p.docs) + g);
                    b.wv = __ldg(reinterpret_cast<const float4*>(p.weights) + g);
                } else {
                    // The index's last partial group: element loads.
                    int dd[4] = {-1, -1, -1, -1};
                    float ww[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        if (4 * g + e < total) {
                            dd[e] = __ldg(p.docs + 4 * g + e);
                            ww[e] = __ldg(p.weights + 4 * g + e);
                        }
                    }
                    b.dv = make_int4(dd[0], dd[1], dd[2], dd[3]);
                    b.wv = make_float4(ww[0], ww[1], ww[2], ww[3]);
                }
                if (lane == 0 && 4 * g > s_lo[c.t]) b.before = __ldg(p.docs + 4 * g - 1);
            };
            auto process = [&](Step c, const Group& b) {
                const long long lo = s_lo[c.t];
                const long long hi = s_hi[c.t];
                const long long g = c.g0 + tid;
                const int up = __shfl_up_sync(0xffffffffu, b.dv.w, 1);
                if (g >= g_hi(c.t)) return;
                const int d[4] = {b.dv.x, b.dv.y, b.dv.z, b.dv.w};
                const float w[4] = {b.wv.x, b.wv.y, b.wv.z, b.wv.w};
                int prev = lane == 0 ? b.before : up;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const long long i = 4 * g + e;
                    const int doc = d[e];
                    const bool head = i >= lo && i < hi && (i == lo || prev != doc);
                    prev = doc;
                    if (!head) continue;
                    float a = __fadd_rn(acc[doc - d0], w[e]);
                    // The rest of a run of equal documents, in posting order (rare).
                    for (long long j = i + 1; j < hi && __ldg(p.docs + j) == doc; ++j) {
                        a = __fadd_rn(a, __ldg(p.weights + j));
                    }
                    acc[doc - d0] = a;
                }
            };
            Step s0 = first_from(0);
            Step s1 = advance(s0);
            Group b0, b1, b2;
            load(s0, b0);
            load(s1, b1);
            while (s0.t < slots) {
                const Step s2 = advance(s1);
                load(s2, b2);
                process(s0, b0);
                if (s1.t != s0.t) __syncthreads();  // slot s0.t's additions land before the next slot's
                s0 = s1;
                s1 = s2;
                b0 = b1;
                b1 = b2;
            }
        } else {
            for (int t = 0; t < slots; ++t) {
                const long long lo = s_lo[t];
                const long long hi = s_hi[t];
                for (long long i = lo + tid; i < hi; i += kLexThreads) {
                    const int doc = __ldg(p.docs + i);
                    if (i > lo && __ldg(p.docs + i - 1) == doc) continue;  // not the head of its run
                    float a = acc[doc - d0];
                    a = __fadd_rn(a, __ldg(p.weights + i));
                    for (long long j = i + 1; j < hi && __ldg(p.docs + j) == doc; ++j) {
                        a = __fadd_rn(a, __ldg(p.weights + j));
                    }
                    acc[doc - d0] = a;
                }
                __syncthreads();  // slot t's additions land before slot t + 1's
            }
        }
    }

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
    p.offsets = offsets;
    p.docs = docs;
    p.weights = weights;
    p.vocab = vocab;
    p.terms = terms;
    p.stride = stride;
    p.n = n;
    p.docs_per_cta = static_cast<int>(per);
    p.init = init;
    p.out = out;
    p.part_max = part_max;
    p.sorted = sorted ? 1 : 0;
    p.vec = (sorted && vocab != INT_MAX && reinterpret_cast<uintptr_t>(docs) % 16 == 0 &&
             reinterpret_cast<uintptr_t>(weights) % 16 == 0)
                ? 1
                : 0;
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
