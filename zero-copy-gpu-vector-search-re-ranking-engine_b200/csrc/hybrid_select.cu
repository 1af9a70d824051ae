// Second kernel of the fused hybrid search: blend the materialised dense and lexical scores of
// one query and select its top-k.
//
// The first kernel (scan_fast_kernel<MODE, JC, true>) streams the dense rows and, in the same
// CTAs, accumulates the BM25 scores of the CTA's documents; it writes both score vectors and
// raises the lexical maximum. The blend needs that maximum over every document
// (src/cuda/lexical.cu:44-72), so it runs here, once the first kernel has finished: 1 / max (0
// when the max is not positive), then w * dense + ((1 - w) * lex) * inv with every operation
// rounded on its own.
//
// Selection inside a CTA (one 1,024-thread CTA per SM, 32 warps hiding each other's latency
// chains): the CTA's documents in chunks of up to 16 per thread, every load of a chunk issued at
// once (16-byte loads, four documents each). A score is compared by its order-preserving bit
// pattern (the high word of its selection key); each chunk's patterns go to shared memory. Two
// lower bounds of the CTA's k-th score, each with k documents at least as good: per warp, the
// k-th largest of its 64 best-two-per-lane scores (k <= 64); over the warps, the k-th largest of
// the 32 warp maxima (k <= 32). Only documents scoring at or above the larger become candidates
// (their 64-bit keys are built then), a few dozen per CTA; a warp per candidate counts its rank
// (the keys are distinct) and the ranks below k place the CTA's top-k. If the candidates ever
// outgrow their buffer, the CTA selects again over all its documents with the general top-k
// buffer.
//
// Across CTAs: each CTA writes its top-k, descending, to its slot of a global array. The last CTA
// (ticket) loads all the lists at once. The k-th largest list head is a lower bound of the
// query's k-th key (k lists hold a key at least as large), so only the keys at or above it, at
// most k * k, are ranked the same way.
//
// The kernel is launched as a programmatic dependent of the scan (griddepcontrol): it may start
// while the scan's last CTAs finish, and waits for the scan's completion and memory before its
// first read.
#include <cuda_runtime.h>

#include <algorithm>

#include "host_common.h"
#include "lexical.h"
#include "scan_kernel.cuh"
#include "topk_cta.cuh"
#include "zcgvs_sm100.h"

namespace zc {

namespace {

constexpr int kSelectThreads = 1024;
constexpr int kSelectWarps = kSelectThreads / 32;
constexpr int kSelectGroups = 4;                                   // 4-document groups per thread per chunk
constexpr int kSelectChunk = kSelectThreads * kSelectGroups;       // groups per chunk
constexpr int kSelectCand = 2048;                                  // candidate buffer (keys)
constexpr int kSelectTop = kSelectCand / 8;                        // largest k of the fast path
constexpr int kSelectFallbackU = 2;

struct SelectParams {
    const float* dense;          // [n] dense scores (masked rows -FLT_MAX), 16-byte aligned
    const float* lex;            // [n] lexical scores, 16-byte aligned
    HybridSelectState* state;    // peak and ticket; zero between calls
    float weight;                // dense weight w
    long long n;
    int k;
    int cap;                     // general top-k buffer capacity (fallback; power of two)
    unsigned int id_base;
    unsigned long long* cand;    // [gridDim.x][k] the CTAs' lists
    int* out_idx;                // [k]
    float* out_scores;           // [k]
};

// Ranks by counting, a warp per candidate: rank = how many of the n distinct keys in keys[] are
// larger. Each candidate ranked below k is written to out[rank]. Called by every thread.
__device__ __forceinline__ void rank_place(const u64* keys, int n, int k, u64* out) {
    const int lane = threadIdx.x & 31;
    for (int c = threadIdx.x >> 5; c < n; c += kSelectWarps) {
        const u64 mine = keys[c];
        int rank = 0;
        for (int j = lane; j < n; j += 32) rank += keys[j] > mine ? 1 : 0;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) rank += __shfl_xor_sync(0xffffffffu, rank, off);
        if (lane == 0 && rank < k) out[rank] = mine;
    }
}

__global__ void __launch_bounds__(kSelectThreads, 1) hybrid_select_kernel(const SelectParams p) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // The chunk's score patterns [4 * kSelectChunk] (0 = no document), then the candidates. The
    // fallback's top-k buffer (64-bit keys from offset 0) reuses them.
    extern __shared__ __align__(16) u64 smem_keys[];
    uint32_t* bits = reinterpret_cast<uint32_t*>(smem_keys);
    u64* cand = smem_keys + 2 * kSelectChunk;
    __shared__ int s_count;
    __shared__ u64 s_thr;
    __shared__ uint32_t s_floor;
    __shared__ u64 s_floor_key;
    __shared__ float s_inv;
    __shared__ int s_last;
    __shared__ u64 s_top[kSelectTop];  // this CTA's top-k, descending
    __shared__ uint32_t s_wmax[kSelectWarps];

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int cta = blockIdx.x;
    const int G = gridDim.x;
    // The CTA's documents in whole 4-document groups; the last group may pass n (masked below;
    // the buffers are padded to 16 bytes).
    const long long groups = (p.n + 3) / 4;
    const long long g0 = groups * cta / G;
    const int ng = static_cast<int>(groups * (cta + 1) / G - g0);
    const float4* dense4 = reinterpret_cast<const float4*>(p.dense) + g0;
    const float4* lex4 = reinterpret_cast<const float4*>(p.lex) + g0;

    float4 dv[kSelectGroups], lv[kSelectGroups];
    auto fetch = [&](int base) {
#pragma unroll
        for (int u = 0; u < kSelectGroups; ++u) {
            const int gi = base + u * kSelectThreads + tid;
            if (gi < ng) {
                dv[u] = __ldcg(dense4 + gi);
                lv[u] = __ldcg(lex4 + gi);
            }
        }
    };
    // The peak's load goes out before the score loads, so it does not queue behind them.
    const unsigned int peak_bits = tid == 0 ? __ldcg(&p.state->peak) : 0u;
    fetch(0);
    if (tid == 0) {
        // max(0, max lexical score): raised as the bits of non-negative floats.
        const float peak = __uint_as_float(peak_bits);
        s_inv = peak > 0.0f ? __fdiv_rn(1.0f, peak) : 0.0f;
        s_floor = 0u;
        s_count = 0;
        s_thr = 0ull;
    }
    __syncthreads();
    const float inv = s_inv;
    const float w = p.weight;

    uint32_t best1 = 0u, best2 = 0u;  // this lane's two best score patterns so far
    for (int base = 0; base < ng; base += kSelectChunk) {
#pragma unroll
        for (int u = 0; u < kSelectGroups; ++u) {
            const int gi = base + u * kSelectThreads + tid;
            const float d[4] = {dv[u].x, dv[u].y, dv[u].z, dv[u].w};
            const float l[4] = {lv[u].x, lv[u].y, lv[u].z, lv[u].w};
            uint32_t b4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const long long r = 4 * (g0 + gi) + e;
                // A finite score's pattern is never 0, the mark of "no document".
                const uint32_t v = (gi < ng && r < p.n) ? orderable_bits(hybrid_blend(d[e], l[e], w, inv)) : 0u;
                b4[e] = v;
                if (v > best2) {
                    best2 = v > best1 ? best1 : v;
                    best1 = v > best1 ? v : best1;
                }
            }
            reinterpret_cast<uint4*>(bits)[u * kSelectThreads + tid] = make_uint4(b4[0], b4[1], b4[2], b4[3]);
        }
        if (base + kSelectChunk < ng) fetch(base + kSelectChunk);
        if (p.k <= 64) {
            uint32_t v[2] = {best1, best2};
            warp_sort_desc_regs<2, uint32_t>(v, lane);
            // Element k - 1 of the sorted 64 sits in lane (k - 1) / 2, register (k - 1) % 2.
            const uint32_t mine = ((p.k - 1) & 1) ? v[1] : v[0];
            const uint32_t bound = __shfl_sync(0xffffffffu, mine, (p.k - 1) >> 1);
            if (lane == 0) {
                if (bound != 0u) atomicMax(&s_floor, bound);
                s_wmax[tid >> 5] = v[0];
            }
        }
        __syncthreads();
        if (p.k <= kSelectWarps && tid < kSelectWarps) {
            // The warp maximum ranked k - 1 among the 32 (equal maxima share a rank; any rank
            // k - 1 maximum has k maxima at least as large).
            const uint32_t mine = s_wmax[tid];
            int rank = 0;
#pragma unroll 8
            for (int j = 0; j < kSelectWarps; ++j) rank += s_wmax[j] > mine ? 1 : 0;
            if (rank == p.k - 1 && mine != 0u) atomicMax(&s_floor, mine);
        }
        __syncthreads();
        const uint32_t floor_bits = s_floor;
#pragma unroll
        for (int u = 0; u < kSelectGroups; ++u) {
            const uint4 b4 = reinterpret_cast<const uint4*>(bits)[u * kSelectThreads + tid];
            const uint32_t bv[4] = {b4.x, b4.y, b4.z, b4.w};
            const int gi = base + u * kSelectThreads + tid;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const bool take = bv[e] != 0u && bv[e] >= floor_bits;
                const uint32_t ballot = __ballot_sync(0xffffffffu, take);
                if (ballot != 0u) {
                    int slot = 0;
                    if (lane == 0) slot = atomicAdd(&s_count, __popc(ballot));
                    slot = __shfl_sync(0xffffffffu, slot, 0) + __popc(ballot & ((1u << lane) - 1u));
                    if (take && slot < kSelectCand) {
                        const uint32_t id = p.id_base + static_cast<uint32_t>(4 * (g0 + gi) + e);
                        cand[slot] = (static_cast<u64>(bv[e]) << 32) | static_cast<uint32_t>(~id);
                    }
                }
            }
        }
        __syncthreads();  // the chunk's patterns are read before the next chunk overwrites them
    }
    const int got = s_count;
    for (int j = tid; j < p.k; j += kSelectThreads) s_top[j] = 0ull;
    if (got <= kSelectCand) {
        __syncthreads();
        rank_place(cand, got, p.k, s_top);
        __syncthreads();
    } else {
        // Too many candidates for the buffer: the general top-k buffer over every document.
        TopkSmem mt;
        mt.buf = smem_keys;
        mt.count = &s_count;
        mt.thr = &s_thr;
        mt.cap = p.cap;
        mt.k = p.k;
        __syncthreads();  // every thread has read got
        if (tid == 0) s_count = 0;
        __syncthreads();
        auto key_of = [&](int i) -> u64 {
            const long long r = 4 * g0 + i;
            if (r >= p.n) return 0ull;
            const float score = hybrid_blend(__ldcg(p.dense + r), __ldcg(p.lex + r), w, inv);
            return make_key(score, p.id_base + static_cast<uint32_t>(r));
        };
        topk_offer_all<kSelectFallbackU>(mt, 0, 4 * ng, 0ull, key_of, kSelectThreads);
        topk_flush_mask(mt, 1u, kSelectThreads);
        for (int j = tid; j < s_count; j += kSelectThreads) s_top[j] = smem_keys[j];
        __syncthreads();
    }

    // This CTA's list, then the ticket.
    for (int j = tid; j < p.k; j += kSelectThreads) p.cand[static_cast<size_t>(cta) * p.k + j] = s_top[j];
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned int ticket = atomicAdd(&p.state->ticket, 1u);
        s_last = (ticket == static_cast<unsigned int>(G - 1)) ? 1 : 0;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    // Last CTA: every list in one load round (two keys per thread when they fit), the floor (the
    // k-th largest list head), the keys at or above it, ranked.
    const int total = G * p.k;
    u64* heads = cand + kSelectCand - kSelectThreads;  // [G] past the kept keys (at most k * k)
    if (tid == 0) {
        s_count = 0;
        s_floor_key = 0ull;
    }
    u64 held[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int j = tid + h * kSelectThreads;
        held[h] = j < total ? __ldcg(p.cand + j) : 0ull;
    }
    for (int c = tid; c < G; c += kSelectThreads) {
        const int j = c * p.k;
        heads[c] = j < 2 * kSelectThreads ? 0ull : __ldcg(p.cand + j);
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int j = tid + h * kSelectThreads;
        if (j < total && j % p.k == 0) heads[j / p.k] = held[h];
    }
    __syncthreads();
    for (int c = tid; c < G; c += kSelectThreads) {
        const u64 mine = heads[c];
        const int rank = key_rank(heads, G, mine);  // heads is 16-byte aligned: eight keys a step
        if (rank == p.k - 1 && mine != 0ull) atomicMax(&s_floor_key, mine);
    }
    __syncthreads();
    const u64 floor = s_floor_key;
    for (int j = tid; j < ((total + 31) & ~31); j += kSelectThreads) {
        const u64 key = j < 2 * kSelectThreads ? held[j / kSelectThreads] : (j < total ? __ldcg(p.cand + j) : 0ull);
        const bool take = key != 0ull && key >= floor;
        const uint32_t ballot = __ballot_sync(0xffffffffu, take);
        if (ballot != 0u) {
            int slot = 0;
            if (lane == 0) slot = atomicAdd(&s_count, __popc(ballot));
            slot = __shfl_sync(0xffffffffu, slot, 0) + __popc(ballot & ((1u << lane) - 1u));
            if (take && slot < kSelectCand) cand[slot] = key;
        }
    }
    for (int j = tid; j < p.k; j += kSelectThreads) s_top[j] = 0ull;
    __syncthreads();
    if (s_count <= kSelectCand) {
        rank_place(cand, s_count, p.k, s_top);
        __syncthreads();
    } else {
        // More keys at the floor than the buffer holds: the general top-k buffer over the lists.
        TopkSmem mt;
        mt.buf = smem_keys;
        mt.count = &s_count;
        mt.thr = &s_thr;
        mt.cap = p.cap;
        mt.k = p.k;
        __syncthreads();
        if (tid == 0) {
            s_count = 0;
            s_thr = 0ull;
        }
        __syncthreads();
        topk_offer_all<kSelectFallbackU>(mt, 0, total, floor, [&](int i) { return __ldcg(p.cand + i); },
                                         kSelectThreads);
        topk_flush_mask(mt, 1u, kSelectThreads);
        for (int j = tid; j < s_count; j += kSelectThreads) s_top[j] = smem_keys[j];
        __syncthreads();
    }
    for (int j = tid; j < p.k; j += kSelectThreads) {
        p.out_idx[j] = key_id(s_top[j]);
        p.out_scores[j] = key_score(s_top[j]);
    }
    if (tid == 0) {
        p.state->peak = 0u;
        p.state->ticket = 0u;
    }
}

// Shared memory: one chunk's score patterns and the candidates; the fallback's top-k buffer (cap
// keys) lives in the same bytes.
constexpr int kSelectSmemKeys = 2 * kSelectChunk + kSelectCand;

// The general top-k buffer's capacity: a power of two within the shared memory, room for k keys
// plus one fallback round (topk_offer_all), or 0 when k is too large for it.
int hybrid_select_cap(int k) {
    int cap = 1;
    while (cap * 2 <= kSelectSmemKeys) cap *= 2;
    return cap >= k + kSelectFallbackU * kSelectThreads ? cap : 0;
}

}  // namespace

int launch_hybrid_select(const float* dense, const float* lex, HybridSelectState* state, float weight, long long n,
                         int k, unsigned int id_base, unsigned long long* cand, int* out_idx, float* out_scores,
                         int grid, cudaStream_t stream) {
    // A CTA's top-k fits its shared list.
    if (k > kSelectTop) return fail(ZCGVS_ERR_UNSUPPORTED, "zcgvs: hybrid select: k too large");
    SelectParams p{};
    p.dense = dense;
    p.lex = lex;
    p.state = state;
    p.weight = weight;
    p.n = n;
    p.k = k;
    p.cap = hybrid_select_cap(k);
    if (p.cap == 0) return fail(ZCGVS_ERR_UNSUPPORTED, "zcgvs: hybrid select: k too large");
    p.id_base = id_base;
    p.cand = cand;
    p.out_idx = out_idx;
    p.out_scores = out_scores;
    const size_t smem = static_cast<size_t>(kSelectSmemKeys) * sizeof(u64);
    cudaError_t e = ensure_smem_optin(reinterpret_cast<const void*>(hybrid_select_kernel));
    if (e != cudaSuccess) return fail_cuda(e, "cudaFuncSetAttribute(hybrid_select_kernel)");
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(kSelectThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    {
        KernelTimer timer("hybrid_select", stream);
        e = cudaLaunchKernelEx(&cfg, hybrid_select_kernel, p);
    }
    if (e != cudaSuccess) return fail_cuda(e, "hybrid_select_kernel launch");
    return ok();
}

}  // namespace zc
