// On-chip top-k accumulator shared by the fused scan, rescore and merge kernels.
//
// Each CTA keeps, per query it serves, a shared-memory buffer of `cap` 64-bit selection keys
// (see common.cuh), a fill count and a threshold: the k-th best key retained so far. Scores
// that cannot beat the threshold are dropped in registers; survivors are appended with one
// shared atomic. When a buffer approaches capacity the whole CTA sorts it (bitonic network,
// descending) and truncates it to k, raising the threshold. Nothing per-document ever reaches
// global memory, which is what replaces the reference's materialised [batch, N] score matrix
// and its multi-pass bitonic top-k (src/cuda/topk.cu:30-189).
//
// Invariant: between flushes at most `max_new` keys are offered per query, and a flush is
// triggered whenever count > cap - max_new, so cap >= k + max_new guarantees no overflow.
#pragma once

#include "common.cuh"

namespace zc {

struct TopkSmem {
    u64* buf;   // [queries][cap]
    int* count;      // [queries]
    u64* thr;   // [queries]
    int cap;         // power of two
    int k;
};

__device__ __forceinline__ void topk_offer(const TopkSmem& t, int q, u64 key) {
    if (key > t.thr[q]) {
        const int slot = atomicAdd(&t.count[q], 1);
        t.buf[q * t.cap + slot] = key;
    }
}

// Offer that also reports whether this append filled the buffer past `cap - max_new`, i.e.
// whether the CTA must flush before the next `max_new` offers.
__device__ __forceinline__ bool topk_offer_check(const TopkSmem& t, int q, u64 key, int max_new) {
    if (key > t.thr[q]) {
        const int slot = atomicAdd(&t.count[q], 1);
        t.buf[q * t.cap + slot] = key;
        return slot >= t.cap - max_new;
    }
    return false;
}

// Sorts the buffers of the queries selected by `mask` (bit q) descending and truncates them
// to k. Only the filled prefix is sorted (rounded up to a power of two), with shift-only index
// arithmetic. Must be called by every thread of the CTA, after a __syncthreads() that follows
// the last offer. Ends with a __syncthreads() when anything was flushed.
__device__ inline void topk_flush_mask(const TopkSmem& t, uint32_t mask, int nthreads) {
    if (mask == 0u) return;
    const int tid = threadIdx.x;
    int segs[32];
    int nseg = 0;
    int longest = 2;
    for (uint32_t m = mask; m != 0u; m &= m - 1u) {
        const int q = __ffs(m) - 1;
        segs[nseg++] = q;
        longest = max(longest, t.count[q]);
    }
    // Every thread must have read the counts it used before padding starts.
    __syncthreads();
    int size = 2;
    while (size < longest) size <<= 1;
    const int cap = t.cap;
    for (int s = 0; s < nseg; ++s) {
        const int q = segs[s];
        for (int i = t.count[q] + tid; i < size; i += nthreads) t.buf[q * cap + i] = 0ull;
    }
    __syncthreads();
    const int half = size >> 1;
    const int half_log = __ffs(half) - 1;
    const int pairs = nseg * half;
    for (int sz = 2; sz <= size; sz <<= 1) {
        for (int stride = sz >> 1; stride > 0; stride >>= 1) {
            const int stride_log = __ffs(stride) - 1;
            for (int p = tid; p < pairs; p += nthreads) {
                const int seg = p >> half_log;
                const int i = p & (half - 1);
                const int lo = ((i >> stride_log) << (stride_log + 1)) | (i & (stride - 1));
                const int hi = lo + stride;
                u64* b = t.buf + segs[seg] * cap;
                const u64 a = b[lo];
                const u64 c = b[hi];
                const bool descending = (lo & sz) == 0;
                if (descending ? (a < c) : (a > c)) {
                    b[lo] = c;
                    b[hi] = a;
                }
            }
            __syncthreads();
        }
    }
    if (tid < nseg) {
        const int q = segs[tid];
        const int n = t.count[q];
        t.count[q] = n < t.k ? n : t.k;
        t.thr[q] = (n >= t.k) ? t.buf[q * cap + t.k - 1] : 0ull;
    }
    __syncthreads();
}

// Warp-cooperative descending bitonic sort of 32 * E keys held in registers, element index
// lane * E + i. Strides below E swap registers inside a lane; larger strides exchange the
// same register with the partner lane (lane ^ stride / E).
template <int E>
__device__ __forceinline__ void warp_sort_desc_regs(u64 (&v)[E], int lane) {
#pragma unroll
    for (int size = 2; size <= 32 * E; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride < E) {
#pragma unroll
                for (int i = 0; i < E; ++i) {
                    const int j = i ^ stride;
                    if (j > i) {
                        const int e = lane * E + i;
                        const bool descending = (e & size) == 0;
                        const u64 a = v[i];
                        const u64 b = v[j];
                        const bool swap = descending ? (a < b) : (a > b);
                        v[i] = swap ? b : a;
                        v[j] = swap ? a : b;
                    }
                }
            } else {
                const int lane_mask = stride / E;
                const bool lower = (lane & lane_mask) == 0;
#pragma unroll
                for (int i = 0; i < E; ++i) {
                    const int e = lane * E + i;
                    const bool descending = (e & size) == 0;
                    const u64 other = __shfl_xor_sync(0xffffffffu, v[i], lane_mask);
                    const u64 hi = v[i] > other ? v[i] : other;
                    const u64 lo = v[i] > other ? other : v[i];
                    v[i] = (lower == descending) ? hi : lo;
                }
            }
        }
    }
}

// Flushes every query whose buffer could overflow on the next `max_new` offers. Called by
// every thread after a __syncthreads() that follows the last offer. The decision is read by
// all threads before a barrier, so no thread can race ahead and offer again while another is
// still reading the counts.
__device__ __forceinline__ void topk_maybe_flush(const TopkSmem& t, int nq, int max_new,
                                                 int nthreads) {
    uint32_t mask = 0;
    for (int q = 0; q < nq; ++q) {
        if (t.count[q] > t.cap - max_new) mask |= 1u << q;
    }
    __syncthreads();
    topk_flush_mask(t, mask, nthreads);
}

__device__ __forceinline__ void topk_maybe_flush_one(const TopkSmem& t, int q, int max_new,
                                                     int nthreads) {
    const bool need = t.count[q] > t.cap - max_new;
    __syncthreads();
    if (need) topk_flush_mask(t, 1u << q, nthreads);
}

__device__ __forceinline__ void topk_flush_all(const TopkSmem& t, int nq, int nthreads) {
    topk_flush_mask(t, nq >= 32 ? 0xffffffffu : ((1u << nq) - 1u), nthreads);
}

// Merges `lists` sorted descending lists of k keys each (list c of query q at
// src[(q * lists + c) * k]) into the accumulator slot `q_local`, which must be empty.
//
// Prefilter: every list holds k keys >= its own k-th key, so the global k-th key is at least
// T = max over lists of their k-th key. Only the prefix of each list that is >= T can reach
// the result, and it is usually a handful of entries, so the merge touches ~k keys instead of
// lists * k. Lists are walked in lock-step rounds with at most `lists` offers per round.
__device__ inline void topk_merge_lists(const TopkSmem& t, int q_local,
                                        const u64* src, int lists, int nthreads,
                                        u64* s_scratch /* >= 32 entries */) {
    const int tid = threadIdx.x;
    const int k = t.k;
    u64 local_max = 0ull;
    for (int c = tid; c < lists; c += nthreads) {
        const u64 kth = __ldcg(src + static_cast<size_t>(c) * k + (k - 1));
        local_max = kth > local_max ? kth : local_max;
    }
    local_max = warp_max_u64(local_max);
    if ((tid & 31) == 0) s_scratch[tid >> 5] = local_max;
    __syncthreads();
    u64 floor_key = 0ull;
    for (int w = 0; w < (nthreads + 31) / 32; ++w) {
        floor_key = s_scratch[w] > floor_key ? s_scratch[w] : floor_key;
    }
    if (tid == 0) {
        t.count[q_local] = 0;
        t.thr[q_local] = floor_key > 0ull ? floor_key - 1ull : 0ull;
    }
    __syncthreads();
    for (int j = 0; j < k; ++j) {
        bool active = false;
        for (int c = tid; c < lists; c += nthreads) {
            const u64 key = __ldcg(src + static_cast<size_t>(c) * k + j);
            if (key != 0ull && key >= floor_key) {
                active = true;
                topk_offer(t, q_local, key);
            }
        }
        if (!__syncthreads_or(active)) break;
        topk_maybe_flush_one(t, q_local, lists, nthreads);
    }
    __syncthreads();
    topk_flush_mask(t, 1u << q_local, nthreads);
}

// Writes the first k entries of a flushed (sorted, truncated) buffer as ids and scores.
__device__ __forceinline__ void topk_write(const TopkSmem& t, int q_local, int* out_idx,
                                           float* out_scores, int nthreads) {
    const int n = t.count[q_local];
    for (int j = threadIdx.x; j < t.k; j += nthreads) {
        const u64 key = j < n ? t.buf[q_local * t.cap + j] : 0ull;
        out_idx[j] = key_id(key);
        out_scores[j] = key_score(key);
    }
}

}  // namespace zc
