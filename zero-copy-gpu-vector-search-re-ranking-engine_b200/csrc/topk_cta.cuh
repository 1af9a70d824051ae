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

// Warp-cooperative descending bitonic sort of 32 * E keys held in registers, element index
// lane * E + i. Strides below E swap registers inside a lane; larger strides exchange the
// same register with the partner lane (lane ^ stride / E). T: any unsigned key type.
template <int E, typename T = u64>
__device__ __forceinline__ void warp_sort_desc_regs(T (&v)[E], int lane) {
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
                        const T a = v[i];
                        const T b = v[j];
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
                    const T other = __shfl_xor_sync(0xffffffffu, v[i], lane_mask);
                    const T hi = v[i] > other ? v[i] : other;
                    const T lo = v[i] > other ? other : v[i];
                    v[i] = (lower == descending) ? hi : lo;
                }
            }
        }
    }
}

// Sorts the first n (<= 32 * E) keys of a shared buffer descending with one warp; entries
// [n, 32 * E) become 0.
template <int E>
__device__ __forceinline__ void warp_sort_buffer_e(u64* buf, int n, int lane) {
    u64 v[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int at = lane * E + e;
        v[e] = at < n ? buf[at] : 0ull;
    }
    warp_sort_desc_regs<E>(v, lane);
    __syncwarp();
#pragma unroll
    for (int e = 0; e < E; ++e) buf[lane * E + e] = v[e];
    __syncwarp();
}

// One warp sorts the first n (<= 256) keys of a shared buffer descending, with a network only
// as wide as n needs (32, 64, 128 or 256 keys): a single warp's sort is a chain of dependent
// shuffles, so its cost follows the width.
static __device__ __noinline__ void warp_sort_buffer(u64* buf, int n, int lane) {
    if (n <= 32) {
        warp_sort_buffer_e<1>(buf, n, lane);
    } else if (n <= 64) {
        warp_sort_buffer_e<2>(buf, n, lane);
    } else if (n <= 128) {
        warp_sort_buffer_e<4>(buf, n, lane);
    } else {
        warp_sort_buffer_e<8>(buf, n, lane);
    }
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

// Offers every key >= floor_key among `total` keys, key i fetched by get(i), into slot q.
// Each thread holds U independent fetches in flight per round, so a round costs one memory
// latency however many keys it covers; the buffer is flushed between rounds when needed.
// Requires t.cap >= t.k + U * nthreads. Called by every thread of the CTA.
template <int U, typename Get>
__device__ void topk_offer_all(const TopkSmem& t, int q, int total, u64 floor_key, Get get,
                               int nthreads) {
    const int lane = threadIdx.x & 31;
    for (int base = 0; base < total; base += nthreads * U) {
        u64 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = base + u * nthreads + static_cast<int>(threadIdx.x);
            v[u] = i < total ? get(i) : 0ull;
        }
        // Keep every fetch of the round ahead of the first offer: without this the compiler
        // sinks each load next to its (atomic) offer and the round pays one memory latency
        // per key instead of one in total.
        asm volatile("" ::: "memory");
        const u64 thr = t.thr[q];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const bool take = v[u] != 0ull && v[u] >= floor_key && v[u] > thr;
            const uint32_t ballot = __ballot_sync(0xffffffffu, take);
            if (ballot != 0u) {
                int slot = 0;
                if (lane == 0) slot = atomicAdd(&t.count[q], __popc(ballot));
                slot = __shfl_sync(0xffffffffu, slot, 0) + __popc(ballot & ((1u << lane) - 1u));
                if (take) t.buf[q * t.cap + slot] = v[u];
            }
        }
        __syncthreads();
        topk_maybe_flush_one(t, q, U * nthreads, nthreads);
    }
}

// Merges `lists` sorted descending lists of k keys each (list c at src[c * k]) into slot
// q_local of the accumulator, which must be empty and have cap >= k + nthreads and
// cap >= next_pow2(lists) (rounds are 8, 2 or 1 keys per thread wide, whichever the capacity
// allows).
//
// Floor: pick j with lists * (j + 1) >= k and let m = ceil(k / (j + 1)). The m-th largest of
// the lists' j-th keys, F, has m lists each holding j + 1 keys >= F, i.e. at least k keys, so
// the merged k-th key is >= F and only keys >= F are offered. For many short lists (one per
// CTA) j = 0: F is the k-th largest list head, which leaves a few hundred candidates out of
// lists * k.
//
// Small k (<= 16, at most 256 lists, all lists fitting the buffer next to 256 candidates): the
// lists are copied into the buffer, one warp sorts their heads for F (the k-th largest head, so
// exactly k lists hold keys >= F and at most k * k keys pass), the CTA keeps the keys >= F and
// one warp sorts them. This replaces two CTA-wide bitonic sorts (a barrier per stage) with two
// short single-warp ones.
__device__ inline bool topk_merge_lists_small(const TopkSmem& t, int q_local, const u64* src, int lists,
                                              int nthreads, u64* s_scratch) {
    const int k = t.k;
    const int total = lists * k;
    if (k > 16 || lists > 256 || total + 256 > t.cap) return false;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    u64* all = t.buf + q_local * t.cap;  // [total] list keys
    u64* cand = all + total;             // [256] heads, then the keys >= F
    for (int i = tid; i < total; i += nthreads) all[i] = __ldcg(src + i);
    if (tid == 0) t.count[q_local] = 0;
    __syncthreads();
    if (tid < 32) {
        for (int c = lane; c < lists; c += 32) cand[c] = all[c * k];
        __syncwarp();
        warp_sort_buffer(cand, lists, lane);
        // With fewer than k non-empty lists the floor is 1: every non-empty key (fewer than
        // k * k of them) passes.
        if (lane == 0) s_scratch[0] = (lists >= k && cand[k - 1] > 1ull) ? cand[k - 1] : 1ull;
    }
    __syncthreads();
    const u64 floor_key = s_scratch[0];
    for (int i = tid; i < total; i += nthreads) {
        const u64 key = all[i];
        if (key >= floor_key) {
            const int slot = atomicAdd(&t.count[q_local], 1);
            if (slot < 256) cand[slot] = key;
        }
    }
    __syncthreads();
    if (tid < 32) {
        const int n = min(t.count[q_local], 256);
        warp_sort_buffer(cand, n, lane);
        const int kept = min(n, k);
        if (lane < kept) all[lane] = cand[lane];
        __syncwarp();
        if (lane == 0) {
            t.count[q_local] = kept;
            t.thr[q_local] = n >= k ? cand[k - 1] : 0ull;
        }
    }
    __syncthreads();
    return true;
}

// How many of the n distinct keys in keys[] (shared memory) are larger than key (its rank, 0 =
// largest). All lanes of a warp read the same entries at once (broadcasts). Eight keys per step
// in four 16-byte loads (when keys[] is 16-byte aligned) into independent counters, so the loads
// of a step are in flight together instead of one shared-memory latency per key.
__device__ __forceinline__ int key_rank(const u64* keys, int n, u64 key) {
    int r[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int j = 0;
    if ((reinterpret_cast<uintptr_t>(keys) & 15u) == 0) {
        const ulonglong2* k2 = reinterpret_cast<const ulonglong2*>(keys);
        for (; j + 8 <= n; j += 8) {
            ulonglong2 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = k2[j / 2 + u];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                r[2 * u] += v[u].x > key ? 1 : 0;
                r[2 * u + 1] += v[u].y > key ? 1 : 0;
            }
        }
    }
    for (; j < n; ++j) r[0] += keys[j] > key ? 1 : 0;
    return ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
}

// Lists at least as many as k: the floor F is the k-th largest list head (found by counting
// ranks, one head per thread), so exactly k lists hold keys >= F and only their prefixes >= F
// are read (a warp per list, 32 keys per step); the kept keys are placed by counting ranks
// instead of sorting. A CTA-wide bitonic network costs a barrier per stage, and its input would
// be every key of the lists. Falls back (returns false) when the candidates outgrow kMergeCand.
constexpr int kMergeCand = 2048;

__device__ inline bool topk_merge_lists_rank(const TopkSmem& t, int q_local, const u64* src, int lists,
                                             int nthreads, u64* s_scratch) {
    const int k = t.k;
    const int lists_pad = (lists + 31) & ~31;
    if (lists < k || lists > nthreads || kMergeCand + lists_pad + k > t.cap) return false;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int nwarps = nthreads >> 5;
    u64* cand = t.buf + q_local * t.cap;  // [kMergeCand] keys >= F
    u64* heads = cand + kMergeCand;       // [lists]
    u64* kept = heads + lists_pad;        // [k] the result, before it moves to the front
    if (tid < lists) heads[tid] = __ldcg(src + static_cast<size_t>(tid) * k);
    if (tid == 0) {
        s_scratch[0] = 1ull;  // F when fewer than k lists are non-empty: every non-empty key
        t.count[q_local] = 0;
    }
    __syncthreads();
    if (tid < lists) {
        const u64 h = heads[tid];
        if (h != 0ull && key_rank(heads, lists, h) == k - 1) s_scratch[0] = h;
    }
    __syncthreads();
    const u64 floor_key = s_scratch[0];
    // Keys >= F: a prefix of each list whose head is >= F. A warp takes lists warp,
    // warp + nwarps, ...; the first 32 keys of up to kPre of them are read at once.
    bool overflow = false;
    auto append = [&](u64 key) {  // warp-wide; returns whether all 32 lanes took a key
        const bool take = key >= floor_key;
        const uint32_t ballot = __ballot_sync(0xffffffffu, take);
        int slot = 0;
        if (lane == 0 && ballot != 0u) slot = atomicAdd(&t.count[q_local], __popc(ballot));
        slot = __shfl_sync(0xffffffffu, slot, 0) + __popc(ballot & ((1u << lane) - 1u));
        if (take) {
            if (slot < kMergeCand) {
                cand[slot] = key;
            } else {
                overflow = true;
            }
        }
        return ballot == 0xffffffffu;
    };
    constexpr int kPre = 8;
    for (int l0 = warp; l0 < lists; l0 += nwarps * kPre) {
        u64 first[kPre];
#pragma unroll
        for (int u = 0; u < kPre; ++u) {
            const int l = l0 + u * nwarps;
            first[u] = (l < lists && heads[l] >= floor_key && lane < k) ? __ldcg(src + static_cast<size_t>(l) * k + lane)
                                                                        : 0ull;
        }
#pragma unroll
        for (int u = 0; u < kPre; ++u) {
            const int l = l0 + u * nwarps;
            if (l >= lists || heads[l] < floor_key) continue;  // uniform in the warp
            if (!append(first[u])) continue;                   // the prefix ended in the first 32
            for (int off = 32; off < k; off += 32) {
                const u64 key = off + lane < k ? __ldcg(src + static_cast<size_t>(l) * k + off + lane) : 0ull;
                if (!append(key)) break;
            }
        }
    }
    if (__syncthreads_or(overflow ? 1 : 0)) return false;
    const int n = t.count[q_local];
    // Exact top k by rank (keys are distinct), then to the front of the buffer.
    for (int i = tid; i < n; i += nthreads) {
        const u64 key = cand[i];
        const int r = key_rank(cand, n, key);
        if (r < k) kept[r] = key;
    }
    __syncthreads();
    const int got = min(n, k);
    for (int j = tid; j < got; j += nthreads) t.buf[q_local * t.cap + j] = kept[j];
    __syncthreads();
    if (tid == 0) {
        t.count[q_local] = got;
        t.thr[q_local] = n >= k ? t.buf[q_local * t.cap + k - 1] : 0ull;
    }
    __syncthreads();
    return true;
}

__device__ inline void topk_merge_lists(const TopkSmem& t, int q_local, const u64* src, int lists,
                                        int nthreads, u64* s_scratch /* >= 32 entries */) {
    if (topk_merge_lists_rank(t, q_local, src, lists, nthreads, s_scratch)) return;
    if (topk_merge_lists_small(t, q_local, src, lists, nthreads, s_scratch)) return;
    const int tid = threadIdx.x;
    const int k = t.k;
    const int j = (k + lists - 1) / lists - 1;
    const int m = (k + j) / (j + 1);
    int width = 2;
    while (width < lists) width <<= 1;
    // Sort the lists' j-th keys (descending) in the front of the buffer; F = entry m - 1.
    u64* heads = t.buf + q_local * t.cap;
    for (int c = tid; c < width; c += nthreads) {
        heads[c] = c < lists ? __ldcg(src + static_cast<size_t>(c) * k + j) : 0ull;
    }
    if (tid == 0) t.count[q_local] = width;
    __syncthreads();
    topk_flush_mask(t, 1u << q_local, nthreads);    // sorts `width` keys; keeps min(width, k)
    const u64 floor_key = heads[m - 1];
    __syncthreads();
    if (tid == 0) {
        t.count[q_local] = 0;
        t.thr[q_local] = floor_key > 0ull ? floor_key - 1ull : 0ull;
    }
    __syncthreads();
    auto fetch = [&](int i) { return __ldcg(src + i); };
    if (t.cap >= k + 8 * nthreads) {
        topk_offer_all<8>(t, q_local, lists * k, floor_key, fetch, nthreads);
    } else if (t.cap >= k + 2 * nthreads) {
        topk_offer_all<2>(t, q_local, lists * k, floor_key, fetch, nthreads);
    } else {
        topk_offer_all<1>(t, q_local, lists * k, floor_key, fetch, nthreads);
    }
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
