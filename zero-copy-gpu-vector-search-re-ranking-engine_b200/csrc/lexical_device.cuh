// Device code of the BM25 accumulation over a CSR inverted index, shared by lexical_kernel (a
// whole CTA per document range, lexical.cu) and the hybrid scan (a group of warps per CTA that
// works beside the dense scan's warps, scan_fast.cuh).
//
// A group of THREADS threads owns the documents [d0, d0 + count) and a shared-memory
// accumulator acc[count]. For each round of up to kLexSlots query term slots:
//
//   * a warp per slot finds the group's slice of the term's posting list with a 32-way search
//     (about log32(df) dependent loads); posting lists are sorted by document within each term,
//     as the reference builder writes them (python/zcgvs_tools/build_lexical.py:143-162);
//   * the slices are added into acc in slot order, a group barrier closing each slot. A run of
//     equal document ids (possible in hand-made indexes) is summed by one thread in posting
//     order, so every document's score is the exact sequential sum in (slot, posting) order: the
//     CPU loop of tests/cpp/test_lexical.cu:71-80. The reference (src/cuda/lexical.cu:17-41)
//     scatter-adds with float atomicAdd instead, whose order changes from run to run.
//   * Indexes whose postings are in any order (the reference launcher's contract) take a slow
//     path with the same sums: one warp walks each term's whole list in posting order, grouping
//     equal documents of a 32-posting step (match_any) and adding them in lane order.
#pragma once

#include <cuda_runtime.h>

#include <climits>

#include "common.cuh"

namespace zc {

// The CSR index as the kernels read it.
struct LexIndex {
    const long long* offsets;   // [vocab + 1]
    const int* docs;            // posting document ids
    const float* weights;       // posting BM25 weights
    int vocab;
    long long n;                // documents
    int sorted;                 // postings sorted by document within each term (else: any order)
    int vec;                    // sorted, docs and weights 16-byte aligned: 16-byte posting loads
};

constexpr int kLexSlots = 128;  // term slots searched per round

// First index in [lo, hi) whose document id is >= target (hi if none), for sorted docs[].
// Whole warp; 32 probes per step.
__device__ __forceinline__ long long lower_bound_warp(const int* __restrict__ docs, long long lo, long long hi,
                                                      int target, int lane) {
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
__device__ __forceinline__ long long lower_bound_hint(const int* __restrict__ docs, long long lo, long long hi,
                                                      int target, long long guess, long long step, int lane) {
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

// Barrier of the lexical group: the whole CTA (BAR == 0) or named barrier BAR over THREADS
// threads (the hybrid scan's lexical warps; its other warps never wait on it).
template <int THREADS, int BAR>
__device__ __forceinline__ void lex_sync() {
    if constexpr (BAR == 0) {
        __syncthreads();
    } else {
        asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(THREADS) : "memory");
    }
}

// Adds the postings of terms[0, slots) (slots <= kLexSlots) that fall in [d0, d0 + count) into
// acc, by the group's THREADS threads (tid = index inside the group). s_lo / s_hi: kLexSlots
// shared entries. `total` = offsets[vocab] when p.vec (the index's end, which the 16-byte loads
// never pass). Starts with a group barrier (the previous round's slices are consumed); a thread
// that reads another thread's entries of acc after the last round needs one more.
template <int THREADS, int BAR>
__device__ void lex_round(const LexIndex& p, const int* __restrict__ terms, int slots, long long d0, int count,
                          float* acc, long long* s_lo, long long* s_hi, long long total, int tid) {
    constexpr int kWarps = THREADS / 32;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    lex_sync<THREADS, BAR>();
    for (int t = warp; t < slots; t += kWarps) {
        const int term = __ldg(terms + t);
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
    lex_sync<THREADS, BAR>();
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
        lex_sync<THREADS, BAR>();
        return;
    }
    if (!p.vec) {
        for (int t = 0; t < slots; ++t) {
            const long long lo = s_lo[t];
            const long long hi = s_hi[t];
            for (long long i = lo + tid; i < hi; i += THREADS) {
                const int doc = __ldg(p.docs + i);
                if (i > lo && __ldg(p.docs + i - 1) == doc) continue;  // not the head of its run
                float a = acc[doc - d0];
                a = __fadd_rn(a, __ldg(p.weights + i));
                for (long long j = i + 1; j < hi && __ldg(p.docs + j) == doc; ++j) {
                    a = __fadd_rn(a, __ldg(p.weights + j));
                }
                acc[doc - d0] = a;
            }
            lex_sync<THREADS, BAR>();  // slot t's additions land before slot t + 1's
        }
        return;
    }
    // 16-byte posting groups, software-pipelined across slots. A step is one group per thread of
    // one slot (thread tid owns group g0 + tid); the loads of the next two steps are in flight
    // while a step's additions run, across the barrier that closes a slot (loads never touch the
    // accumulator), so a slot's memory latency overlaps the work of the slots before it. Slots
    // without postings here are skipped. A posting is the head of its run unless the posting
    // before it (the same thread's, the previous lane's last one, or for lane 0 a load) holds the
    // same document; it continues a run when the posting after it (the same thread's, the next
    // lane's first one, or for lane 31 a load) does, which only hand-made indexes have.
    struct Step {
        int t;
        long long g0;
    };
    struct Group {
        int4 dv;
        float4 wv;
        int before;
        int after;
    };
    auto g_lo = [&](int t) { return s_lo[t] >> 2; };
    auto g_hi = [&](int t) { return (s_hi[t] + 3) >> 2; };
    auto first_from = [&](int t) {
        while (t < slots && g_lo(t) >= g_hi(t)) ++t;
        return Step{t, t < slots ? g_lo(t) : 0};
    };
    auto advance = [&](Step c) {
        if (c.t >= slots) return c;
        const long long g0 = c.g0 + THREADS;
        return g0 < g_hi(c.t) ? Step{c.t, g0} : first_from(c.t + 1);
    };
    auto load = [&](Step c, Group& b) {
        b.dv = make_int4(-1, -1, -1, -1);
        b.wv = make_float4(0.f, 0.f, 0.f, 0.f);
        b.before = -1;
        b.after = -1;
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
        if (lane == 31 && 4 * g + 4 < s_hi[c.t]) b.after = __ldg(p.docs + 4 * g + 4);
    };
    auto process = [&](Step c, const Group& b) {
        const long long g = c.g0 + tid;
        const int up = __shfl_up_sync(0xffffffffu, b.dv.w, 1);
        const int down = __shfl_down_sync(0xffffffffu, b.dv.x, 1);
        if (g >= g_hi(c.t)) return;
        // Elements [eb, ee) of this group lie in the slot's slice (eb > 0 only in its first
        // group, ee < 4 only in its last); element eb is the slice's first posting when
        // at_lo.
        const long long base = 4 * g;
        const long long lo = s_lo[c.t];
        const long long hi = s_hi[c.t];
        const bool at_lo = lo >= base;
        const int eb = at_lo ? static_cast<int>(lo - base) : 0;
        const int ee = static_cast<int>(min(hi - base, 4LL));
        const int d[4] = {b.dv.x, b.dv.y, b.dv.z, b.dv.w};
        const float w[4] = {b.wv.x, b.wv.y, b.wv.z, b.wv.w};
        const int prev0 = lane == 0 ? b.before : up;
        const int next3 = lane == 31 ? b.after : down;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            if (e < eb || e >= ee) continue;
            const int doc = d[e];
            const int prev = e == 0 ? prev0 : d[e - 1];
            if (!(e == eb && at_lo) && prev == doc) continue;  // a run's later posting
            float a = __fadd_rn(acc[doc - d0], w[e]);
            const bool run = e < 3 ? (e + 1 < ee && d[e + 1] == doc) : (base + 4 < hi && next3 == doc);
            if (run) {
                // The rest of a run of equal documents, in posting order (hand-made indexes).
                for (long long j = base + e + 1; j < hi && __ldg(p.docs + j) == doc; ++j) {
                    a = __fadd_rn(a, __ldg(p.weights + j));
                }
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
        if (s1.t != s0.t) lex_sync<THREADS, BAR>();  // slot s0.t's additions land before the next slot's
        s0 = s1;
        s1 = s2;
        b0 = b1;
        b1 = b2;
    }
}

}  // namespace zc
