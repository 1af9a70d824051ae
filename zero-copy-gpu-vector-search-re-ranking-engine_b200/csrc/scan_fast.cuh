// Warp-specialised streaming scan for one query per pass (the HBM-bound single-query case).
//
// Same contract and numerics as scan_kernel (scan_kernel.cuh); different schedule, with no
// CTA-wide barrier anywhere between the first and the last tile:
//
//   * Producer warp: keeps an S-deep ring of stages full with bulk copies (rows + per-row
//     scales / mask), waiting on each stage's "empty" mbarrier.
//   * kFastConsumers consumer warps: wait on the stage's "full" mbarrier, score their rows (16
//     lanes per row, two rows per lane group), then one lane arrives on "empty". Scores that
//     beat the CTA threshold are appended to one CTA candidate buffer with a single
//     ballot-aggregated shared atomic per warp iteration. The buffer is zero-initialised
//     shared memory; appends beyond its capacity spill to a per-CTA global area sized for every
//     row the CTA owns, so no score can ever be lost.
//   * Selector warp: follows the buffer as it fills, keeps its own top-k of the keys it has
//     seen (warp bitonic sort) and publishes their k-th key as the CTA threshold. Keys it reads
//     before they are written read as 0, so its threshold is computed from a subset of the
//     candidates and is always a valid lower bound of the CTA's true k-th key.
//   * After the last tile: every candidate at or above the threshold is selected into the CTA
//     list (workspace), and the last CTA of the pass merges the CTA lists (as scan_kernel).
//
// Hybrid variant (LEX = true, one query): the selector's place goes to kFusedLexWarps lexical
// warps that accumulate the BM25 scores of the CTA's documents (lexical_device.cuh, a named
// barrier among themselves) while the producer and consumers stream the dense rows; consumers
// write each row's dense score instead of selecting. The blend needs the lexical maximum over
// every document, so it and the top-k run in the next kernel (hybrid_select.cu), which this one
// lets start early (griddepcontrol). The posting lists are read while HBM streams the rows, so
// the lexical pass costs no time of its own.
#pragma once

#include "scan_kernel.cuh"

namespace zc {

constexpr int kFastConsumers = 16;
constexpr int kFastProducerWarp = kFastConsumers;
constexpr int kFastSelectorWarp = kFastConsumers + 1;
constexpr int kFastThreads = (kFastConsumers + 2) * 32;
// Shared append region per consumer warp (keys), and the whole candidate buffer.
constexpr int kRegionCap = 128;
constexpr int kCandCap = kFastConsumers * kRegionCap;

// Selector buffer: 32 lanes x kSelE registers.
constexpr int kSelE = 8;
constexpr int kSelCap = 32 * kSelE;

// Hybrid variant: lexical warps after the producer (warps kFusedLexWarp0 ...).
constexpr int kFusedLexWarps = 7;
constexpr int kFusedLexWarp0 = kFastConsumers + 1;
constexpr int kFusedLexThreads = kFusedLexWarps * 32;
constexpr int kFusedThreads = (kFastConsumers + 1 + kFusedLexWarps) * 32;

template <int MODE, int JC, bool LEX = false>
__global__ void __launch_bounds__(LEX ? kFusedThreads : kFastThreads, 1) scan_fast_kernel(const ScanParams p) {
    using Traits = ModeTraits<MODE>;
    constexpr int EPC = Traits::kEpc;
    constexpr bool kInt = (MODE == kModeI8R);
    constexpr int LPR = 16;
    constexpr int RPW = 2;                        // lane groups per warp
    constexpr int RW = 2;                         // rows per lane group per iteration
    constexpr int kRowsPerWarp = RPW * RW;
    constexpr int kRowsPerStep = kFastConsumers * kRowsPerWarp;
    constexpr int kGroupShift = 3;                // log2(LPR) - log2(RW)
    constexpr int kThreads = LEX ? kFusedThreads : kFastThreads;
    constexpr int kWarpsAll = kThreads / 32;
    using QElem = typename std::conditional<kInt, int, float>::type;

    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float s_red[kWarpsAll];
    __shared__ float s_qscale[1];
    __shared__ float s_inv;
    __shared__ u64 s_scratch[32];
    __shared__ u64 s_thr;
    __shared__ u64 s_merge_thr;
    __shared__ int s_abort;
    __shared__ int s_done;
    __shared__ int s_last;
    __shared__ int s_merge_count;
    __shared__ int s_sel_count;
    __shared__ int s_sel_complete;
    __shared__ int s_wcount[kFastConsumers];

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int pass = blockIdx.x;                  // one query per pass
    const int cta = blockIdx.y;
    const int G = gridDim.y;
    const int R = p.rows_per_tile;
    const int S = p.stages;
    const int stage_bytes = p.stage_bytes;
    const int k = p.k;

    uint8_t* stages = smem;
    uint8_t* qsmem = smem + p.smem_query_off;
    u64* cbuf = reinterpret_cast<u64*>(smem + p.smem_topk_off);
    u64* sbuf = cbuf + kCandCap;                  // selector buffer, kSelCap keys
    u64* full = reinterpret_cast<u64*>(smem + p.smem_bar_off);
    u64* empty = full + S;
    volatile int* abort_flag = &s_abort;
    volatile u64* cta_thr = &s_thr;

    const int t_begin = static_cast<int>((p.ntiles * cta) / G);
    const int t_end = static_cast<int>((p.ntiles * (cta + 1)) / G);
    const int my_tiles = t_end - t_begin;
    const bool need_side = p.side_scales || p.mask != nullptr;
    // Spill area for this (pass, CTA), one slice per consumer warp with a slot for every row the
    // warp can score.
    const long long warp_rows = static_cast<long long>(my_tiles) * kRowsPerWarp *
                                ((R + kRowsPerStep - 1) / kRowsPerStep);
    unsigned long long* spill = p.spill + (static_cast<size_t>(pass) * G + cta) * p.spill_stride;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kFastConsumers);
        }
        fence_mbarrier_init();
        s_thr = 0ull;
        s_abort = 0;
        s_done = 0;
        s_sel_complete = 0;
        s_inv = (p.lex != nullptr) ? hybrid_inverse(p, pass) : 0.0f;
    }
    if constexpr (LEX) {
        // The select kernel only reads this kernel's outputs after griddepcontrol.wait.
        asm volatile("griddepcontrol.launch_dependents;");
    } else {
        for (int i = tid; i < kCandCap; i += kFastThreads) cbuf[i] = 0ull;
    }
    stage_queries<MODE, 1, kThreads>(p, qsmem, s_qscale, pass, 1, s_red);
    __syncthreads();

    if (warp == kFastProducerWarp) {
        // ---------------- producer warp ----------------
        const u64 stream_policy = l2_policy_evict_first();
        int issued = 0;
        int s = 0;
        uint32_t empty_phase = 0;
        for (int i = 0; i < my_tiles; ++i) {
            if (i >= S) {
                bool ok = true;
                if (lane == 0) {
                    ok = !*abort_flag &&
                         mbar_wait_bounded(&empty[s], empty_phase, p.status, kStatusTileWaitTimeout);
                    if (!ok) *abort_flag = 1;
                }
                if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
            }
            const int row0 = (t_begin + i) * R;
            const int rows = min(R, static_cast<int>(p.n - row0));
            uint8_t* st = stages + s * stage_bytes;
            const bool side_bulk = p.side_tma && rows == R;
            if (need_side && !side_bulk) {
                for (int r = lane; r < rows; r += 32) {
                    if (p.side_scales) reinterpret_cast<float*>(st + p.side_off_scales)[r] = __ldg(p.row_scales + row0 + r);
                    if (p.mask != nullptr) st[p.side_off_mask + r] = __ldg(p.mask + row0 + r);
                }
                __syncwarp();
            }
            if (lane == 0) {
                const uint32_t bytes = static_cast<uint32_t>(rows) * static_cast<uint32_t>(p.row_bytes);
                uint32_t total = bytes;
                if (side_bulk) {
                    if (p.side_scales) total += 4u * R;
                    if (p.mask != nullptr) total += R;
                }
                fence_proxy_async_shared();
                mbar_arrive_expect_tx(&full[s], total);
                bulk_copy_g2s_hint(st, p.corpus + static_cast<size_t>(row0) * p.row_bytes, bytes, &full[s],
                                   stream_policy);
                if (side_bulk) {
                    if (p.side_scales) {
                        bulk_copy_g2s_hint(st + p.side_off_scales, p.row_scales + row0, 4u * R, &full[s],
                                           stream_policy);
                    }
                    if (p.mask != nullptr) {
                        bulk_copy_g2s_hint(st + p.side_off_mask, p.mask + row0, R, &full[s], stream_policy);
                    }
                }
            }
            issued = i + 1;
            __syncwarp();
            if (++s == S) {
                s = 0;
                if (i >= S) empty_phase ^= 1u;
            }
        }
        // If the ring was abandoned, wait (bounded) for every copy still in flight before the
        // CTA can retire.
        if (lane == 0 && *abort_flag) {
            for (int i = max(0, issued - S); i < issued; ++i) {
                mbar_wait_bounded(&full[i % S], static_cast<uint32_t>((i / S) & 1), p.status, kStatusDrainTimeout);
            }
        }
    } else if (!LEX && warp == kFastSelectorWarp) {
        // ---------------- selector warp ----------------
        // Follows the shared buffer and keeps the best keys it has seen in sbuf (kSelCap
        // slots). When sbuf fills it sorts it in registers, keeps k and publishes the k-th key.
        // Polling is bounded in time; giving up only leaves the threshold lower (the result
        // stays exact).
        int scount = 0;
        u64 sthr = 0ull;
        const u64 start = global_timer_ns();
        volatile u64* vbuf = cbuf;
        int pos = 0;                              // lane w < kFastConsumers follows region w
        for (uint32_t spin = 0;; ++spin) {
            const int done = *reinterpret_cast<volatile int*>(&s_done);
            // Keys appended before a consumer counted itself done are visible after this fence.
            __threadfence_block();
            bool progress = false;
            for (;;) {
                const u64 key = (lane < kFastConsumers && pos < kRegionCap) ? vbuf[lane * kRegionCap + pos] : 0ull;
                const bool ready = key != 0ull;
                const uint32_t any = __ballot_sync(0xffffffffu, ready);
                if (any == 0u) break;
                progress = true;
                pos += ready ? 1 : 0;
                const bool take = ready && key > sthr;
                const uint32_t ballot = __ballot_sync(0xffffffffu, take);
                if (take) sbuf[scount + __popc(ballot & ((1u << lane) - 1u))] = key;
                scount += __popc(ballot);
                if (scount > kSelCap - 32 || (sthr == 0ull && scount >= k + 32)) {
                    __syncwarp();
                    // One fixed-width network inside the polling loop (the loop stays small).
                    warp_sort_buffer_e<kSelE>(sbuf, scount, lane);
                    if (scount >= k) {
                        sthr = sbuf[k - 1];
                        if (lane == 0) *cta_thr = sthr;
                    }
                    scount = min(scount, k);
                }
            }
            if (done == kFastConsumers && !progress) {
                if (lane == 0) s_sel_complete = 1;
                break;
            }
            __nanosleep(128);
            if ((spin & 63u) == 0u && global_timer_ns() - start > kWaitBudgetNs) break;
        }
        // sbuf[0, scount) holds the best keys the selector saw (its top k among them, unsorted):
        // the whole CTA ranks them once the scan is over.
        if (lane == 0) s_sel_count = scount;
    } else if (LEX && warp >= kFusedLexWarp0) {
        // ---------------- lexical warps (hybrid variant) ----------------
        if constexpr (LEX) {
            __shared__ long long s_lo[kLexSlots];
            __shared__ long long s_hi[kLexSlots];
            __shared__ float s_lmax[kFusedLexWarps];
            const int ltid = tid - kFusedLexWarp0 * 32;
            const u64 keep_policy = l2_policy_evict_last();
            float* acc = reinterpret_cast<float*>(smem + p.smem_lex_off);
            const long long d_begin = static_cast<long long>(t_begin) * R;
            const int count = static_cast<int>(min(static_cast<long long>(my_tiles) * R, p.n - d_begin));
            const long long total = p.lexi.vec ? __ldg(p.lexi.offsets + p.lexi.vocab) : 0;
            const int* terms = p.lex_terms + static_cast<size_t>(pass) * p.lex_stride;
            float* out = p.lex_out + static_cast<size_t>(pass) * p.n;
            float best = 0.0f;
            // The CTA's documents, lex_window at a time (the accumulator's size).
            for (int w0 = 0; w0 < count; w0 += p.lex_window) {
                const long long d0 = d_begin + w0;
                const int wc = min(p.lex_window, count - w0);
                for (int i = ltid; i < wc; i += kFusedLexThreads) acc[i] = 0.0f;
                for (int t0 = 0; t0 < p.lex_stride; t0 += kLexSlots) {
                    lex_round<kFusedLexThreads, 1>(p.lexi, terms + t0, min(kLexSlots, p.lex_stride - t0), d0, wc, acc,
                                                   s_lo, s_hi, total, ltid);
                }
                lex_sync<kFusedLexThreads, 1>();
                for (int i = ltid; i < wc; i += kFusedLexThreads) {
                    const float v = acc[i];
                    st_global_hint(out + d0 + i, v, keep_policy);  // kept in L2 for the select kernel
                    best = fmaxf(best, v);
                }
                lex_sync<kFusedLexThreads, 1>();  // read out before the next window clears it
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, off));
            if (lane == 0) s_lmax[ltid >> 5] = best;
            lex_sync<kFusedLexThreads, 1>();
            if (ltid == 0) {
                float m = 0.0f;
                for (int w = 0; w < kFusedLexWarps; ++w) m = fmaxf(m, s_lmax[w]);
                atomicMax(p.lex_peak, __float_as_uint(m > 0.0f ? m : 0.0f));
            }
        }
    } else {
        // ---------------- consumer warps ----------------
        const int grp = lane / LPR;
        const int gl = lane % LPR;
        QElem qreg[JC][EPC];
#pragma unroll
        for (int j = 0; j < JC; ++j) {
#pragma unroll
            for (int e = 0; e < EPC; ++e) {
                qreg[j][e] = reinterpret_cast<const QElem*>(qsmem)[(gl + LPR * j) * EPC + e];
            }
        }
        const float qscale = s_qscale[0];
        const float inv = s_inv;
        const u64 keep_policy = LEX ? l2_policy_evict_last() : 0ull;
        const float* lex_row = p.lex != nullptr ? p.lex + static_cast<size_t>(pass) * p.n : nullptr;
        u64* region = cbuf + warp * kRegionCap;
        unsigned long long* wspill = spill + warp * warp_rows;
        int wcount = 0;         // keys this warp appended (replicated in every lane)

        int s = 0;
        uint32_t full_phase = 0;
        for (int i = 0; i < my_tiles; ++i) {
            const int row0 = (t_begin + i) * R;
            const int rows = min(R, static_cast<int>(p.n - row0));
            bool ok = true;
            if (lane == 0) {
                ok = !*abort_flag && mbar_wait_bounded(&full[s], full_phase, p.status, kStatusTileWaitTimeout);
                if (!ok) *abort_flag = 1;
            }
            if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
            const uint8_t* st = stages + s * stage_bytes;
            const float* side_scale = reinterpret_cast<const float*>(st + p.side_off_scales);
            const uint8_t* side_mask = st + p.side_off_mask;
            const uint32_t id0 = p.id_base + static_cast<uint32_t>(row0);
            // The threshold only rises; reading it once per tile keeps it off the row path.
            const u64 thr = *cta_thr;
            const float thr_score = score_from_bits(static_cast<uint32_t>(thr >> 32));
            const bool full_tile = rows == R;

            for (int rb = warp * kRowsPerWarp; rb < rows; rb += kRowsPerStep) {
                // Hybrid: this lane's row's lexical score, loaded before the dot product so
                // its latency overlaps the arithmetic.
                const int r_own = rb + (gl >> kGroupShift) * RPW + grp;
                float lexv = 0.0f;
                if (lex_row != nullptr && (full_tile || r_own < rows)) lexv = __ldg(lex_row + row0 + r_own);
                QElem acc[RW];
#pragma unroll
                for (int rr = 0; rr < RW; ++rr) {
                    acc[rr] = QElem(0);
                    const int r = rb + rr * RPW + grp;
                    if (full_tile || r < rows) {
                        const uint8_t* rowp = st + r * p.stride + gl * 16;
#pragma unroll
                        for (int j = 0; j < JC; ++j) {
                            const uint4 raw = lds128(rowp + LPR * 16 * j);
                            if constexpr (kInt) {
                                acc[rr] = dp4a_chunk(raw, qreg[j], acc[rr]);
                            } else {
                                accumulate_chunk<MODE, false>(raw, qreg[j], p.scale, acc[rr]);
                            }
                        }
                    }
                }
                transpose_reduce<RW, LPR>(acc, lane);
                const int r = rb + (gl >> kGroupShift) * RPW + grp;
                const bool leader = (gl & ((1 << kGroupShift) - 1)) == 0 && (full_tile || r < rows);
                bool take = false;
                u64 key = 0ull;
                if (leader) {
                    float score;
                    if constexpr (kInt) {
                        score = __fmul_rn(__fmul_rn(__int2float_rn(acc[0]), qscale), side_scale[r]);
                    } else {
                        score = acc[0];
                    }
                    if (p.mask != nullptr && side_mask[r] == 0) score = -FLT_MAX;
                    if constexpr (LEX) {
                        // Kept in L2 for the select kernel that reads it next.
                        st_global_hint(p.out_matrix + static_cast<size_t>(pass) * p.n + row0 + r, score, keep_policy);
                    } else {
                        if (lex_row != nullptr) score = hybrid_blend(score, lexv, p.dense_weight, inv);
                        // Cheap float pre-check; only candidates at or above the threshold's
                        // score pay for the exact 64-bit key comparison.
                        if (!(score < thr_score) || thr == 0ull) {
                            key = make_key(score, id0 + r);
                            take = key > thr;
                        }
                    }
                }
                if constexpr (LEX) continue;
                const uint32_t ballot = __ballot_sync(0xffffffffu, take);
                if (take) {
                    const int slot = wcount + __popc(ballot & ((1u << lane) - 1u));
                    if (slot < kRegionCap) {
                        region[slot] = key;
                    } else if (slot - kRegionCap < warp_rows) {
                        wspill[slot - kRegionCap] = key;
                    }
                }
                wcount += __popc(ballot);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive_cta(&empty[s]);
            if (++s == S) {
                s = 0;
                full_phase ^= 1u;
            }
        }
        if (lane == 0) {
            s_wcount[warp] = wcount;
            __threadfence_block();
            atomicAdd(&s_done, 1);
        }
    }
    if constexpr (LEX) return;
    __syncthreads();

    // The stage ring (free now) holds the merge buffer.
    TopkSmem mt;
    mt.buf = reinterpret_cast<u64*>(stages);
    mt.count = &s_merge_count;
    mt.thr = &s_merge_thr;
    mt.cap = p.cap_final;
    mt.k = k;
    // When no warp spilled and the selector followed every region to the end, it has seen
    // every candidate: its sorted buffer already is this CTA's list.
    bool spilled = false;
    for (int w = 0; w < kFastConsumers; ++w) spilled |= s_wcount[w] > kRegionCap;
    if (!spilled && s_sel_complete) {
        // Its keys are distinct: each one's rank among them is its place in the sorted list.
        unsigned long long* dst = p.lists + (static_cast<size_t>(pass) * G + cta) * k;
        const int n = s_sel_count;
        for (int i = tid; i < n; i += kFastThreads) {
            const u64 key = sbuf[i];
            const int r = key_rank(sbuf, n, key);
            if (r < k) dst[r] = key;
        }
        for (int j = min(n, k) + tid; j < k; j += kFastThreads) dst[j] = 0ull;
    } else {
    // Otherwise select this CTA's top-k from every candidate at or above the selector's
    // threshold: the shared regions first, then any spill.
    const u64 floor_key = s_thr;
    if (tid == 0) {
        s_merge_count = 0;
        s_merge_thr = floor_key > 0ull ? floor_key - 1ull : 0ull;
    }
    __syncthreads();
    // All shared regions in one wide round, then any warp's spill slice (rare).
    topk_offer_all<4>(mt, 0, kCandCap, floor_key, [&](int i) {
        const int w = i / kRegionCap;
        return (i - w * kRegionCap) < s_wcount[w] ? cbuf[i] : 0ull;
    }, kFastThreads);
    for (int w = 0; w < kFastConsumers; ++w) {
        const int extra = static_cast<int>(min(static_cast<long long>(s_wcount[w]) - kRegionCap, warp_rows));
        topk_offer_all<4>(mt, 0, extra, floor_key,
                          [&](int i) { return __ldcg(spill + w * warp_rows + i); }, kFastThreads);
    }
    __syncthreads();
    topk_flush_mask(mt, 1u, kFastThreads);
    {
        unsigned long long* dst = p.lists + (static_cast<size_t>(pass) * G + cta) * k;
        const int n = s_merge_count;
        for (int j = tid; j < k; j += kFastThreads) dst[j] = j < n ? mt.buf[j] : 0ull;
    }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned int ticket = atomicAdd(&p.counters[pass], 1u);
        s_last = (ticket == static_cast<unsigned int>(G - 1)) ? 1 : 0;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const unsigned long long* src = p.lists + static_cast<size_t>(pass) * G * k;
    topk_merge_lists(mt, 0, src, G, kFastThreads, s_scratch);
    topk_write(mt, 0, p.out_idx + static_cast<size_t>(pass) * k, p.out_scores + static_cast<size_t>(pass) * k,
               kFastThreads);
    __syncthreads();
    if (tid == 0) p.counters[pass] = 0u;
}

}  // namespace zc
