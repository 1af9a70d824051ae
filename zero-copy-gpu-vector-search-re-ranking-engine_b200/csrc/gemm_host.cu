// Host side and helper kernels of the tensor-core batched search (gemm_scan.cuh).
//
// zcgvs_gemm_topk runs these kernels on one stream, all on the caller's workspace:
//   1. prep      : queries -> fp16 (ZCGVS_DTYPE_F16), per-row int8 + scale (ZCGVS_DTYPE_I8_ROW,
//                  the quantiser of the streaming scan), or int8 -2 / +2 per sign with the sum
//                  of the signs (ZCGVS_DTYPE_BINARY) in the layout the TMA loads read.
//   2. sample    : the tensor-core scan over the first T document tiles, writing each query's
//                  maximum score per 32-document chunk.
//   3. threshold : per query, from those chunk maxima: the safe bound, the k-th largest (k
//                  chunks each hold a document scoring >= it, so every member of the exact top-k
//                  scores >= it), and a tighter statistical bound, the 16th largest, which a
//                  sample of T = 16 / E of the tiles places so that about E documents of the whole
//                  corpus pass it. The filter starts with the tighter of the two.
//   4. filter    : the tensor-core scan over all tiles; every document whose key (score, id) is
//                  >= its query's threshold key goes to the CTA's mailbox (a shared-memory
//                  reservation and plain stores: the epilogue never waits on a global atomic).
//      bucket    : mailbox entries -> per-query candidate buffers (parallel global atomics).
//   5. select    : per query, the exact (score desc, id asc) top-k of its candidates.
//   6. retry     : the result of a query is exact when at least k candidates passed a bound and
//                  none were lost. Otherwise the query is scanned again: with the safe bound when
//                  a statistical bound let fewer than k through, or with its threshold raised to
//                  the k-th largest key it did capture (k captured documents bound the k-th best
//                  from below) when its candidates overflowed a buffer. The retry scans only the
//                  query blocks holding such a query and returns at once when there is none, so
//                  the launch sequence is fixed (capturable in a CUDA graph).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cfloat>
#include <climits>
#include <string>

#include "gemm_scan.cuh"
#include "host_common.h"
#include "topk_cta.cuh"
#include "zcgvs_sm100.h"

namespace zc {
namespace gemm {

namespace {

constexpr int kCandCap = 16384;
static_assert(kStatusOverflow == ZCGVS_DEVICE_CANDIDATE_OVERFLOW && kStatusTmemWait == ZCGVS_DEVICE_TMEM_WAIT_TIMEOUT,
              "device status bits must match the header");

// Per-query candidate buffer entries a search uses: kCandCap, or a smaller test cap
// (zcgvs_test_set_candidate_cap). The workspace layout always reserves kCandCap per query.
std::atomic<int> g_test_cand_cap{0};
int cand_cap() {
    const int cap = g_test_cand_cap.load(std::memory_order_relaxed);
    return cap > 0 ? cap : kCandCap;
}
constexpr int kStatRank = 16;  // rank of the statistical threshold among the sample's chunk maxima
constexpr int kPasses = 3;     // the filter pass and up to two retries
constexpr int kSelectThreads = 512;
constexpr int kSelectCap = 4096;  // selection buffer (32 KB): k (<= 1024) + 4 keys per thread per round
constexpr size_t kAlign = 256;

int operand_row_bytes(int mode, int dtype, int dim) {
    return mode == kModeBin ? dim : static_cast<int>(row_bytes_of(dtype, dim));
}

// Queries -> the MMA operand layout: fp16 rows, or int8 rows with a per-row scale computed
// exactly as the streaming scan's quantiser (scan_kernel.cuh, stage_queries), or for 1-bit
// corpora the row q'[p] = -2 s (s = +1 where the query value is >= 0, the sign bit of
// src/cuda/convert.cu:34-53, else -1) of dimension 32 w + 8 i + j at position 32 w + 4 j + i
// (the expanders' byte order) and qscale = the sum of the signs.
template <int MODE>
__global__ void prep_queries_kernel(const float* __restrict__ queries, int dim, void* out, float* qscale) {
    __shared__ float s_red[8];
    __shared__ float s_scale;
    __shared__ int s_sum[8];
    const int q = blockIdx.x;
    const float* src = queries + static_cast<size_t>(q) * dim;
    if constexpr (MODE == kModeBin) {
        int8_t* dst = static_cast<int8_t*>(out) + static_cast<size_t>(q) * dim;
        int sum = 0;
        for (int pos = threadIdx.x; pos < dim; pos += blockDim.x) {
            const int r = pos & 31;
            const int d = (pos & ~31) + 8 * (r & 3) + (r >> 2);
            const bool set = src[d] >= 0.0f;
            dst[pos] = static_cast<int8_t>(set ? -2 : 2);
            sum += set ? 1 : -1;
        }
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if ((threadIdx.x & 31) == 0) s_sum[threadIdx.x >> 5] = sum;
        __syncthreads();
        if (threadIdx.x == 0) {
            int total = 0;
            for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) total += s_sum[w];
            qscale[q] = static_cast<float>(total);
        }
    } else if constexpr (MODE == kModeF16) {
        __half* dst = static_cast<__half*>(out) + static_cast<size_t>(q) * dim;
        for (int j = threadIdx.x; j < dim; j += blockDim.x) dst[j] = __float2half_rn(src[j]);
    } else {
        float m = 0.0f;
        for (int j = threadIdx.x; j < dim; j += blockDim.x) m = fmaxf(m, fabsf(src[j]));
        m = warp_max_f32(m);
        if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = m;
        __syncthreads();
        if (threadIdx.x == 0) {
            float mm = 0.0f;
            for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) mm = fmaxf(mm, s_red[w]);
            s_scale = mm > 0.0f ? __fdiv_rn(mm, 127.0f) : 1.0f;
            qscale[q] = s_scale;
        }
        __syncthreads();
        const float inv = __fdiv_rn(1.0f, s_scale);
        int8_t* dst = static_cast<int8_t*>(out) + static_cast<size_t>(q) * dim;
        for (int j = threadIdx.x; j < dim; j += blockDim.x) {
            const float r = rintf(__fmul_rn(src[j], inv));
            dst[j] = static_cast<int8_t>(fminf(fmaxf(r, -127.0f), 127.0f));
        }
    }
}

// thr_key[q] = the smallest key of the k-th largest chunk maximum's score (0, i.e. keep every
// document, with fewer than k chunks); clears the candidate counter and the done flag of q;
// block 0 clears the retry flag.
__global__ void __launch_bounds__(kSelectThreads) threshold_kernel(const float* __restrict__ chunk_max, int chunks,
                                                                   int k, int cap, unsigned long long* thr_key,
                                                                   unsigned long long* thr_safe,
                                                                   unsigned int* cand_count, int* done,
                                                                   unsigned int* retry, unsigned int* mneed,
                                                                   int mtiles) {
    extern __shared__ __align__(16) u64 keys[];
    __shared__ int s_count;
    __shared__ u64 s_thr;
    const int q = blockIdx.x;
    TopkSmem t;
    t.buf = keys;
    t.count = &s_count;
    t.thr = &s_thr;
    t.cap = cap;
    t.k = max(k, kStatRank);
    if (threadIdx.x == 0) {
        s_count = 0;
        s_thr = 0ull;
    }
    __syncthreads();
    const float* row = chunk_max + static_cast<size_t>(q) * chunks;
    topk_offer_all<4>(t, 0, chunks, 0ull, [&](int i) { return make_key(row[i], static_cast<uint32_t>(i)); },
                      kSelectThreads);
    topk_flush_mask(t, 1u, kSelectThreads);
    __syncthreads();
    if (threadIdx.x == 0) {
        // keys[r - 1] holds the r-th largest when there are at least r chunks (r <= t.k).
        auto bound = [&](int r) {
            const float score = chunks >= r ? key_score(keys[r - 1]) : -INFINITY;
            return score > -INFINITY ? (static_cast<u64>(orderable_bits(score)) << 32) : 0ull;
        };
        const u64 safe = bound(k);
        thr_safe[q] = safe;
        thr_key[q] = kStatRank < k ? max(bound(kStatRank), safe) : safe;
        if (q < mtiles) {
            for (int i = 0; i < kPasses; ++i) mneed[i * mtiles + q] = 0u;
        }
        cand_count[q] = 0u;
        done[q] = 0;
        if (q == 0) {
            for (int i = 0; i < 2 * kPasses; ++i) retry[i] = 0u;  // retry requests, mailbox overflows
        }
    }
}

// threshold_kernel for samples of at most kThrRegs * 32 chunks: one warp per query holds the
// query's chunk maxima in registers (as orderable bits) and builds the r-th largest bit by bit
// from the top, keeping a bit when at least r maxima are at or above the candidate; the same
// bounds without a sort. Padding slots hold 0, below every float's orderable bits.
constexpr int kThrRegs = 64;
constexpr int kThrWarps = 2;  // small blocks: a 64-query batch spreads over 32 SMs

__global__ void __launch_bounds__(kThrWarps * 32) threshold_regs_kernel(const float* __restrict__ chunk_max,
                                                                        int chunks, int k, int batch,
                                                                        unsigned long long* thr_key,
                                                                        unsigned long long* thr_safe,
                                                                        unsigned int* cand_count, int* done,
                                                                        unsigned int* retry, unsigned int* mneed,
                                                                        int mtiles) {
    const int lane = threadIdx.x & 31;
    const int q = blockIdx.x * kThrWarps + (threadIdx.x >> 5);
    if (q >= batch) return;
    const float* row = chunk_max + static_cast<size_t>(q) * chunks;
    uint32_t v[kThrRegs];
#pragma unroll
    for (int j = 0; j < kThrRegs; ++j) {
        const int i = j * 32 + lane;
        v[j] = i < chunks ? orderable_bits(__ldg(row + i)) : 0u;
    }
    auto rth = [&](int r) -> uint32_t {
        uint32_t t = 0u;
        for (int bit = 31; bit >= 0; --bit) {
            const uint32_t cand = t | (1u << bit);
            int c = 0;
#pragma unroll
            for (int j = 0; j < kThrRegs; ++j) c += v[j] >= cand ? 1 : 0;
            if (__reduce_add_sync(0xffffffffu, c) >= r) t = cand;
        }
        return t;
    };
    const uint32_t neg_inf = orderable_bits(-INFINITY);
    auto bound = [&](int r) -> u64 {
        if (chunks < r) return 0ull;
        const uint32_t t = rth(r);
        return t > neg_inf ? (static_cast<u64>(t) << 32) : 0ull;
    };
    const u64 safe = bound(k);
    const u64 key = kStatRank < k ? max(bound(kStatRank), safe) : safe;
    if (lane == 0) {
        thr_safe[q] = safe;
        thr_key[q] = key;
        if (q < mtiles) {
            for (int i = 0; i < kPasses; ++i) mneed[i * mtiles + q] = 0u;
        }
        cand_count[q] = 0u;
        done[q] = 0;
        if (q == 0) {
            for (int i = 0; i < 2 * kPasses; ++i) retry[i] = 0u;  // retry requests, mailbox overflows
        }
    }
}

// Moves the mailbox entries of every filter epilogue warp (one mailbox segment per warp of
// this kernel) into per-query candidate buffers. The lanes of a warp holding entries of the
// same query take their slots with one atomic (few queries with many candidates each would
// otherwise serialise on their counters).
// On a retry pass (retry != nullptr) it runs only when some query is being retried.
constexpr int kBucketThreads = 256;

__global__ void __launch_bounds__(kBucketThreads) bucket_kernel(
    const unsigned long long* __restrict__ mb_key, const unsigned int* __restrict__ mb_query,
    const unsigned int* __restrict__ mb_count, int segments, int mb_cap, unsigned int* cand_count,
    unsigned long long* cand, int cap, const unsigned int* retry) {
    if (retry != nullptr && *reinterpret_cast<const volatile unsigned int*>(retry) == 0u) return;
    const int c = blockIdx.x * (kBucketThreads / 32) + static_cast<int>(threadIdx.x >> 5);
    if (c >= segments) return;
    const unsigned int n = mb_count[c];
    const size_t base = static_cast<size_t>(c) * mb_cap;
    const unsigned int lane = threadIdx.x & 31u;
    // Four 32-entry chunks per step: their loads, then their atomics, are in flight together.
    constexpr int kU = 4;
    for (unsigned int i0 = 0; i0 < n; i0 += 32u * kU) {
        unsigned long long key[kU];
        unsigned int q[kU], peers[kU], slot[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const unsigned int i = i0 + 32u * u + lane;
            key[u] = i < n ? mb_key[base + i] : 0ull;  // 0: empty, or a tie rejected by its key
            q[u] = i < n ? mb_query[base + i] : 0xFFFFFFFFu;
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            if (key[u] == 0ull) q[u] = 0xFFFFFFFFu;
            peers[u] = __match_any_sync(0xffffffffu, q[u]);
            slot[u] = 0u;
            if (q[u] != 0xFFFFFFFFu && static_cast<int>(lane) == __ffs(peers[u]) - 1) {
                slot[u] = atomicAdd(cand_count + q[u], static_cast<unsigned int>(__popc(peers[u])));
            }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const unsigned int at = __shfl_sync(0xffffffffu, slot[u], __ffs(peers[u]) - 1) +
                                    static_cast<unsigned int>(__popc(peers[u] & ((1u << lane) - 1u)));
            if (q[u] != 0xFFFFFFFFu && at < static_cast<unsigned int>(cap)) cand[static_cast<size_t>(q[u]) * cap + at] = key[u];
        }
    }
}

// The exact top-k of each query's candidates after filter pass `pass`. flags[i] (i < kPasses)
// requests retry pass i, flags[kPasses + i] records a mailbox overflow in pass i; mneed[i] lists
// the query blocks retry pass i scans. A query is answered when at least k candidates passed
// its bound and none were lost, or on the last pass (then an overflow is recorded in the status
// word). Otherwise it asks for the next pass with the safe bound (a statistical bound let fewer
// than k through) or a raised bound (the k-th largest key it captured, after an overflow).
//
// Selection by radix: passes over 8-bit digits from the top (the query's candidates re-read
// each pass, from L1 after the first) find the prefix of the k-th largest key, stopping once
// the keys sharing the prefix are exactly the ones still needed. Once the keys sharing the
// prefix fit the sort buffer (typically after the score's leading digits: the rest are the
// boundary score's ties, told apart by id digits), they are copied there and the remaining
// passes read only them. Each warp counts digits in its
// own histogram (one leader lane per group of equal digits adds the group's size: no shared
// atomics, which serialise when every candidate shares the top digits). The selected keys, k
// in all (keys are distinct), land at per-warp offsets and are sorted in shared memory. A
// network over all candidates would cost a compare-exchange per key and stage of a sort k to
// 16 times wider.
constexpr int kSelectSort = 1024;  // >= ZCGVS_MAX_K, a power of two
// One query per block: 1,024 threads when the batch leaves SMs idle (latency of the passes),
// 512 (more blocks per SM) otherwise.
template <int kPickThreads>
__global__ void __launch_bounds__(kPickThreads) select_kernel(const unsigned long long* __restrict__ cand,
                                                                unsigned int* cand_count, int cap, int k,
                                                                unsigned long long* thr_key,
                                                                const unsigned long long* thr_safe, int* done,
                                                                unsigned int* flags, unsigned int* mneed, int mtiles,
                                                                unsigned int* status, int pass, int* out_idx,
                                                                float* out_scores) {
    constexpr int kSelectWarps = kPickThreads / 32;
    __shared__ u64 keys[kSelectSort];
    __shared__ unsigned int whist[kSelectWarps][256];
    __shared__ unsigned int hist[256];
    __shared__ int s_wbase[kSelectWarps];
    __shared__ int s_count;
    __shared__ u64 s_thr;
    __shared__ int s_digit, s_above, s_group, s_fill;
    const int q = blockIdx.x;
    if (pass > 0 && (*reinterpret_cast<const volatile unsigned int*>(flags + pass) == 0u || done[q])) return;
    const bool final = pass == kPasses - 1;
    const unsigned int total = cand_count[q];
    const bool overflow = total > static_cast<unsigned int>(cap) || flags[kPasses + pass] != 0u;
    // Only the entries this pass wrote (the buffer may hold older ones past them).
    const int n = static_cast<int>(min(total, static_cast<unsigned int>(min(cap, kCandCap))));
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const unsigned long long* mine = cand + static_cast<size_t>(q) * cap;  // non-zero keys
    // Candidate i of a round: every warp runs the same number of rounds (warp-wide shuffles).
    const int rounds = (n + kPickThreads - 1) / kPickThreads;
    // Prefix (under mask) of the k-th largest key; with n <= k every candidate is kept.
    u64 prefix = 0ull, mask = 0ull;
    if (n > k) {
        int rem = k;
        int src_n = n;         // keys in the pass's source
        bool compact = false;  // the source is keys[]: the keys sharing the prefix
        for (int shift = 56; shift >= 0; shift -= 8) {
#pragma unroll
            for (int j = 0; j < 8; ++j) whist[warp][lane + 32 * j] = 0u;
            __syncwarp();
            const int src_rounds = (src_n + kPickThreads - 1) / kPickThreads;
#pragma unroll 4
            for (int r = 0; r < src_rounds; ++r) {
                const int i = r * kPickThreads + tid;
                const u64 key = i < src_n ? (compact ? keys[i] : __ldg(mine + i)) : 0ull;
                const bool in = key != 0ull && (key & mask) == prefix;
                const unsigned int digit = in ? static_cast<unsigned int>(key >> shift) & 0xFFu : 0x100u + lane;
                const unsigned int peers = __match_any_sync(0xffffffffu, digit);
                if (in && lane == __ffs(peers) - 1) whist[warp][digit] += static_cast<unsigned int>(__popc(peers));
                __syncwarp();
            }
            __syncthreads();
            if (tid < 256) {
                unsigned int c = 0u;
#pragma unroll
                for (int w = 0; w < kSelectWarps; ++w) c += whist[w][tid];
                hist[tid] = c;
            }
            __syncthreads();
            if (tid < 32) {
                // Lane l holds digits 255 - 8 l down to 248 - 8 l; counts above each from a scan.
                unsigned int c[8];
                unsigned int sum = 0u;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    c[j] = hist[255 - 8 * lane - j];
                    sum += c[j];
                }
                unsigned int incl = sum;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const unsigned int t = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += t;
                }
                unsigned int above = incl - sum;  // keys with a larger digit than this lane's first
                int found = -1;
                unsigned int found_above = 0u, found_group = 0u;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (found < 0 && above + c[j] >= static_cast<unsigned int>(rem)) {
                        found = 255 - 8 * lane - j;
                        found_above = above;
                        found_group = c[j];
                    }
                    above += c[j];
                }
                const unsigned int hit = __ballot_sync(0xffffffffu, found >= 0);
                const int src = __ffs(hit) - 1;  // the highest digit reaching rem
                if (lane == src) {
                    s_digit = found;
                    s_above = static_cast<int>(found_above);
                    s_group = static_cast<int>(found_group);
                }
            }
            __syncthreads();
            prefix |= static_cast<u64>(s_digit) << shift;
            mask |= 0xFFull << shift;
            rem -= s_above;
            if (s_group == rem) break;  // every key with this prefix is in
            if (!compact && s_group <= kSelectSort && shift > 0) {
                // keys[] is free until the final gather: copy the keys sharing the prefix.
                if (tid == 0) s_fill = 0;
                __syncthreads();
#pragma unroll 4
                for (int r = 0; r < rounds; ++r) {
                    const int i = r * kPickThreads + tid;
                    const u64 key = i < n ? __ldg(mine + i) : 0ull;
                    const bool take = key != 0ull && (key & mask) == prefix;
                    const unsigned int ballot = __ballot_sync(0xffffffffu, take);
                    int base = 0;
                    if (lane == 0 && ballot != 0u) base = atomicAdd(&s_fill, __popc(ballot));
                    base = __shfl_sync(0xffffffffu, base, 0);
                    if (take) keys[base + __popc(ballot & ((1u << lane) - 1u))] = key;
                }
                __syncthreads();
                src_n = s_group;
                compact = true;
            }
        }
        __syncthreads();  // keys[] is rewritten by the gather below
    }
    // Gather the selected keys (k of them, or all n) at per-warp offsets and sort them.
    int wsel = 0;  // this warp's selected keys (the same in every lane)
#pragma unroll 4
    for (int r = 0; r < rounds; ++r) {
        const int i = r * kPickThreads + tid;
        const u64 key = i < n ? __ldg(mine + i) : 0ull;
        wsel += __popc(__ballot_sync(0xffffffffu, key != 0ull && (key & mask) >= prefix));
    }
    if (lane == 0) s_wbase[warp] = wsel;
    __syncthreads();
    if (tid == 0) {
        int run = 0;
        for (int w = 0; w < kSelectWarps; ++w) {
            const int c = s_wbase[w];
            s_wbase[w] = run;
            run += c;
        }
        s_count = min(run, kSelectSort);  // min(n, k)
        s_thr = 0ull;
    }
    __syncthreads();
    int slot = s_wbase[warp];
#pragma unroll 4
    for (int r = 0; r < rounds; ++r) {
        const int i = r * kPickThreads + tid;
        const u64 key = i < n ? __ldg(mine + i) : 0ull;
        const bool take = key != 0ull && (key & mask) >= prefix;
        const unsigned int ballot = __ballot_sync(0xffffffffu, take);
        const int at = slot + __popc(ballot & ((1u << lane) - 1u));
        if (take && at < kSelectSort) keys[at] = key;
        slot += __popc(ballot);
    }
    __syncthreads();
    TopkSmem t;
    t.buf = keys;
    t.count = &s_count;
    t.thr = &s_thr;
    t.cap = kSelectSort;
    t.k = k;
    topk_flush_mask(t, 1u, kPickThreads);  // sorts the selected keys; keeps min(count, k)
    const bool short_list = !overflow && n < k && thr_key[q] != thr_safe[q];
    if ((overflow || short_list) && !final) {
        if (tid == 0) {
            if (short_list) {
                thr_key[q] = thr_safe[q];
            } else if (n >= k) {
                thr_key[q] = keys[k - 1];  // k captured documents bound the k-th best
            }
            cand_count[q] = 0u;
            mneed[(pass + 1) * mtiles + q / kBM] = 1u;
            atomicOr(flags + pass + 1, 1u);
        }
        return;
    }
    if ((overflow || short_list) && tid == 0) atomicOr(status, kStatusOverflow);
    topk_write(t, 0, out_idx + static_cast<size_t>(q) * k, out_scores + static_cast<size_t>(q) * k, kPickThreads);
    if (tid == 0) done[q] = 1;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult qres{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qres) != cudaSuccess ||
            qres != cudaDriverEntryPointSuccess) {
            ptr = nullptr;
        }
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }();
    return fn;
}

// 2-D tiled tensor map over a row-major [rows, row_bytes] operand: box = 128 bytes of K by
// box_rows rows, 128-byte swizzle; rows past the end read as zero.
int make_map(CUtensorMap* map, const void* base, int mode, long long rows, int row_bytes, int box_rows) {
    const auto fn = encode_fn();
    if (fn == nullptr) return fail(ZCGVS_ERR_CUDA, "zcgvs gemm: cuTensorMapEncodeTiled is unavailable");
    const bool f16 = (mode == kModeF16);
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(f16 ? row_bytes / 2 : row_bytes), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(f16 ? kBKBytes / 2 : kBKBytes), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                          const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        return fail(ZCGVS_ERR_CUDA, "zcgvs gemm: cuTensorMapEncodeTiled failed (" + std::to_string(static_cast<int>(r)) + ")");
    }
    return ZCGVS_OK;
}

// 2-D map over packed 1-bit rows [rows, row_bytes]: box = 128 bytes (1,024 dimensions, 8 K
// slices) of 256 rows, 128-byte swizzle; bytes and rows past the end read as zero.
int make_raw_map(CUtensorMap* map, const void* base, long long rows, int row_bytes) {
    const auto fn = encode_fn();
    if (fn == nullptr) return fail(ZCGVS_ERR_CUDA, "zcgvs gemm: cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
    const cuuint32_t box[2] = {128u, static_cast<cuuint32_t>(kBN)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        return fail(ZCGVS_ERR_CUDA, "zcgvs gemm: cuTensorMapEncodeTiled failed (" + std::to_string(static_cast<int>(r)) + ")");
    }
    return ZCGVS_OK;
}

// The operand maps of a search: queries (prepared in the workspace) and corpus.
int make_maps(CUtensorMap* mq, CUtensorMap* mx, int mode, int dtype, const void* corpus, long long n, int dim,
              const void* prepared, int batch) {
    const int a_bytes = operand_row_bytes(mode, dtype, dim);
    int status = make_map(mq, prepared, mode, batch, a_bytes, kBM);
    if (status != ZCGVS_OK) return status;
    if (mode == kModeBin) return make_raw_map(mx, corpus, n, static_cast<int>(row_bytes_of(dtype, dim)));
    return make_map(mx, corpus, mode, n, a_bytes, kBN);
}

struct GemmLayout {
    int mode = 0;
    int kblocks = 0, mtiles = 0, ntiles = 0, sample_tiles = 0;
    size_t q_bytes = 0;
    size_t off_q = 0, off_qscale = 0, off_cmax = 0, off_thr = 0, off_count = 0, off_done = 0, off_cand = 0;
    size_t off_mb_key = 0, off_mb_query = 0, off_mb_count = 0, total = 0;
    int mb_cap = 0, mb_ctas = 0, expected = 0;
    size_t off_thr_safe = 0, off_mneed = 0;
};

int plan_gemm(int dtype, long long n, int dim, int batch, int k, GemmLayout& g) {
    if (dtype == ZCGVS_DTYPE_F16) {
        g.mode = kModeF16;
    } else if (dtype == ZCGVS_DTYPE_I8_ROW) {
        g.mode = kModeI8R;
    } else if (dtype == ZCGVS_DTYPE_BINARY) {
        g.mode = kModeBin;
    } else {
        return fail(ZCGVS_ERR_UNSUPPORTED,
                    "zcgvs gemm: the tensor-core scan takes float16, per-row int8 or 1-bit corpora");
    }
    // Bytes of one row of the MMA operands (1-bit rows become one int8 per dimension).
    const int row_bytes = operand_row_bytes(g.mode, dtype, dim);
    if (row_bytes % kBKBytes != 0) {
        return fail(ZCGVS_ERR_UNSUPPORTED, "zcgvs gemm: rows must be a multiple of 128 bytes (dim % " +
                                               std::to_string(g.mode == kModeF16 ? 64 : 128) + " == 0)");
    }
    g.kblocks = row_bytes / kBKBytes;
    g.mtiles = (batch + kBM - 1) / kBM;
    g.ntiles = static_cast<int>((n + kBN - 1) / kBN);
    // Expected candidates per query E; the statistical bound (rank 16) needs a sample of 16 / E
    // of the tiles for about E documents of the corpus to pass it.
    g.expected = std::min(4096, std::max(1024, 8 * k));
    const long long want = (static_cast<long long>(g.ntiles) * kStatRank + g.expected - 1) / g.expected;
    g.sample_tiles = static_cast<int>(std::max<long long>(1, std::min<long long>(g.ntiles, want)));
    g.q_bytes = static_cast<size_t>(batch) * row_bytes;
    size_t off = 16 + 8 * kPasses;  // status word, per-pass retry and overflow flags
    auto take = [&](size_t bytes) {
        off = round_up(off, kAlign);
        const size_t at = off;
        off += bytes;
        return at;
    };
    g.off_q = take(g.q_bytes);
    g.off_qscale = take(4ull * batch);
    g.off_cmax = take(4ull * batch * g.sample_tiles * kChunks);
    g.off_thr = take(8ull * batch);
    g.off_thr_safe = take(8ull * batch);
    g.off_mneed = take(4ull * kPasses * g.mtiles);
    g.off_count = take(4ull * batch);
    g.off_done = take(4ull * batch);
    g.off_cand = take(8ull * batch * kCandCap);
    // Mailboxes: 4x the candidates one filter CTA is expected to produce, never more than its
    // items can produce at all. A query keeps about k * tiles / sample tiles documents (every
    // document when the sample has fewer than k chunks).
    g.mb_ctas = device_sm_count();
    const long long items = static_cast<long long>(g.mtiles) * g.ntiles;
    const long long per_cta = (items + g.mb_ctas - 1) / g.mb_ctas;
    const double frac = g.sample_tiles * kChunks < k
                            ? 1.0
                            : std::min(1.0, std::max(static_cast<double>(g.expected),
                                                     static_cast<double>(k) * g.ntiles / g.sample_tiles) /
                                                static_cast<double>(n));
    const long long rows = std::min(batch, kBM);
    const long long bound = per_cta * rows * kBN;
    const long long want_mb = std::max<long long>(4096, static_cast<long long>(4.0 * frac * static_cast<double>(bound)));
    // Per epilogue warp: a quarter of the CTA's share (a warp sees a quarter of the rows and
    // half of the columns, so this leaves a margin of 2), rounded up.
    g.mb_cap = static_cast<int>(round_up(static_cast<size_t>((std::min(bound, want_mb) + 3) / 4), 1024));
    g.off_mb_key = take(8ull * g.mb_ctas * kEpiWarps * g.mb_cap);
    g.off_mb_query = take(4ull * g.mb_ctas * kEpiWarps * g.mb_cap);
    g.off_mb_count = take(4ull * g.mb_ctas * kEpiWarps);
    g.total = round_up(off, kAlign);
    return ZCGVS_OK;
}

// Shared memory past the stage ring: 1-bit raw slices and their barriers, the other barriers,
// and per epilogue warp and accumulator the side data (scales, validity).
size_t fixed_smem(int mode, int stages) {
    const int raw = mode == kModeBin ? kRawSlots : 0;
    return 1024 + static_cast<size_t>(raw) * kRawBytes + 8 * (2 * stages + 5 + raw) + 16 +
           kEpiWarps * 2 * (kHalf * 4 + 16);
}

int stage_count(int mode) {
    const long long budget = device_max_smem() - 2048;
    const long long room = budget - static_cast<long long>(fixed_smem(mode, 8));
    return static_cast<int>(std::max<long long>(2, std::min<long long>(8, room / kStageBytes)));
}

size_t gemm_smem(int mode, int stages) { return static_cast<size_t>(stages) * kStageBytes + fixed_smem(mode, stages); }

// Vector side-data loads need 16-byte aligned row scales and 4-byte aligned mask bytes.
int side_vec_ok(const float* row_scales, const uint8_t* mask) {
    return (reinterpret_cast<uintptr_t>(row_scales) % 16 == 0 && reinterpret_cast<uintptr_t>(mask) % 4 == 0) ? 1 : 0;
}

using GemmFn = void (*)(const CUtensorMap, const CUtensorMap, const GemmParams);

template <int EPI>
GemmFn gemm_fn(int mode) {
    switch (mode) {
        case kModeI8R: return gemm_scan_kernel<kModeI8R, EPI>;
        case kModeBin: return gemm_scan_kernel<kModeBin, EPI>;
        default: return gemm_scan_kernel<kModeF16, EPI>;
    }
}

int launch_gemm(GemmFn fn, int mode, const CUtensorMap& mq, const CUtensorMap& mx, GemmParams p,
                cudaStream_t stream, const char* tag) {
    cudaError_t e = ensure_smem_optin(reinterpret_cast<const void*>(fn));
    if (e != cudaSuccess) return fail_cuda(e, "cudaFuncSetAttribute(gemm_scan_kernel)");
    const long long items = static_cast<long long>(p.mtiles) * p.ntiles;
    const int grid = static_cast<int>(std::min<long long>(items, device_sm_count()));
    const int threads = mode == kModeBin ? threads_of<kModeBin>() : kThreads;
    {
        KernelTimer timer(tag, stream);
        fn<<<grid, threads, gemm_smem(mode, p.stages), stream>>>(mq, mx, p);
    }
    e = cudaGetLastError();
    return e == cudaSuccess ? ok() : fail_cuda(e, "gemm_scan_kernel launch");
}

int prep(const GemmLayout& g, const float* queries, int batch, int dim, uint8_t* ws, cudaStream_t stream) {
    if (g.mode == kModeBin) {
        prep_queries_kernel<kModeBin><<<batch, 256, 0, stream>>>(queries, dim, ws + g.off_q,
                                                                reinterpret_cast<float*>(ws + g.off_qscale));
    } else if (g.mode == kModeI8R) {
        prep_queries_kernel<kModeI8R><<<batch, 256, 0, stream>>>(queries, dim, ws + g.off_q,
                                                                reinterpret_cast<float*>(ws + g.off_qscale));
    } else {
        prep_queries_kernel<kModeF16><<<batch, 256, 0, stream>>>(queries, dim, ws + g.off_q,
                                                                reinterpret_cast<float*>(ws + g.off_qscale));
    }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ok() : fail_cuda(e, "prep_queries_kernel launch");
}

int validate(const void* corpus, int dtype, const float* row_scales, long long n, int dim, const float* queries,
             int batch, int metric, const void* workspace) {
    if (corpus == nullptr || queries == nullptr || workspace == nullptr) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs gemm: null corpus, query or workspace pointer");
    }
    if (n > INT_MAX) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs gemm: corpus exceeds the supported document count");
    if (metric != ZCGVS_METRIC_DOT && metric != ZCGVS_METRIC_COSINE && metric != ZCGVS_METRIC_L2) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs gemm: unknown metric");
    }
    // 1-bit corpora score by Hamming distance whatever the metric (src/cuda/similarity.cu:380-390).
    if (metric == ZCGVS_METRIC_L2 && dtype != ZCGVS_DTYPE_BINARY) {
        return fail(ZCGVS_ERR_UNSUPPORTED, "zcgvs gemm: the tensor-core scan scores dot/cosine");
    }
    if (dtype == ZCGVS_DTYPE_I8_ROW && row_scales == nullptr) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs gemm: the per-row int8 store needs row_scales");
    }
    if ((reinterpret_cast<uintptr_t>(corpus) & 15u) != 0 || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs gemm: corpus must be 16-byte and workspace 256-byte aligned");
    }
    if (batch > INT_MAX / 2) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs gemm: batch too large");
    return ZCGVS_OK;
}

}  // namespace
}  // namespace gemm
}  // namespace zc

extern "C" {

size_t zcgvs_gemm_topk_workspace_bytes(int dtype, int64_t doc_count, int dim, int batch, int k) {
    if (doc_count <= 0 || dim <= 0 || batch <= 0 || k <= 0) return 0;
    zc::gemm::GemmLayout g;
    const size_t bytes = zc::gemm::plan_gemm(dtype, doc_count, dim, batch, std::min(k, ZCGVS_MAX_K), g) == ZCGVS_OK
                             ? g.total
                             : 0;
    zc::ok();
    return bytes;
}

int zcgvs_gemm_topk(const void* corpus, int dtype, const float* row_scales, int64_t doc_count, int dim,
                    const float* queries, int batch, const uint8_t* mask, int metric, int k, int id_base,
                    int* out_indices, float* out_scores, void* workspace, size_t workspace_bytes, void* stream) {
    using namespace zc;
    using namespace zc::gemm;
    if (doc_count <= 0 || batch <= 0 || dim <= 0) return ok();
    int status = validate(corpus, dtype, row_scales, doc_count, dim, queries, batch, metric, workspace);
    if (status != ZCGVS_OK) return status;
    if (k <= 0 || k > ZCGVS_MAX_K) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs gemm: k must be in [1, " + std::to_string(ZCGVS_MAX_K) + "]");
    }
    if (k > doc_count) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs gemm: k exceeds corpus size");
    if (out_indices == nullptr || out_scores == nullptr) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs gemm: null output");
    if (id_base < 0 || static_cast<long long>(id_base) + doc_count - 1 > INT_MAX) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs gemm: id_base + doc_count exceeds the int32 id range");
    }
    GemmLayout g;
    status = plan_gemm(dtype, doc_count, dim, batch, k, g);
    if (status != ZCGVS_OK) return status;
    if (workspace_bytes < g.total) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs gemm: workspace smaller than zcgvs_gemm_topk_workspace_bytes()");
    }
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    CUtensorMap mq, mx;
    status = make_maps(&mq, &mx, g.mode, dtype, corpus, doc_count, dim, ws + g.off_q, batch);
    if (status != ZCGVS_OK) return status;
    status = prep(g, queries, batch, dim, ws, st);
    if (status != ZCGVS_OK) return status;

    GemmParams p{};
    p.n = doc_count;
    p.batch = batch;
    p.kblocks = g.kblocks;
    p.mtiles = g.mtiles;
    p.dim = dim;
    p.id_base = static_cast<unsigned>(id_base);
    p.qscale = reinterpret_cast<const float*>(ws + g.off_qscale);
    p.row_scales = row_scales;
    p.mask = mask;
    p.chunk_max = reinterpret_cast<float*>(ws + g.off_cmax);
    p.thr_key = reinterpret_cast<const unsigned long long*>(ws + g.off_thr);
    unsigned int* cand_count = reinterpret_cast<unsigned int*>(ws + g.off_count);
    unsigned long long* cand = reinterpret_cast<unsigned long long*>(ws + g.off_cand);
    p.mb_key = reinterpret_cast<unsigned long long*>(ws + g.off_mb_key);
    p.mb_query = reinterpret_cast<unsigned int*>(ws + g.off_mb_query);
    p.mb_count = reinterpret_cast<unsigned int*>(ws + g.off_mb_count);
    p.mb_cap = g.mb_cap;
    p.status = reinterpret_cast<unsigned int*>(ws);
    p.stages = stage_count(g.mode);
    p.side_vec = side_vec_ok(row_scales, mask);

    // Threshold pre-pass over the first sample tiles.
    GemmParams ps = p;
    ps.ntiles = g.sample_tiles;
    ps.n = std::min<long long>(doc_count, static_cast<long long>(g.sample_tiles) * kBN);
    status = launch_gemm(gemm_fn<kTileMax>(g.mode), g.mode, mq, mx, ps, st, "gemm_sample");
    if (status != ZCGVS_OK) return status;
    const int chunks = g.sample_tiles * kChunks;
    const int tcap = kSelectCap;
    unsigned long long* thr_key = reinterpret_cast<unsigned long long*>(ws + g.off_thr);
    int* done = reinterpret_cast<int*>(ws + g.off_done);
    unsigned int* retry = reinterpret_cast<unsigned int*>(ws + 16);  // [2 * kPasses] flags
    cudaError_t e = ensure_smem_optin(reinterpret_cast<const void*>(threshold_kernel));
    if (e != cudaSuccess) return fail_cuda(e, "cudaFuncSetAttribute(threshold_kernel)");
    unsigned long long* thr_safe = reinterpret_cast<unsigned long long*>(ws + g.off_thr_safe);
    unsigned int* mneed = reinterpret_cast<unsigned int*>(ws + g.off_mneed);
    {
        KernelTimer timer("gemm_threshold", st);
        if (chunks <= kThrRegs * 32) {
            threshold_regs_kernel<<<(batch + kThrWarps - 1) / kThrWarps, kThrWarps * 32, 0, st>>>(
                p.chunk_max, chunks, k, batch, thr_key, thr_safe, cand_count, done, retry, mneed, g.mtiles);
        } else {
            threshold_kernel<<<batch, kSelectThreads, static_cast<size_t>(tcap) * 8, st>>>(
                p.chunk_max, chunks, k, tcap, thr_key, thr_safe, cand_count, done, retry, mneed, g.mtiles);
        }
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "threshold_kernel launch");
    e = ensure_smem_optin(reinterpret_cast<const void*>(select_kernel<512>));
    if (e == cudaSuccess) e = ensure_smem_optin(reinterpret_cast<const void*>(select_kernel<1024>));
    if (e != cudaSuccess) return fail_cuda(e, "cudaFuncSetAttribute(select_kernel)");

    // Filter pass over the whole corpus and its selection, then the (usually empty) retry.
    p.ntiles = g.ntiles;
    p.done = done;
    const long long items = static_cast<long long>(p.mtiles) * p.ntiles;
    const int filter_ctas = static_cast<int>(std::min<long long>(items, g.mb_ctas));
    const int cap = cand_cap();
    for (int pass = 0; pass < kPasses; ++pass) {
        p.retry = pass == 0 ? nullptr : retry + pass;
        p.mneed = pass == 0 ? nullptr : mneed + static_cast<size_t>(pass) * g.mtiles;
        p.mb_overflow = retry + kPasses + pass;
        status = launch_gemm(gemm_fn<kFilter>(g.mode), g.mode, mq, mx, p, st, pass == 0 ? "gemm_filter" : "gemm_retry");
        if (status != ZCGVS_OK) return status;
        {
            KernelTimer timer("gemm_bucket", st);
            const int segments = filter_ctas * kEpiWarps;
            const int blocks = (segments + kBucketThreads / 32 - 1) / (kBucketThreads / 32);
            bucket_kernel<<<blocks, kBucketThreads, 0, st>>>(p.mb_key, p.mb_query, p.mb_count, segments, g.mb_cap,
                                                             cand_count, cand, cap, p.retry);
        }
        e = cudaGetLastError();
        if (e != cudaSuccess) return fail_cuda(e, "bucket_kernel launch");
        {
            KernelTimer timer("gemm_select", st);
            if (batch < device_sm_count()) {
                select_kernel<1024><<<batch, 1024, 0, st>>>(cand, cand_count, cap, k, thr_key, thr_safe, done,
                                                            retry, mneed, g.mtiles, p.status, pass, out_indices,
                                                            out_scores);
            } else {
                select_kernel<512><<<batch, 512, 0, st>>>(cand, cand_count, cap, k, thr_key, thr_safe, done,
                                                          retry, mneed, g.mtiles, p.status, pass, out_indices,
                                                          out_scores);
            }
        }
        e = cudaGetLastError();
        if (e != cudaSuccess) return fail_cuda(e, "select_kernel launch");
    }
    return ok();
}

int zcgvs_test_set_candidate_cap(int cap) {
    if (cap < 0 || cap > zc::gemm::kCandCap) {
        return zc::fail(ZCGVS_ERR_INVALID_ARG,
                        "zcgvs_test_set_candidate_cap: cap must be 0 (default) or 1.." + std::to_string(zc::gemm::kCandCap));
    }
    zc::gemm::g_test_cand_cap.store(cap, std::memory_order_relaxed);
    return zc::ok();
}

size_t zcgvs_gemm_similarity_workspace_bytes(int dtype, int64_t doc_count, int dim, int batch) {
    if (doc_count <= 0 || dim <= 0 || batch <= 0) return 0;
    zc::gemm::GemmLayout g;
    const size_t bytes = zc::gemm::plan_gemm(dtype, doc_count, dim, batch, 1, g) == ZCGVS_OK
                             ? zc::round_up(g.off_qscale + 4ull * batch, 256)
                             : 0;
    zc::ok();
    return bytes;
}

int zcgvs_gemm_similarity(const void* corpus, int dtype, const float* row_scales, int64_t doc_count, int dim,
                          const float* queries, int batch, const uint8_t* mask, int metric, float* scores,
                          void* workspace, size_t workspace_bytes, void* stream) {
    using namespace zc;
    using namespace zc::gemm;
    if (doc_count <= 0 || batch <= 0 || dim <= 0) return ok();
    int status = validate(corpus, dtype, row_scales, doc_count, dim, queries, batch, metric, workspace);
    if (status != ZCGVS_OK) return status;
    if (scores == nullptr) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs gemm: null score pointer");
    GemmLayout g;
    status = plan_gemm(dtype, doc_count, dim, batch, 1, g);
    if (status != ZCGVS_OK) return status;
    if (workspace_bytes < g.off_qscale + 4ull * batch) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs gemm: workspace smaller than zcgvs_gemm_similarity_workspace_bytes()");
    }
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    CUtensorMap mq, mx;
    status = make_maps(&mq, &mx, g.mode, dtype, corpus, doc_count, dim, ws + g.off_q, batch);
    if (status != ZCGVS_OK) return status;
    status = prep(g, queries, batch, dim, ws, st);
    if (status != ZCGVS_OK) return status;
    GemmParams p{};
    p.n = doc_count;
    p.batch = batch;
    p.kblocks = g.kblocks;
    p.mtiles = g.mtiles;
    p.dim = dim;
    p.ntiles = g.ntiles;
    p.qscale = reinterpret_cast<const float*>(ws + g.off_qscale);
    p.row_scales = row_scales;
    p.mask = mask;
    p.out_matrix = scores;
    p.status = reinterpret_cast<unsigned int*>(ws);
    p.stages = stage_count(g.mode);
    p.side_vec = side_vec_ok(row_scales, mask);
    return launch_gemm(gemm_fn<kEmit>(g.mode), g.mode, mq, mx, p, st, "gemm_emit");
}

}  // extern "C"
