// Tensor-core corpus scan for large query batches (tcgen05 + TMEM + TMA), sm_100a.
//
// For a batch of B queries the scan is a dense contraction S = Q . X^T ([B, d] x [d, N]); the
// reference computes it with one CUDA-core kernel per 8 queries (src/cuda/similarity.cu:83-164)
// and writes the [B, N] score matrix to HBM before its top-k. Here:
//
//   * Work items are (query block m of 128 rows, document tile n of 256 rows); a persistent CTA
//     walks items m-fastest so the CTAs running at the same time share document tiles in L2.
//   * Warp 8 (producer) moves 128-byte K slices of the query block (128 x 128 B) and of the
//     document tile (256 x 128 B) into a ring of shared-memory stages with 2-D TMA loads
//     (128-byte swizzle, the canonical K-major layout of the tensor-core descriptors).
//   * Warp 9 (one elected thread) issues tcgen05.mma (kind::f16: fp16 x fp16 -> fp32, or
//     kind::i8: int8 x int8 -> int32, both operands K-major) into one of two 128 x 256 fp32/int32
//     accumulators in tensor memory, and commits each stage back to the producer and each
//     finished accumulator to the epilogue through mbarriers.
//   * Warps 0-7 (epilogue) read the accumulator with tcgen05.ld (warp w owns TMEM lanes
//     32 (w % 4) .. + 31, i.e. query rows, and column half w / 4) while the next item's MMAs
//     run in the other accumulator,
//     and either write the scores (EMIT), reduce each query's maximum over the tile (TILE_MAX,
//     the threshold pre-pass) or keep only scores at or above a per-query threshold (FILTER),
//     appending them as 64-bit selection keys to a per-query candidate buffer.
//
// 1-bit corpora (kModeBin, the Hamming score (d - 2 h) / d of src/cuda/similarity.cu:166-240)
// run on the same int8 tensor-core path. A 2-D TMA brings 128 packed bytes (1,024 dimensions) of
// 256 rows at a time into one of two raw slots (128-byte swizzle, so that reading one 16-byte
// column of consecutive rows hits distinct banks), and eight more warps (10-17, the expanders)
// turn each 16-byte K slice (128 dimensions) of it into the int8 operand of a stage: bit b of a word becomes the byte 0xFF (-1) when set, else 0 (one shift
// and one sign-replicating byte permute per 4 output bytes). The queries are prepared as
// q' = -2 s (s = +1 for a set bit, else -1), so the accumulator holds 2 sum_i s_i b_i and the
// exact integer dot product of the two sign vectors is acc - sum_i s_i = d - 2 h. Within each
// 32-dimension word the expansion stores dimension 8 i + j at byte 4 j + i; the query rows use
// the same order, which leaves the dot product unchanged. The epilogue compares these integers
// with per-query integer bounds and divides (IEEE, as the reference) only for the values it
// keeps.
//
// Every mbarrier wait is bounded; on a timeout the kernel records a status bit, stops issuing,
// waits (bounded) for its own copies and MMAs in flight, frees its tensor memory and returns.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include <climits>

#include "common.cuh"

namespace zc {

namespace gemm {

constexpr int kBM = 128;                  // query rows per item (TMEM lanes)
constexpr int kBN = 256;                  // document rows per item (TMEM columns)
constexpr int kBKBytes = 128;             // one 128-byte swizzle row of K per stage
constexpr int kStageA = kBM * kBKBytes;   // 16 KB
constexpr int kStageB = kBN * kBKBytes;   // 32 KB
constexpr int kStageBytes = kStageA + kStageB;
constexpr int kEpiWarps = 8;              // two per TMEM lane quarter, one per column half
constexpr int kThreads = 32 * (kEpiWarps + 2);  // warps 0-7 epilogue, 8 producer, 9 MMA
constexpr int kProducerWarp = kEpiWarps;
constexpr int kMmaWarp = kEpiWarps + 1;
constexpr int kHalf = kBN / 2;            // columns per epilogue warp
constexpr int kTmemCols = 512;            // two 256-column accumulators
constexpr int kChunks = kBN / 32;         // threshold granularity: 32-document chunks per tile
// 1-bit corpora: expander warps and the raw slots (128 packed bytes = 8 K slices of 256 rows).
constexpr int kExpWarps = 8;
constexpr int kFirstExpWarp = kEpiWarps + 2;
constexpr int kSlicesPerUnit = 8;
constexpr int kRawBytes = kBN * 128;      // 32 KB per raw slot
constexpr int kRawSlots = 2;
constexpr int kExpBarrier = 1;            // named barrier of the expander warps

template <int MODE>
constexpr int threads_of() {
    return 32 * (kEpiWarps + 2 + (MODE == kModeBin ? kExpWarps : 0));
}

template <int MODE>
constexpr bool int8_operands() {
    return MODE == kModeI8R || MODE == kModeBin;
}

enum Epilogue : int { kEmit = 0, kTileMax = 1, kFilter = 2 };

constexpr uint32_t kStatusTmemWait = 4u;    // an accumulator hand-off wait ran out
constexpr uint32_t kStatusOverflow = 8u;    // a candidate buffer overflowed

struct GemmParams {
    long long n;                 // documents
    int batch;                   // queries
    int kblocks;                 // d * elem_bytes / 128 (1-bit: d / 128)
    int mtiles, ntiles;          // items = mtiles * ntiles
    unsigned id_base;
    int dim;                     // 1-bit: the score divisor d
    const float* qscale;         // I8R: [batch] query scales; 1-bit: [batch] sum of the query's signs
    const float* row_scales;     // I8R: [n]
    const uint8_t* mask;         // optional [n]
    float* out_matrix;           // kEmit: [batch][n]
    float* chunk_max;            // kTileMax: [batch][ntiles * kChunks] maxima of 32-column chunks
    const unsigned long long* thr_key;  // kFilter: [batch] key thresholds (0 = keep everything)
    const int* done;             // kFilter: [batch] queries already answered (skipped), or nullptr
    const unsigned int* retry;   // kFilter: run only when *retry != 0 (nullptr = always)
    const unsigned int* mneed;   // kFilter: [mtiles] query blocks to scan (nullptr = all)
    unsigned long long* mb_key;  // kFilter: mailbox [gridDim.x * 4 epilogue warps][mb_cap] keys (0 = empty)
    unsigned int* mb_query;      // kFilter: the query of each mailbox entry
    unsigned int* mb_count;      // kFilter: [gridDim.x * 4] entries written (capped at mb_cap)
    unsigned int* mb_overflow;   // kFilter: set when any mailbox overflowed
    int mb_cap;                  // entries per epilogue warp
    unsigned int* status;
    int stages;
    int side_vec;                // row_scales 16-byte and mask 4-byte aligned: vector side loads
};

__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t smem_addr) {
    // K-major, 128-byte swizzle: 8-row core groups 1024 bytes apart (SBO = 64 x 16 B), leading
    // offset unused (1), descriptor version 1 (sm_100), base offset 0 (stages are 1024-aligned).
    return static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
           (static_cast<uint64_t>(64) << 32) | (static_cast<uint64_t>(1) << 46) | (static_cast<uint64_t>(2) << 61);
}

// Instruction descriptor: D format (1 = f32, 2 = s32), A/B formats, K-major operands,
// N >> 3 at bit 17, M >> 4 at bit 24.
template <int MODE>
__device__ __forceinline__ constexpr uint32_t instr_desc() {
    return int8_operands<MODE>() ? ((2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kBN >> 3) << 17) |
                               (static_cast<uint32_t>(kBM >> 4) << 24))
                            : ((1u << 4) | (static_cast<uint32_t>(kBN >> 3) << 17) |
                               (static_cast<uint32_t>(kBM >> 4) << 24));
}

template <int MODE>
__device__ __forceinline__ void mma_issue(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate) {
    constexpr uint32_t idesc = instr_desc<MODE>();
    if constexpr (int8_operands<MODE>()) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
    }
}

__device__ __forceinline__ void mma_commit(u64* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, u64* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Byte i of the result = 0xFF when bit 8 i + 7 of x is set, else 0 (prmt with the
// sign-replicate flag on each selector nibble).
__device__ __forceinline__ uint32_t sign_bytes(uint32_t x) {
    uint32_t r;
    asm("prmt.b32 %0, %1, 0, 0xBA98;" : "=r"(r) : "r"(x));
    return r;
}

// w * m as an integer multiply (the FMA pipe), for a multiplier the compiler cannot see.
__device__ __forceinline__ uint32_t mul_lo(uint32_t w, uint32_t m) {
    uint32_t r;
    asm("mul.lo.u32 %0, %1, %2;" : "=r"(r) : "r"(w), "r"(m));
    return r;
}

// One packed word -> 32 int8 operand bytes: o[j] byte i = -(bit 8 i + j of w). pow2[k] = 2^k
// held in registers: the seven shifts run as multiplies on the FMA pipe, leaving the integer
// ALU to the byte permutes (and to the epilogue).
__device__ __forceinline__ void expand_word(uint32_t w, const uint32_t (&pow2)[8], uint4& lo, uint4& hi) {
    lo = make_uint4(sign_bytes(mul_lo(w, pow2[7])), sign_bytes(mul_lo(w, pow2[6])), sign_bytes(mul_lo(w, pow2[5])),
                    sign_bytes(mul_lo(w, pow2[4])));
    hi = make_uint4(sign_bytes(mul_lo(w, pow2[3])), sign_bytes(mul_lo(w, pow2[2])), sign_bytes(mul_lo(w, pow2[1])),
                    sign_bytes(w));
}

// Named barrier over `count` threads that also ANDs a predicate across them.
__device__ __forceinline__ bool bar_and(int id, int count, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.b32 p, %1, 0;\n\t"
        "bar.red.and.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(pred ? 1 : 0), "r"(id), "r"(count)
        : "memory");
    return r != 0u;
}

// 1-bit score of an integer dot product of sign vectors, as the reference rounds it.
__device__ __forceinline__ float bin_score(int d, float dimf) { return __fdiv_rn(__int2float_rn(d), dimf); }

// Integer bounds of a float threshold for 1-bit scores (strictly increasing in d):
// bin_score(d) > thr exactly when d >= d_gt, and bin_score(d) == thr exactly when d == d_eq
// (INT_MAX when no d scores thr).
__device__ __forceinline__ void bin_bounds(float thr, int dim, int& d_gt, int& d_eq) {
    const float dimf = static_cast<float>(dim);
    const float lim = dimf + 2.0f;
    const int d0 = __float2int_rn(fminf(fmaxf(__fmul_rn(thr, dimf), -lim), lim));
    // thr * d is within 1 of the boundary, so [d0 - 2, d0 + 2] brackets it.
    d_gt = d0 + 3;
    d_eq = INT_MAX;
#pragma unroll
    for (int d = d0 + 2; d >= d0 - 2; --d) {
        const float s = bin_score(d, dimf);
        if (s > thr) d_gt = d;
        if (s == thr) d_eq = d;
    }
}

// v[j] for a warp-uniform runtime j without indexing the register array (which would move
// it to local memory): a uniform branch over the 32 cases.
__device__ __forceinline__ float pick32(const float (&v)[32], int j) {
    switch (j) {
#define ZC_PICK(i) \
    case i:        \
        return v[i];
        ZC_PICK(0) ZC_PICK(1) ZC_PICK(2) ZC_PICK(3) ZC_PICK(4) ZC_PICK(5) ZC_PICK(6) ZC_PICK(7)
        ZC_PICK(8) ZC_PICK(9) ZC_PICK(10) ZC_PICK(11) ZC_PICK(12) ZC_PICK(13) ZC_PICK(14) ZC_PICK(15)
        ZC_PICK(16) ZC_PICK(17) ZC_PICK(18) ZC_PICK(19) ZC_PICK(20) ZC_PICK(21) ZC_PICK(22) ZC_PICK(23)
        ZC_PICK(24) ZC_PICK(25) ZC_PICK(26) ZC_PICK(27) ZC_PICK(28) ZC_PICK(29) ZC_PICK(30) ZC_PICK(31)
#undef ZC_PICK
        default:
            return v[31];
    }
}

// Item w of this CTA's walk is skipped when its query block needs no scan (retry passes).
__device__ __forceinline__ bool item_skipped(const GemmParams& p, long long w) {
    return p.mneed != nullptr && p.mneed[w % p.mtiles] == 0u;
}

// The CTA's walk over the items: blockIdx.x, then every gridDim.x-th item, skipping items.
__device__ __forceinline__ long long walk_next(const GemmParams& p, long long w, long long items) {
    do {
        w += gridDim.x;
    } while (w < items && item_skipped(p, w));
    return w;
}

__device__ __forceinline__ long long walk_first(const GemmParams& p, long long items) {
    const long long w = blockIdx.x;
    return (w < items && item_skipped(p, w)) ? walk_next(p, w, items) : w;
}

template <int MODE, int EPI>
__global__ void __launch_bounds__(threads_of<MODE>(), 1)
    gemm_scan_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_x,
                     const GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // Stage ring first, 1024-aligned (the swizzle pattern and base offset 0 assume it).
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int S = p.stages;
    constexpr int R = MODE == kModeBin ? kRawSlots : 0;
    uint8_t* raw = smem + static_cast<size_t>(S) * kStageBytes;  // 1-bit: [R][kBN][128] packed, swizzled
    u64* full = reinterpret_cast<u64*>(raw + static_cast<size_t>(R) * kRawBytes);
    u64* empty = full + S;
    u64* acc_full = empty + S;        // [2]
    u64* acc_empty = acc_full + 2;    // [2]
    u64* drain = acc_empty + 2;       // [1]
    u64* raw_full = drain + 1;        // [R]
    // Per epilogue warp and accumulator: the tile's row scales and validity bytes.
    // 16-byte aligned: the epilogue stores float4s here.
    float* side = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(raw_full + R) + 15) & ~uintptr_t(15));  // [8][2][kHalf]
    uint32_t* side_bits = reinterpret_cast<uint32_t*>(side + kEpiWarps * 2 * kHalf);  // [8][2][4] validity
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    // A retry pass with nothing to retry returns before allocating anything.
    if (EPI == kFilter && p.retry != nullptr && *reinterpret_cast<const volatile unsigned int*>(p.retry) == 0u) return;
    const long long items = static_cast<long long>(p.mtiles) * p.ntiles;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            // 1-bit: the query copy and one arrival per expander warp fill a stage.
            mbar_init(&full[s], MODE == kModeBin ? 1 + kExpWarps : 1);
            mbar_init(&empty[s], 1);
        }
        for (int r = 0; r < R; ++r) mbar_init(&raw_full[r], 1);
        for (int a = 0; a < 2; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], kEpiWarps);
        }
        mbar_init(drain, 1);
        fence_mbarrier_init();
        s_abort = 0;
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = s_tmem;
    volatile int* abort_flag = &s_abort;

    if (warp == kProducerWarp) {
        if (lane == 0) {
            int s = 0;
            uint32_t phase = 0;
            long long issued = 0;
            bool ok = true;
            for (long long w = blockIdx.x; w < items && ok; w += gridDim.x) {
                if (item_skipped(p, w)) continue;
                const int m = static_cast<int>(w % p.mtiles);
                const int n = static_cast<int>(w / p.mtiles);
                for (int kb = 0; kb < p.kblocks; ++kb) {
                    if (issued >= S) {
                        ok = !*abort_flag && mbar_wait_sleep_bounded(&empty[s], phase ^ 1u, p.status, kStatusTileWaitTimeout);
                        if (!ok) {
                            *abort_flag = 1;
                            break;
                        }
                    }
                    uint8_t* st = smem + static_cast<size_t>(s) * kStageBytes;
                    constexpr int kElems = int8_operands<MODE>() ? kBKBytes : kBKBytes / 2;
                    if constexpr (MODE == kModeBin) {
                        // The expander warps write the document half of the stage.
                        mbar_arrive_expect_tx(&full[s], kStageA);
                        tma_load_2d(st, &map_q, kb * kElems, m * kBM, &full[s]);
                    } else {
                        mbar_arrive_expect_tx(&full[s], kStageBytes);
                        tma_load_2d(st, &map_q, kb * kElems, m * kBM, &full[s]);
                        tma_load_2d(st + kStageA, &map_x, kb * kElems, n * kBN, &full[s]);
                    }
                    ++issued;
                    if (++s == S) {
                        s = 0;
                        phase ^= 1u;
                    }
                }
            }
            // Wait (bounded) for the copies still in flight before the CTA can retire.
            if (*abort_flag) {
                for (long long i = issued > S ? issued - S : 0; i < issued; ++i) {
                    mbar_wait_bounded(&full[i % S], static_cast<uint32_t>((i / S) & 1), p.status, kStatusDrainTimeout);
                }
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            int s = 0;
            uint32_t phase = 0;
            long long local = 0;
            bool ok = true;
            for (long long w = blockIdx.x; w < items && ok; w += gridDim.x) {
                if (item_skipped(p, w)) continue;
                const int a = static_cast<int>(local & 1);
                if (local >= 2) {
                    ok = !*abort_flag &&
                         mbar_wait_sleep_bounded(&acc_empty[a], static_cast<uint32_t>(((local >> 1) - 1) & 1), p.status,
                                           kStatusTmemWait);
                    if (!ok) {
                        *abort_flag = 1;
                        break;
                    }
                }
                tc_fence_after();
                const uint32_t tmem_d = tmem_base + static_cast<uint32_t>(a * kBN);
                for (int kb = 0; kb < p.kblocks; ++kb) {
                    ok = !*abort_flag && mbar_wait_sleep_bounded(&full[s], phase, p.status, kStatusTileWaitTimeout);
                    if (!ok) {
                        *abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + static_cast<size_t>(s) * kStageBytes);
                    const uint32_t b_addr = a_addr + kStageA;
                    const uint64_t a_desc = smem_desc_sw128(a_addr);
                    const uint64_t b_desc = smem_desc_sw128(b_addr);
#pragma unroll
                    for (int kk = 0; kk < kBKBytes / 32; ++kk) {
                        // Each MMA consumes 32 bytes of K (16 fp16 or 32 int8): advance both start
                        // addresses by 32 bytes (2 units of 16 B) inside the swizzled row.
                        mma_issue<MODE>(tmem_d, a_desc + static_cast<uint64_t>(2 * kk),
                                        b_desc + static_cast<uint64_t>(2 * kk), (kb > 0 || kk > 0) ? 1u : 0u);
                    }
                    mma_commit(&empty[s]);  // frees the stage when these MMAs have read it
                    if (++s == S) {
                        s = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit(&acc_full[a]);  // accumulator a is complete
                ++local;
            }
            // Make sure no MMA is in flight before the tensor memory is released.
            mma_commit(drain);
            mbar_wait_bounded(drain, 0u, p.status, kStatusDrainTimeout);
        }
    } else if (warp >= kFirstExpWarp) {
        if constexpr (MODE == kModeBin) {
            // ---------------- expander warps 10-17 (1-bit corpora) ----------------
            // Thread et expands row et of each K slice. Thread 0 fetches the raw
            // units (128 packed bytes of the tile's rows) into the two slots, the next one as soon
            // as every expander is done with a slot. A wait that runs out makes the warp skip the
            // rest of the unit; the four warps agree at the unit's end whether to go on, so the
            // named barrier always sees all of them.
            constexpr int kExpThreads = kExpWarps * 32;
            const int et = tid - kFirstExpWarp * 32;
            uint32_t pow2[8];
            const uint32_t one = p.kblocks > 0 ? 1u : 0u;  // 1, as a runtime value
#pragma unroll
            for (int k = 0; k < 8; ++k) pow2[k] = one << k;
            const int units_per_item = (p.kblocks + kSlicesPerUnit - 1) / kSlicesPerUnit;
            long long pw = walk_first(p, items);  // next unit to fetch: item pw, unit pu
            int pu = 0;
            long long fetched = 0;
            auto fetch = [&]() {
                if (pw >= items) return;
                const int slot = static_cast<int>(fetched % R);
                mbar_arrive_expect_tx(&raw_full[slot], kRawBytes);
                tma_load_2d(raw + static_cast<size_t>(slot) * kRawBytes, &map_x, pu * 128,
                            static_cast<int>(pw / p.mtiles) * kBN, &raw_full[slot]);
                ++fetched;
                if (++pu == units_per_item) {
                    pu = 0;
                    pw = walk_next(p, pw, items);
                }
            };
            if (et == 0) {
                for (int i = 0; i < R; ++i) fetch();
            }
            long long u = 0;  // raw units expanded
            long long c = 0;  // slices expanded (= stages filled)
            int s = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (long long w = walk_first(p, items); w < items && ok; w = walk_next(p, w, items)) {
                for (int kb0 = 0; kb0 < p.kblocks; kb0 += kSlicesPerUnit) {
                    const int slot = static_cast<int>(u % R);
                    const uint8_t* src = raw + static_cast<size_t>(slot) * kRawBytes;
                    bool good = !*abort_flag && mbar_wait_bounded(&raw_full[slot], static_cast<uint32_t>((u / R) & 1),
                                                                  p.status, kStatusTileWaitTimeout);
                    good = __all_sync(0xffffffffu, good);
                    const int kb_end = min(kb0 + kSlicesPerUnit, p.kblocks);
                    for (int kb = kb0; kb < kb_end; ++kb) {
                        if (good && c >= S) {
                            good = !*abort_flag &&
                                   mbar_wait_bounded(&empty[s], phase ^ 1u, p.status, kStatusTileWaitTimeout);
                            good = __all_sync(0xffffffffu, good);
                        }
                        if (good) {
                            const int col = kb - kb0;  // 16-byte column of the raw rows
                            uint8_t* dst = smem + static_cast<size_t>(s) * kStageBytes + kStageA;
#pragma unroll
                            for (int h = 0; h < kBN / kExpThreads; ++h) {
                                const int r = et + h * kExpThreads;
                                // Both the raw slot and the stage are 128-byte swizzled K-major
                                // tiles: 16-byte unit x of row r sits at x ^ (r % 8).
                                const uint4 bits =
                                    *reinterpret_cast<const uint4*>(src + r * 128 + ((col ^ (r & 7)) << 4));
                                uint8_t* out = dst + (r >> 3) * 1024 + (r & 7) * 128;
                                const uint32_t words[4] = {bits.x, bits.y, bits.z, bits.w};
#pragma unroll
                                for (int wi = 0; wi < 4; ++wi) {
                                    uint4 lo, hi;
                                    expand_word(words[wi], pow2, lo, hi);
                                    *reinterpret_cast<uint4*>(out + (((2 * wi) ^ (r & 7)) << 4)) = lo;
                                    *reinterpret_cast<uint4*>(out + (((2 * wi + 1) ^ (r & 7)) << 4)) = hi;
                                }
                            }
                            fence_proxy_async_shared();  // the tensor core reads these bytes
                            __syncwarp();
                            if (lane == 0) mbar_arrive_cta(&full[s]);
                        }
                        ++c;
                        if (++s == S) {
                            s = 0;
                            phase ^= 1u;
                        }
                    }
                    // Every expander is done with the slot, and all agree whether to go on.
                    ok = bar_and(kExpBarrier, kExpThreads, good);
                    if (!ok) break;
                    if (et == 0) fetch();
                    ++u;
                }
            }
            if (!ok && et == 0) {
                *abort_flag = 1;
                // Wait (bounded) for the units still in flight before the CTA can retire.
                for (long long i = u; i < fetched; ++i) {
                    mbar_wait_bounded(&raw_full[i % R], static_cast<uint32_t>((i / R) & 1), p.status,
                                      kStatusDrainTimeout);
                }
            }
        }
    } else {
        // ---------------- epilogue warps 0-7 ----------------
        // Warp w reads TMEM lanes 32 (w % 4) .. + 31 (query rows) and columns
        // (w / 4) * 128 .. + 127 of each accumulator (documents): four 32-column chunks.
        const int row = (warp & 3) * 32 + lane;
        const int half = warp >> 2;
        long long local = 0;
        uint32_t wcount = 0u;  // this warp's mailbox entries (kFilter), the same in every lane
        const size_t seg = (static_cast<size_t>(blockIdx.x) * kEpiWarps + warp) * static_cast<size_t>(p.mb_cap);
        // Side data of an item for this warp's half tile, one load per lane (documents 4 lane ..
        // 4 lane + 3): the row scales (per-row int8) and the allow-mask bytes. Loaded one item
        // ahead so the latency overlaps the previous item's epilogue.
        auto next_item = [&](long long w) {
            do {
                w += gridDim.x;
            } while (w < items && item_skipped(p, w));
            return w;
        };
        auto load_side = [&](long long w, float4& sv, uint32_t& mv) {
            sv = make_float4(0.f, 0.f, 0.f, 0.f);
            mv = 0u;
            if (w >= items) return;
            const long long d = (w / p.mtiles) * kBN + half * kHalf + 4 * lane;
            if (p.side_vec && d + 3 < p.n) {
                if constexpr (MODE == kModeI8R) sv = __ldg(reinterpret_cast<const float4*>(p.row_scales + d));
                mv = p.mask != nullptr ? __ldg(reinterpret_cast<const uint32_t*>(p.mask + d)) : 0x01010101u;
            } else {
                float t[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    if (d + i < p.n) {
                        if constexpr (MODE == kModeI8R) t[i] = __ldg(p.row_scales + d + i);
                        const uint32_t allowed = p.mask != nullptr ? (__ldg(p.mask + d + i) != 0 ? 1u : 0u) : 1u;
                        mv |= allowed << (8 * i);
                    }
                }
                sv = make_float4(t[0], t[1], t[2], t[3]);
            }
        };
        long long w = blockIdx.x;
        if (w < items && item_skipped(p, w)) w = next_item(w);
        float4 sv;
        uint32_t mv;
        load_side(w, sv, mv);
        while (w < items) {
            const int m = static_cast<int>(w % p.mtiles);
            const int n = static_cast<int>(w / p.mtiles);
            const int a = static_cast<int>(local & 1);
            const int q = m * kBM + row;
            const bool q_ok = q < p.batch;
            const long long doc0 = static_cast<long long>(n) * kBN + half * kHalf;  // this warp's first column
            // This warp's copy of the side data (the epilogue warps never wait on one another):
            // a validity word per 32-document chunk (padding rows and masked documents are
            // invalid) and, for per-row int8, row scales with NaN for invalid documents (a NaN
            // score fails every comparison).
            float* scales = side + (warp * 2 + a) * kHalf;
            uint32_t* vbits = side_bits + (warp * 2 + a) * 4;
            {
                const uint32_t nib = (mv & 1u) | ((mv >> 7) & 2u) | ((mv >> 14) & 4u) | ((mv >> 21) & 8u);
                if constexpr (MODE == kModeI8R) {
                    const float nan = __int_as_float(0x7fc00000);
                    *reinterpret_cast<float4*>(scales + 4 * lane) =
                        make_float4((nib & 1u) ? sv.x : nan, (nib & 2u) ? sv.y : nan, (nib & 4u) ? sv.z : nan,
                                    (nib & 8u) ? sv.w : nan);
                }
#pragma unroll
                for (int cl = 0; cl < 4; ++cl) {
                    const uint32_t word = __reduce_or_sync(0xffffffffu, (lane >> 3) == cl ? nib << (4 * (lane & 7)) : 0u);
                    if (lane == 0) vbits[cl] = word;
                }
                __syncwarp();
            }
            const long long w_next = next_item(w);
            load_side(w_next, sv, mv);

            bool ok = true;
            if (lane == 0) {
                ok = !*abort_flag && mbar_wait_sleep_bounded(&acc_full[a], static_cast<uint32_t>((local >> 1) & 1), p.status,
                                                       kStatusTmemWait);
                if (!ok) *abort_flag = 1;
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            tc_fence_after();
            float qs = 1.0f, thr = INFINITY;
            unsigned long long thr_key = ~0ull;
            bool live = q_ok;
            // 1-bit: the query's sign sum, and the integer form of its threshold.
            int sq = 0, d_gt = INT_MAX, d_eq = INT_MAX;
            if (q_ok) {
                if constexpr (MODE == kModeI8R) qs = __ldg(p.qscale + q);
                if constexpr (MODE == kModeBin) sq = __float2int_rn(__ldg(p.qscale + q));
                if constexpr (EPI == kFilter) {
                    live = p.done == nullptr || p.done[q] == 0;
                    thr_key = p.thr_key[q];
                    thr = thr_key == 0ull ? -INFINITY : score_from_bits(static_cast<uint32_t>(thr_key >> 32));
                    if constexpr (MODE == kModeBin) {
                        if (thr_key == 0ull) {
                            d_gt = INT_MIN;
                        } else {
                            bin_bounds(thr, p.dim, d_gt, d_eq);
                        }
                    }
                }
            }
            const float dimf = static_cast<float>(p.dim);
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16) +
                                   static_cast<uint32_t>(a * kBN + half * kHalf);
            // A warp whose 32 rows are all padding (or answered) queries only hands the
            // accumulator back.
            const int chunks = __any_sync(0xffffffffu, EPI == kFilter ? live : q_ok) ? 4 : 0;
#pragma unroll 1
            for (int cl = 0; cl < chunks; ++cl) {
                uint32_t v[32];
                __syncwarp();  // tcgen05.ld is warp-collective; the append branch below diverges
                tmem_ld32(taddr + static_cast<uint32_t>(cl * 32), v);
                const uint32_t valid = vbits[cl];
                const long long dchunk = doc0 + cl * 32;
                float sc[32];
                int dv[32];  // 1-bit: integer dot products of the sign vectors
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    if constexpr (MODE == kModeI8R) {
                        sc[j] = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(v[j])), qs), scales[cl * 32 + j]);
                    } else if constexpr (MODE == kModeBin) {
                        dv[j] = static_cast<int>(v[j]) - sq;
                    } else {
                        sc[j] = __uint_as_float(v[j]);
                    }
                }
                if constexpr (EPI == kEmit) {
                    if (q_ok) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const long long d = dchunk + j;
                            if (d < p.n) {
                                const float val = MODE == kModeBin ? bin_score(dv[j], dimf) : sc[j];
                                p.out_matrix[static_cast<size_t>(q) * p.n + d] = ((valid >> j) & 1u) ? val : -FLT_MAX;
                            }
                        }
                    }
                } else if constexpr (EPI == kTileMax) {
                    float best = -INFINITY;
                    if constexpr (MODE == kModeBin) {
                        int dbest = INT_MIN;
                        if (valid == 0xffffffffu) {
#pragma unroll
                            for (int j = 0; j < 32; ++j) dbest = max(dbest, dv[j]);
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; ++j) dbest = max(dbest, ((valid >> j) & 1u) ? dv[j] : INT_MIN);
                        }
                        if (dbest != INT_MIN) best = bin_score(dbest, dimf);
                    } else {
                        // fmaxf ignores the NaN scores of invalid per-row int8 documents.
                        if (valid == 0xffffffffu) {
#pragma unroll
                            for (int j = 0; j < 32; ++j) best = fmaxf(best, sc[j]);
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; ++j) best = fmaxf(best, ((valid >> j) & 1u) ? sc[j] : -INFINITY);
                        }
                    }
                    if (q_ok) p.chunk_max[(static_cast<size_t>(q) * p.ntiles + n) * kChunks + half * 4 + cl] = best;
                } else {
                    // Candidates go to this warp's own mailbox segment at a register counter:
                    // the epilogue issues no atomics and never waits on a store. Most chunks
                    // hold none: a max over the lane's 32 scores (one operation each) decides
                    // whether the per-score masks are built at all.
                    bool maybe;
                    if constexpr (MODE == kModeBin) {
                        int dmax = dv[0];
#pragma unroll
                        for (int j = 1; j < 32; ++j) dmax = max(dmax, dv[j]);
                        maybe = live && (dmax >= d_gt || dmax >= d_eq);
                    } else {
                        float fmax = sc[0];
#pragma unroll
                        for (int j = 1; j < 32; ++j) fmax = fmaxf(fmax, sc[j]);  // NaN (invalid) ignored
                        maybe = live && fmax >= thr;
                    }
                    if (__ballot_sync(0xffffffffu, maybe) == 0u) continue;
                    uint32_t pass = 0u, ties = 0u;
                    if (maybe) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            if constexpr (MODE == kModeBin) {
                                pass |= (dv[j] >= d_gt ? 1u : 0u) << j;
                                ties |= (dv[j] == d_eq ? 1u : 0u) << j;
                            } else {
                                pass |= (sc[j] > thr ? 1u : 0u) << j;
                                ties |= (sc[j] == thr ? 1u : 0u) << j;
                            }
                        }
                        pass &= valid;
                        ties &= valid;
                    }
                    // A score equal to the threshold's passes only if its key (ties by id) does.
                    while (ties != 0u) {
                        const int j = __ffs(ties) - 1;
                        ties &= ties - 1u;
                        if (make_key(thr, p.id_base + static_cast<unsigned>(dchunk + j)) >= thr_key) pass |= 1u << j;
                    }
                    const uint32_t cnt = static_cast<uint32_t>(__popc(pass));
                    const uint32_t some = __ballot_sync(0xffffffffu, cnt != 0u);
                    if (some == 0u) continue;
                    // Slots: one ballot when no lane has more than one candidate (the common
                    // case), else an inclusive warp scan of the counts.
                    uint32_t excl, total;
                    if (__ballot_sync(0xffffffffu, cnt > 1u) == 0u) {
                        excl = static_cast<uint32_t>(__popc(some & ((1u << lane) - 1u)));
                        total = static_cast<uint32_t>(__popc(some));
                    } else {
                        uint32_t incl = cnt;
#pragma unroll
                        for (int o = 1; o < 32; o <<= 1) {
                            const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
                            if (lane >= o) incl += t;
                        }
                        excl = incl - cnt;
                        total = __shfl_sync(0xffffffffu, incl, 31);
                    }
                    uint32_t slot = wcount + excl;
                    wcount += total;
                    uint32_t bits = pass;
                    while (bits != 0u) {
                        const int j = __ffs(bits) - 1;
                        bits &= bits - 1u;
                        float val;
                        if constexpr (MODE == kModeBin) {
                            int dsel = dv[0];
#pragma unroll
                            for (int jj = 1; jj < 32; ++jj) dsel = (j == jj) ? dv[jj] : dsel;
                            val = bin_score(dsel, dimf);
                        } else {
                            val = sc[0];
#pragma unroll
                            for (int jj = 1; jj < 32; ++jj) val = (j == jj) ? sc[jj] : val;
                        }
                        const unsigned long long key = make_key(val, p.id_base + static_cast<unsigned>(dchunk + j));
                        if (slot < static_cast<uint32_t>(p.mb_cap)) {
                            p.mb_key[seg + slot] = key;
                            p.mb_query[seg + slot] = static_cast<unsigned int>(q);
                        }
                        ++slot;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cta(&acc_empty[a]);
            ++local;
            w = w_next;
        }
        if constexpr (EPI == kFilter) {
            if (lane == 0) {
                p.mb_count[blockIdx.x * kEpiWarps + warp] = min(wcount, static_cast<uint32_t>(p.mb_cap));
                if (wcount > static_cast<uint32_t>(p.mb_cap)) atomicOr(p.mb_overflow, 1u);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    if (warp == kMmaWarp) {
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                     : "memory");
    }
}

}  // namespace gemm
}  // namespace zc
