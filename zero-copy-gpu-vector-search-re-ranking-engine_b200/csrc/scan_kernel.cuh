// Streaming corpus scan with fused top-k for single- and small-batch queries.
//
// Replaces the reference pipeline `similarityScanKernel`/`hammingScanKernel`
// (src/cuda/similarity.cu:83-238) -> [batch, N] fp32 score matrix in HBM -> `launchTopK`
// (src/cuda/topk.cu:132-189) with one kernel per call:
//
//   * Work split: the corpus is cut into tiles of R whole rows; CTA y of the grid owns a
//     contiguous range of tiles, CTA x a pass of QB queries (x varies fastest, so the passes
//     that read the same rows run side by side and share L2).
//   * Staging: when rows are 16-byte multiples, one thread moves each tile global -> shared
//     with a single bulk async copy (cp.async.bulk, the TMA engine's 1-D form) into an
//     S-deep ring of stages tracked by mbarriers; otherwise all threads copy rows into a
//     zero-padded 16-byte stride (the reference's scalar fallback, :273-287).
//   * Scoring: warp per row for fp32 / fp16 / int8 rows, lanes striding 16-byte chunks;
//     partial sums of the QB queries are combined with one transposing warp reduction.
//     Binary rows are thread per row (XOR + popc), like the reference's Hamming kernel.
//   * Selection: scores go straight into the CTA's on-chip top-k (topk_cta.cuh); at the end
//     each CTA writes k keys per query to the workspace and the last CTA to finish a pass
//     merges them and writes the final [QB, k] ids and scores.
//
// Numerics follow the reference: fp16 and int8 rows are widened to fp32 and multiplied by the
// fp32 query (decode.cuh:22-43); L2 is -sum((q - x)^2); Hamming scores are
// (dim - 2 h) / dim. The per-row int8 mode scores float(int32 dot) * s_q * s_row exactly.
#pragma once

#include <type_traits>

#include "common.cuh"
#include "lexical_device.cuh"
#include "topk_cta.cuh"

namespace zc {

constexpr int kScanThreads = 512;
constexpr int kScanWarps = kScanThreads / 32;

struct ScanParams {
    const uint8_t* corpus;
    const float* row_scales;       // kModeI8R: [n]
    float scale;                   // kModeI8M
    long long n;                   // rows
    int dim;
    int row_bytes;                 // bytes of one row in global memory
    int stride;                    // bytes of one row in shared memory (multiple of 16)
    int nch;                       // stride / 16
    int elems_per_row;             // storage elements per global row (dim, or words)
    const void* queries;           // fp32 [batch, dim], or packed words when query_packed
    int query_packed;
    int batch;
    const uint8_t* mask;
    int k;
    int cap;                       // top-k buffer capacity (power of two)
    int rows_per_tile;
    long long ntiles;
    int use_tma;
    int stages;
    unsigned int id_base;
    unsigned long long* lists;     // [batch][gridDim.y][k]
    unsigned int* counters;        // [gridDim.x]
    unsigned int* status;
    int* out_idx;                  // [batch][k]
    float* out_scores;             // [batch][k]
    float* out_matrix;             // score-matrix mode: [batch][n]
    int query_bytes;               // bytes of one staged query
    int stage_bytes;               // one pipeline stage: rows, then per-row side data
    int side_scales;               // stage the per-row scales (kModeI8R)
    int side_tma;                  // side data may ride the tile's bulk copies (aligned)
    int side_off_scales;           // offsets of the side data inside a stage
    int side_off_mask;
    int merge_cap;                 // warp-specialised kernel: selector buffer capacity
    int cap_final;                 // warp-specialised kernel: merge buffer capacity
    unsigned long long* spill;     // warp-specialised kernel: [passes][G][spill_stride]
    long long spill_stride;
    int smem_query_off;
    int smem_topk_off;
    int smem_bar_off;
    // Hybrid lexical + dense scoring (nullptr lex = dense only): lex[batch][n] lexical scores,
    // lex_part[batch][lex_parts] non-negative partial maxima from the lexical kernel.
    const float* lex;
    const float* lex_part;
    int lex_parts;
    float dense_weight;
    // Hybrid scan with lexical warps (scan_fast_kernel<MODE, JC, true>, one query): the CSR
    // index, the query terms [lex_stride], the lexical scores out [n] and their maximum, raised
    // with an unsigned atomicMax on the bits of each CTA's max(0, max) (valid for non-negative
    // floats); the dense scores go to out_matrix [n]. The BM25 accumulator (lex_window
    // documents) sits at smem_lex_off of the dynamic shared memory; a CTA scores its documents
    // lex_window at a time.
    LexIndex lexi;
    const int* lex_terms;
    int lex_stride;
    float* lex_out;
    unsigned int* lex_peak;
    int smem_lex_off;
    int lex_window;
};

// Convex blend of a dense score with a max-normalised lexical score in the reference's
// operation order, w * dense + ((1 - w) * lex) * inv (src/cuda/lexical.cu:66-72), every step
// rounded on its own as in the CPU loop of tests/cpp/test_lexical.cu:82-89.
__device__ __forceinline__ float hybrid_blend(float dense, float lex, float w, float inv) {
    return __fadd_rn(__fmul_rn(w, dense), __fmul_rn(__fmul_rn(__fsub_rn(1.0f, w), lex), inv));
}

// 1 / max(0, max of the lexical partial maxima of query q), or 0 when that max is not positive
// (src/cuda/lexical.cu:66-67). Called by one thread.
__device__ __forceinline__ float hybrid_inverse(const ScanParams& p, int q) {
    float peak = 0.0f;
    for (int i = 0; i < p.lex_parts; ++i) peak = fmaxf(peak, p.lex_part[static_cast<size_t>(q) * p.lex_parts + i]);
    return peak > 0.0f ? __fdiv_rn(1.0f, peak) : 0.0f;
}

template <int MODE>
struct ModeTraits;
template <>
struct ModeTraits<kModeF32> {
    static constexpr int kEpc = 4;  // fp32 query values per 16-byte chunk
    static constexpr int kElemBytes = 4;
};
template <>
struct ModeTraits<kModeF16> {
    static constexpr int kEpc = 8;
    static constexpr int kElemBytes = 2;
};
template <>
struct ModeTraits<kModeI8M> {
    static constexpr int kEpc = 16;
    static constexpr int kElemBytes = 1;
};
template <>
struct ModeTraits<kModeI8R> {
    static constexpr int kEpc = 4;  // four packed int8x4 words per chunk
    static constexpr int kElemBytes = 1;
};
template <>
struct ModeTraits<kModeBin> {
    static constexpr int kEpc = 4;  // four 32-bit words per chunk
    static constexpr int kElemBytes = 4;
};

__device__ __forceinline__ uint4 lds128(const void* p) {
    return *reinterpret_cast<const uint4*>(p);
}

// Accumulates one 16-byte corpus chunk against one query's matching values.
template <int MODE, bool L2>
__device__ __forceinline__ void accumulate_chunk(const uint4 raw, const float* qv, float scale,
                                                 float& acc) {
    auto step = [&](float x, float q) {
        if constexpr (L2) {
            const float d = q - x;
            acc = fmaf(d, d, acc);
        } else {
            acc = fmaf(q, x, acc);
        }
    };
    if constexpr (MODE == kModeF32) {
        step(__uint_as_float(raw.x), qv[0]);
        step(__uint_as_float(raw.y), qv[1]);
        step(__uint_as_float(raw.z), qv[2]);
        step(__uint_as_float(raw.w), qv[3]);
    } else if constexpr (MODE == kModeF16) {
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
            step(f.x, qv[2 * i]);
            step(f.y, qv[2 * i + 1]);
        }
    } else if constexpr (MODE == kModeI8M) {
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int8_t v = static_cast<int8_t>((w[i] >> (8 * b)) & 0xffu);
                step(static_cast<float>(v) * scale, qv[4 * i + b]);
            }
        }
    }
}

__device__ __forceinline__ int dp4a_chunk(const uint4 raw, const int* qw, int acc) {
    acc = __dp4a(static_cast<int>(raw.x), qw[0], acc);
    acc = __dp4a(static_cast<int>(raw.y), qw[1], acc);
    acc = __dp4a(static_cast<int>(raw.z), qw[2], acc);
    acc = __dp4a(static_cast<int>(raw.w), qw[3], acc);
    return acc;
}

// Stages the query pass into shared memory in the form the row loop consumes: fp32 values
// zero-padded to whole chunks, per-row int8 quantisation (I8R) or packed sign bits (Bin).
template <int MODE, int QB, int NT = kScanThreads>
__device__ void stage_queries(const ScanParams& p, uint8_t* qsmem, float* qscale, int q0,
                              int nq, float* red /* [(NT / 32) * QB] */) {
    constexpr int kWarps = NT / 32;
    const int tid = threadIdx.x;
    if constexpr (MODE == kModeF32 || MODE == kModeF16 || MODE == kModeI8M) {
        const int qf = p.query_bytes / 4;
        float* dst = reinterpret_cast<float*>(qsmem);
        const float* src = static_cast<const float*>(p.queries);
        for (int e = tid; e < QB * qf; e += NT) {
            const int q = e / qf;
            const int j = e - q * qf;
            dst[e] = (q < nq && j < p.dim) ? src[static_cast<size_t>(q0 + q) * p.dim + j] : 0.0f;
        }
    } else if constexpr (MODE == kModeI8R) {
        // s = max|x| / 127 (1 when the row is all zero), q = clamp(rint(x * (1/s)), -127, 127):
        // the reference quantiser (src/cuda/convert.cu:25-32) applied with a per-row scale.
        const float* src = static_cast<const float*>(p.queries);
        float amax[QB];
#pragma unroll
        for (int q = 0; q < QB; ++q) amax[q] = 0.0f;
        for (int j = tid; j < p.dim; j += NT) {
#pragma unroll
            for (int q = 0; q < QB; ++q) {
                if (q < nq) amax[q] = fmaxf(amax[q], fabsf(src[static_cast<size_t>(q0 + q) * p.dim + j]));
            }
        }
#pragma unroll
        for (int q = 0; q < QB; ++q) {
            const float m = warp_max_f32(amax[q]);
            if ((tid & 31) == 0) red[q * kWarps + (tid >> 5)] = m;
        }
        __syncthreads();
        if (tid < QB) {
            float m = 0.0f;
            for (int w = 0; w < kWarps; ++w) m = fmaxf(m, red[tid * kWarps + w]);
            qscale[tid] = (m > 0.0f) ? __fdiv_rn(m, 127.0f) : 1.0f;
        }
        __syncthreads();
        int8_t* dst = reinterpret_cast<int8_t*>(qsmem);
        for (int e = tid; e < QB * p.query_bytes; e += NT) {
            const int q = e / p.query_bytes;
            const int j = e - q * p.query_bytes;
            int8_t v = 0;
            if (q < nq && j < p.dim) {
                const float inv = __fdiv_rn(1.0f, qscale[q]);
                const float r = rintf(__fmul_rn(src[static_cast<size_t>(q0 + q) * p.dim + j], inv));
                v = static_cast<int8_t>(fminf(fmaxf(r, -127.0f), 127.0f));
            }
            dst[e] = v;
        }
    } else {  // kModeBin
        const int qw = p.query_bytes / 4;
        const int words = (p.dim + 31) / 32;
        uint32_t* dst = reinterpret_cast<uint32_t*>(qsmem);
        for (int e = tid; e < QB * qw; e += NT) {
            const int q = e / qw;
            const int w = e - q * qw;
            uint32_t bits = 0u;
            if (q < nq && w < words) {
                if (p.query_packed) {
                    bits = static_cast<const uint32_t*>(p.queries)[static_cast<size_t>(q0 + q) * words + w];
                } else {
                    const float* row = static_cast<const float*>(p.queries) + static_cast<size_t>(q0 + q) * p.dim;
                    for (int b = 0; b < 32; ++b) {
                        const int d = 32 * w + b;
                        if (d < p.dim && row[d] >= 0.0f) bits |= (1u << b);
                    }
                }
            }
            dst[e] = bits;
        }
    }
}

// Copies `rows` rows into a stage with the 16-byte padded stride (non-TMA path).
template <int ELEM_BYTES>
__device__ void fill_stage_plain(const ScanParams& p, uint8_t* stage, long long row0, int rows) {
    // Rows only; per-row side data is loaded by the caller.
    using Elem = typename std::conditional<ELEM_BYTES == 4, uint32_t,
                 typename std::conditional<ELEM_BYTES == 2, uint16_t, uint8_t>::type>::type;
    const int epr = p.elems_per_row;
    const int spr = p.stride / ELEM_BYTES;
    const Elem* src = reinterpret_cast<const Elem*>(p.corpus) + row0 * epr;
    Elem* dst = reinterpret_cast<Elem*>(stage);
    const int total = rows * spr;
    for (int i = threadIdx.x; i < total; i += kScanThreads) {
        const int r = i / spr;
        const int e = i - r * spr;
        dst[i] = (e < epr) ? src[static_cast<size_t>(r) * epr + e] : Elem(0);
    }
}

// MODE: storage; QB: queries per pass; JC: chunks per lane held in registers (0 = generic
// loop, query read from shared memory); LPR: lanes per row (32 / LPR lane groups per warp);
// RW: rows each lane group scores per iteration; L2: metric; EMIT: write the score matrix
// instead of selecting. One warp iteration scores (32 / LPR) * RW rows and shares a single
// reduction and epilogue among them.
template <int MODE, int QB, int JC, int LPR, int RW, bool L2, bool EMIT>
__global__ void __launch_bounds__(kScanThreads, 1) scan_kernel(const ScanParams p) {
    using Traits = ModeTraits<MODE>;
    constexpr int EPC = Traits::kEpc;
    constexpr bool kInt = (MODE == kModeI8R);
    constexpr int RPW = 32 / LPR;              // lane groups per warp
    constexpr int kRowsPerWarp = RPW * RW;     // rows per warp iteration
    constexpr int kRowsPerStep = kScanWarps * kRowsPerWarp;
    constexpr int V = RW * QB;                 // partial sums per lane
    static_assert(V <= LPR, "more partial sums than lanes in a row group");
    constexpr int kGroupShift = Log2<LPR>::value - Log2<V>::value;

    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float s_red[kScanWarps * QB];
    __shared__ float s_qscale[QB];
    __shared__ float s_inv[QB];
    __shared__ u64 s_scratch[32];
    __shared__ int s_last;
    __shared__ int s_abort;

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int pass = blockIdx.x;
    const int cta = blockIdx.y;
    const int G = gridDim.y;
    const int q0 = pass * QB;
    const int nq = min(QB, p.batch - q0);

    const int R = p.rows_per_tile;
    const int stage_bytes = p.stage_bytes;
    uint8_t* stages = smem;
    uint8_t* qsmem = smem + p.smem_query_off;
    u64* bars = reinterpret_cast<u64*>(smem + p.smem_bar_off);
    const bool need_side = p.side_scales || p.mask != nullptr;

    TopkSmem tk;
    tk.buf = reinterpret_cast<u64*>(smem + p.smem_topk_off);
    tk.count = reinterpret_cast<int*>(tk.buf + QB * p.cap);
    tk.thr = reinterpret_cast<u64*>(tk.count + 2 * QB);  // 8-byte aligned
    tk.cap = p.cap;
    tk.k = p.k;

    const int t_begin = static_cast<int>((p.ntiles * cta) / G);
    const int t_end = static_cast<int>((p.ntiles * (cta + 1)) / G);
    const int my_tiles = t_end - t_begin;
    const int S = p.use_tma ? p.stages : 1;

    // One bulk copy per tile for the rows, plus (full tiles only) one each for the per-row
    // scales and allow-mask bytes, all completing on the stage's mbarrier.
    auto issue = [&](int i, int s) {
        const int row0 = (t_begin + i) * R;
        const int rows = min(R, static_cast<int>(p.n - row0));
        const uint32_t bytes = static_cast<uint32_t>(rows) * static_cast<uint32_t>(p.row_bytes);
        const bool side_bulk = p.side_tma && rows == R;
        uint32_t total = bytes;
        if (side_bulk) {
            if (p.side_scales) total += 4u * R;
            if (p.mask != nullptr) total += R;
        }
        uint8_t* st = stages + s * stage_bytes;
        u64* bar = &bars[s];
        mbar_arrive_expect_tx(bar, total);
        bulk_copy_g2s(st, p.corpus + static_cast<size_t>(row0) * p.row_bytes, bytes, bar);
        if (side_bulk) {
            if (p.side_scales) bulk_copy_g2s(st + p.side_off_scales, p.row_scales + row0, 4u * R, bar);
            if (p.mask != nullptr) bulk_copy_g2s(st + p.side_off_mask, p.mask + row0, R, bar);
        }
    };

    if (tid == 0) s_abort = 0;
    if (p.use_tma) {
        if (tid == 0) {
            for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
            fence_mbarrier_init();
        }
        __syncthreads();
        if (tid == 0) {
            for (int i = 0; i < S && i < my_tiles; ++i) issue(i, i);
        }
    }

    stage_queries<MODE, QB>(p, qsmem, s_qscale, q0, nq, s_red);
    if (!EMIT && tid < QB) {
        tk.count[tid] = 0;
        tk.thr[tid] = 0ull;
        s_inv[tid] = (p.lex != nullptr && tid < nq) ? hybrid_inverse(p, q0 + tid) : 0.0f;
    }
    __syncthreads();

    // Warp-mode lane roles: lane group `grp` scores row (step base + grp); lane `gl` of the
    // group owns 16-byte chunks gl, gl + LPR, ...
    const int grp = lane / LPR;
    const int gl = lane % LPR;

    // Register-resident query slices for the fast path (JC chunks per lane).
    using QElem = typename std::conditional<kInt, int, float>::type;
    QElem qreg[JC > 0 ? JC : 1][QB][EPC];
    if constexpr (JC > 0 && MODE != kModeBin) {
#pragma unroll
        for (int j = 0; j < JC; ++j) {
            const int c = gl + LPR * j;
#pragma unroll
            for (int q = 0; q < QB; ++q) {
#pragma unroll
                for (int e = 0; e < EPC; ++e) {
                    qreg[j][q][e] = (c < p.nch)
                        ? reinterpret_cast<const QElem*>(qsmem + q * p.query_bytes)[c * EPC + e]
                        : QElem(0);
                }
            }
        }
    }

    bool aborted = false;
    int i = 0;
    int s = 0;
    uint32_t phase = 0;
    for (; i < my_tiles; ++i) {
        const int row0 = (t_begin + i) * R;
        const int rows = min(R, static_cast<int>(p.n - row0));
        bool failed = false;
        if (p.use_tma) {
            failed = !mbar_wait_bounded(&bars[s], phase, p.status, kStatusTileWaitTimeout);
        } else {
            fill_stage_plain<Traits::kElemBytes>(p, stages, row0, rows);
        }
        uint8_t* st = stages + s * stage_bytes;
        const bool side_plain = need_side && !(p.use_tma && p.side_tma && rows == R);
        if (side_plain) {
            for (int r = tid; r < rows; r += kScanThreads) {
                if (p.side_scales) reinterpret_cast<float*>(st + p.side_off_scales)[r] = __ldg(p.row_scales + row0 + r);
                if (p.mask != nullptr) st[p.side_off_mask + r] = __ldg(p.mask + row0 + r);
            }
        }
        if (!p.use_tma || side_plain) __syncthreads();
        const float* side_scale = reinterpret_cast<const float*>(st + p.side_off_scales);
        const uint8_t* side_mask = st + p.side_off_mask;
        const uint32_t id0 = p.id_base + static_cast<uint32_t>(row0);
        bool need_flush = false;

        if constexpr (MODE == kModeBin) {
            // Thread per row. Each thread starts its chunk walk at a row-dependent offset so a
            // quarter-warp's 16-byte reads fall in distinct bank groups.
            for (int r = tid; r < rows; r += kScanThreads) {
                const uint8_t* rowp = st + r * p.stride;
                int h[QB];
#pragma unroll
                for (int q = 0; q < QB; ++q) h[q] = 0;
                int u = r % p.nch;
                for (int c = 0; c < p.nch; ++c) {
                    const uint4 w = lds128(rowp + u * 16);
#pragma unroll
                    for (int q = 0; q < QB; ++q) {
                        const uint4 qw = lds128(qsmem + q * p.query_bytes + u * 16);
                        h[q] += __popc(w.x ^ qw.x) + __popc(w.y ^ qw.y) + __popc(w.z ^ qw.z) +
                                __popc(w.w ^ qw.w);
                    }
                    u = (u + 1 == p.nch) ? 0 : u + 1;
                }
                const bool masked = (p.mask != nullptr) && side_mask[r] == 0;
#pragma unroll
                for (int q = 0; q < QB; ++q) {
                    if (q < nq) {
                        float score = __fdiv_rn(static_cast<float>(p.dim - 2 * h[q]),
                                                static_cast<float>(p.dim));
                        if (masked) score = -FLT_MAX;
                        if (!EMIT && p.lex != nullptr) {
                            score = hybrid_blend(score, __ldg(p.lex + static_cast<size_t>(q0 + q) * p.n + row0 + r),
                                                 p.dense_weight, s_inv[q]);
                        }
                        if constexpr (EMIT) {
                            p.out_matrix[static_cast<size_t>(q0 + q) * p.n + row0 + r] = score;
                        } else {
                            need_flush |= topk_offer_check(tk, q, make_key(score, id0 + r), R);
                        }
                    }
                }
            }
        } else {
            for (int rb = warp * kRowsPerWarp; rb < rows; rb += kRowsPerStep) {
                QElem acc[V];
#pragma unroll
                for (int v = 0; v < V; ++v) acc[v] = QElem(0);
#pragma unroll
                for (int rr = 0; rr < RW; ++rr) {
                    const int r = rb + rr * RPW + grp;    // uniform within the lane group
                    if (r >= rows) continue;
                    const uint8_t* rowp = st + r * p.stride;
                    if constexpr (JC > 0) {
                        // The fast path is only planned when the row is exactly JC sweeps of
                        // the group, so every chunk index is in range.
#pragma unroll
                        for (int j = 0; j < JC; ++j) {
                            const int c = gl + LPR * j;
                            const uint4 raw = lds128(rowp + c * 16);
#pragma unroll
                            for (int q = 0; q < QB; ++q) {
                                if constexpr (kInt) {
                                    acc[rr * QB + q] = dp4a_chunk(raw, qreg[j][q], acc[rr * QB + q]);
                                } else {
                                    accumulate_chunk<MODE, L2>(raw, qreg[j][q], p.scale, acc[rr * QB + q]);
                                }
                            }
                        }
                    } else {
                        for (int c = gl; c < p.nch; c += LPR) {
                            const uint4 raw = lds128(rowp + c * 16);
#pragma unroll
                            for (int q = 0; q < QB; ++q) {
                                const uint8_t* qrow = qsmem + q * p.query_bytes + c * EPC * sizeof(QElem);
                                QElem qv[EPC];
#pragma unroll
                                for (int e = 0; e < EPC; e += 4) {
                                    const uint4 v = lds128(qrow + e * sizeof(QElem));
                                    qv[e] = *reinterpret_cast<const QElem*>(&v.x);
                                    qv[e + 1] = *reinterpret_cast<const QElem*>(&v.y);
                                    qv[e + 2] = *reinterpret_cast<const QElem*>(&v.z);
                                    qv[e + 3] = *reinterpret_cast<const QElem*>(&v.w);
                                }
                                if constexpr (kInt) {
                                    acc[rr * QB + q] = dp4a_chunk(raw, qv, acc[rr * QB + q]);
                                } else {
                                    accumulate_chunk<MODE, L2>(raw, qv, p.scale, acc[rr * QB + q]);
                                }
                            }
                        }
                    }
                }
                transpose_reduce<V, LPR>(acc, lane);
                const int idx = gl >> kGroupShift;
                const int q = idx % QB;
                const int r = rb + (idx / QB) * RPW + grp;
                if ((gl & ((1 << kGroupShift) - 1)) == 0 && q < nq && r < rows) {
                    float score;
                    if constexpr (kInt) {
                        score = __fmul_rn(__fmul_rn(__int2float_rn(acc[0]), s_qscale[q]), side_scale[r]);
                    } else {
                        score = L2 ? -acc[0] : acc[0];
                    }
                    if (p.mask != nullptr && side_mask[r] == 0) score = -FLT_MAX;
                    if (!EMIT && p.lex != nullptr) {
                        score = hybrid_blend(score, __ldg(p.lex + static_cast<size_t>(q0 + q) * p.n + row0 + r),
                                             p.dense_weight, s_inv[q]);
                    }
                    if constexpr (EMIT) {
                        p.out_matrix[static_cast<size_t>(q0 + q) * p.n + row0 + r] = score;
                    } else {
                        need_flush |= topk_offer_check(tk, q, make_key(score, id0 + r), R);
                    }
                }
            }
        }

        // One barrier per tile. It both releases the stage for the next bulk copy and tells
        // every thread whether some buffer needs a flush or some wait ran out (rare paths).
        if (failed) s_abort = 1;
        if (__syncthreads_or(failed || need_flush)) {
            aborted = s_abort != 0;
            if constexpr (!EMIT) {
                uint32_t mask = 0;
                for (int q = 0; q < nq; ++q) {
                    if (tk.count[q] > tk.cap - R) mask |= 1u << q;
                }
                topk_flush_mask(tk, mask, kScanThreads);
            }
            if (aborted) break;
        }
        if (p.use_tma && tid == 0 && i + S < my_tiles) {
            fence_proxy_async_shared();
            issue(i + S, s);
        }
        if (++s == S) {
            s = 0;
            phase ^= 1u;
        }
    }

    // A wait ran out: make sure no bulk copy into this CTA's shared memory is still pending
    // before the CTA can retire (bounded as well), then finish normally so the workspace
    // counters stay consistent; the status word tells the host the results are invalid.
    if (aborted && p.use_tma && tid == 0) {
        const int last = min(i + S - 1, my_tiles - 1);
        for (int j = i; j <= last; ++j) {
            mbar_wait_bounded(&bars[j % S], static_cast<uint32_t>((j / S) & 1), p.status,
                              kStatusDrainTimeout);
        }
    }
    if constexpr (EMIT) return;

    __syncthreads();
    topk_flush_all(tk, nq, kScanThreads);
    for (int q = 0; q < nq; ++q) {
        unsigned long long* dst = p.lists + (static_cast<size_t>(q0 + q) * G + cta) * p.k;
        const int n = tk.count[q];
        for (int j = tid; j < p.k; j += kScanThreads) dst[j] = j < n ? tk.buf[q * p.cap + j] : 0ull;
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
    // The stage ring is idle now: it holds the merge buffer (p.cap_final keys).
    __shared__ int s_merge_count;
    __shared__ u64 s_merge_thr;
    TopkSmem mt;
    mt.buf = reinterpret_cast<u64*>(stages);
    mt.count = &s_merge_count;
    mt.thr = &s_merge_thr;
    mt.cap = p.cap_final;
    mt.k = p.k;
    for (int q = 0; q < nq; ++q) {
        const unsigned long long* src = p.lists + static_cast<size_t>(q0 + q) * G * p.k;
        topk_merge_lists(mt, 0, src, G, kScanThreads, s_scratch);
        topk_write(mt, 0, p.out_idx + static_cast<size_t>(q0 + q) * p.k,
                   p.out_scores + static_cast<size_t>(q0 + q) * p.k, kScanThreads);
        __syncthreads();
    }
    if (tid == 0) p.counters[pass] = 0u;
}

}  // namespace zc
