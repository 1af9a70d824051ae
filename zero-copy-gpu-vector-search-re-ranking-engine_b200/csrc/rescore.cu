// Candidate rescoring: gather + exact score + second top-k + id remap in one kernel.
//
// Replaces the reference's rescore chain of Searcher::recordPipeline
// (src/search/searcher.cpp:266-279): launchGatherRescore (src/cuda/rescore.cu:20-63, a block per
// (candidate, query) that re-stages the query and writes a [batch, M] score matrix), a second
// launchTopK over that matrix, and launchRemapIndices (:65-79) from candidate positions back to
// corpus ids. Here one kernel does all of it on chip:
//
//   * Work split: the M candidates of a query are cut into contiguous slices, one per CTA of a
//     thread-block cluster (grid = [C, batch], cluster = C CTAs). C grows when the batch is
//     too small to fill the GPU, so a single query's gather is spread over up to 8 SMs.
//   * Gather: a warp per candidate row; kRows rows per warp are in flight at once, every lane
//     loading 16-byte chunks of each (rows that are not 16-byte multiples take an element-wise
//     path). The query is staged once per CTA in shared memory, in the same form the corpus
//     scan uses (fp32, or per-row int8 for ZCGVS_DTYPE_I8_ROW).
//   * Selection: each candidate becomes a 64-bit key (score, global id), so ties break on the
//     corpus id (score desc, id asc) and the remap step disappears. A CTA sorts its slice and
//     keeps k keys; rank 0 of the cluster pulls the other CTAs' lists through distributed
//     shared memory and selects the final k.
//
// Numerics follow the reference: rows are widened to fp32 and multiplied by the fp32 query
// (src/cuda/rescore.cu:52-56, decode.cuh:22-43), L2 is -sum((q - x)^2); per-row int8 stores
// score float(int32 dot) * s_q * s_row exactly. Candidates outside [0, doc_count) are dropped
// (the reference scores them -FLT_MAX, :45-50), so they never displace a real document.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <string>

#include "host_common.h"
#include "scan_kernel.cuh"
#include "zcgvs_sm100.h"

namespace cg = cooperative_groups;

namespace zc {

constexpr int kRescoreThreads = 256;
constexpr int kRescoreWarps = kRescoreThreads / 32;
constexpr int kRescoreRows = 4;          // rows in flight per warp
constexpr int kRescoreMaxCluster = 8;
constexpr int kRescoreMaxKeys = 8192;    // key buffer limit per CTA (64 KB)

struct RescoreParams {
    const uint8_t* store;
    const float* row_scales;
    float scale;
    long long n;
    int dim;
    int row_bytes;
    int vec;                // rows are 16-byte multiples on 16-byte boundaries
    int nch;                // 16-byte chunks per row (vector path)
    const float* queries;
    int query_bytes;        // staged query bytes (multiple of 16)
    const int* candidates;  // [batch, m]
    int m;
    int k;
    int slice;              // candidates per CTA
    int cap;                // key buffer capacity (power of two)
    int* out_idx;           // fused mode: [batch, k]
    float* out_scores;
    float* out_values;      // score-matrix mode: [batch, m]
};

template <int MODE>
__device__ __forceinline__ float decode_elem(const uint8_t* row, int j, float scale) {
    if constexpr (MODE == kModeF32) {
        return reinterpret_cast<const float*>(row)[j];
    } else if constexpr (MODE == kModeF16) {
        return __half2float(reinterpret_cast<const __half*>(row)[j]);
    } else {
        return static_cast<float>(reinterpret_cast<const int8_t*>(row)[j]) * scale;
    }
}

// Scores kRescoreRows candidate slots [base, base + kRescoreRows) of query `q` with one warp.
// Returns, in lane rr, the key of slot base + rr (0 when the slot is empty or invalid) and,
// through `score_out`, its score (-FLT_MAX when invalid).
template <int MODE, bool L2>
__device__ __forceinline__ void score_rows(const RescoreParams& p, const uint8_t* qsmem, float qscale,
                                           int q, int base, int end, int lane, u64& key_out,
                                           float& score_out) {
    constexpr bool kInt = (MODE == kModeI8R);
    using Acc = typename std::conditional<kInt, int, float>::type;
    int id[kRescoreRows];
    bool ok[kRescoreRows];
    Acc acc[kRescoreRows];
#pragma unroll
    for (int rr = 0; rr < kRescoreRows; ++rr) {
        const int slot = base + rr;
        id[rr] = slot < end ? __ldg(p.candidates + static_cast<size_t>(q) * p.m + slot) : -1;
        ok[rr] = id[rr] >= 0 && id[rr] < p.n;
        acc[rr] = Acc(0);
    }
    if (p.vec) {
        constexpr int kEpc = ModeTraits<MODE>::kEpc;
        // Four steps (16 row loads per lane) in flight: a 2 KB row is four steps of a warp.
#pragma unroll 4
        for (int c = lane; c < p.nch; c += 32) {
            uint4 raw[kRescoreRows];
#pragma unroll
            for (int rr = 0; rr < kRescoreRows; ++rr) {
                raw[rr] = ok[rr] ? __ldg(reinterpret_cast<const uint4*>(
                                       p.store + static_cast<size_t>(id[rr]) * p.row_bytes) + c)
                                 : make_uint4(0u, 0u, 0u, 0u);
            }
            if constexpr (kInt) {
                const int4 qw = reinterpret_cast<const int4*>(qsmem)[c];
                const int qv[4] = {qw.x, qw.y, qw.z, qw.w};
#pragma unroll
                for (int rr = 0; rr < kRescoreRows; ++rr) acc[rr] = dp4a_chunk(raw[rr], qv, acc[rr]);
            } else {
                float qv[kEpc];
#pragma unroll
                for (int e = 0; e < kEpc; e += 4) {
                    const float4 f = reinterpret_cast<const float4*>(qsmem)[(c * kEpc + e) / 4];
                    qv[e] = f.x;
                    qv[e + 1] = f.y;
                    qv[e + 2] = f.z;
                    qv[e + 3] = f.w;
                }
#pragma unroll
                for (int rr = 0; rr < kRescoreRows; ++rr) accumulate_chunk<MODE, L2>(raw[rr], qv, p.scale, acc[rr]);
            }
        }
    } else {
        for (int j = lane; j < p.dim; j += 32) {
#pragma unroll
            for (int rr = 0; rr < kRescoreRows; ++rr) {
                if (!ok[rr]) continue;
                const uint8_t* row = p.store + static_cast<size_t>(id[rr]) * p.row_bytes;
                if constexpr (kInt) {
                    acc[rr] += static_cast<int>(reinterpret_cast<const int8_t*>(row)[j]) *
                               static_cast<int>(reinterpret_cast<const int8_t*>(qsmem)[j]);
                } else {
                    const float x = decode_elem<MODE>(row, j, p.scale);
                    const float qv = reinterpret_cast<const float*>(qsmem)[j];
                    if constexpr (L2) {
                        const float d = qv - x;
                        acc[rr] = fmaf(d, d, acc[rr]);
                    } else {
                        acc[rr] = fmaf(qv, x, acc[rr]);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int rr = 0; rr < kRescoreRows; ++rr) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc[rr] += __shfl_xor_sync(0xffffffffu, acc[rr], off);
    }
    key_out = 0ull;
    score_out = -FLT_MAX;
#pragma unroll
    for (int rr = 0; rr < kRescoreRows; ++rr) {
        if (lane == rr && ok[rr]) {
            float score;
            if constexpr (kInt) {
                score = __fmul_rn(__fmul_rn(__int2float_rn(acc[rr]), qscale), __ldg(p.row_scales + id[rr]));
            } else {
                score = L2 ? -acc[rr] : acc[rr];
            }
            score_out = score;
            key_out = make_key(score, static_cast<uint32_t>(id[rr]));
        }
    }
}

// EMIT = false: fused rescore + top-k; EMIT = true: [batch, m] score matrix (the reference
// launchGatherRescore contract).
template <int MODE, bool L2, bool EMIT>
__global__ void __launch_bounds__(kRescoreThreads) rescore_kernel(const RescoreParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float s_red[kRescoreWarps];
    __shared__ float s_qscale[1];
    __shared__ int s_count;
    __shared__ u64 s_thr;
    u64* keys = reinterpret_cast<u64*>(smem);
    uint8_t* qsmem = smem + static_cast<size_t>(p.cap) * sizeof(u64);

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int q = blockIdx.y;
    const int rank = blockIdx.x;
    const int s0 = rank * p.slice;
    const int s1 = min(p.m, s0 + p.slice);

    ScanParams sp{};
    sp.queries = p.queries;
    sp.dim = p.dim;
    sp.query_bytes = p.query_bytes;
    stage_queries<MODE, 1, kRescoreThreads>(sp, qsmem, s_qscale, q, 1, s_red);
    if constexpr (!EMIT) {
        for (int i = tid; i < p.cap; i += kRescoreThreads) keys[i] = 0ull;
    }
    __syncthreads();
    const float qscale = s_qscale[0];

    for (int base = s0 + warp * kRescoreRows; base < s1; base += kRescoreWarps * kRescoreRows) {
        u64 key;
        float score;
        score_rows<MODE, L2>(p, qsmem, qscale, q, base, s1, lane, key, score);
        if (lane < kRescoreRows && base + lane < s1) {
            if constexpr (EMIT) {
                p.out_values[static_cast<size_t>(q) * p.m + base + lane] = score;
            } else {
                keys[base + lane - s0] = key;
            }
        }
    }
    if constexpr (EMIT) return;

    TopkSmem t;
    t.buf = keys;
    t.count = &s_count;
    t.thr = &s_thr;
    t.cap = p.cap;
    t.k = p.k;
    if (tid == 0) s_count = max(s1 - s0, 0);
    __syncthreads();
    topk_flush_mask(t, 1u, kRescoreThreads);
    __syncthreads();

    const int C = gridDim.x;
    if (C > 1) {
        cg::cluster_group cluster = cg::this_cluster();
        cluster.sync();  // every CTA's list is sorted
        if (rank == 0) {
            for (int r = 1; r < C; ++r) {
                const u64* remote = cluster.map_shared_rank(keys, r);
                for (int j = tid; j < p.k; j += kRescoreThreads) keys[r * p.k + j] = remote[j];
            }
        }
        cluster.sync();  // the other CTAs' shared memory may be released after this
        if (rank != 0) return;
        if (tid == 0) s_count = C * p.k;
        __syncthreads();
        topk_flush_mask(t, 1u, kRescoreThreads);
        __syncthreads();
    }
    topk_write(t, 0, p.out_idx + static_cast<size_t>(q) * p.k, p.out_scores + static_cast<size_t>(q) * p.k,
               kRescoreThreads);
}

using RescoreFn = void (*)(const RescoreParams);

template <bool EMIT>
RescoreFn rescore_lookup(int mode, bool l2) {
    switch (mode) {
        case kModeF32: return l2 ? rescore_kernel<kModeF32, true, EMIT> : rescore_kernel<kModeF32, false, EMIT>;
        case kModeF16: return l2 ? rescore_kernel<kModeF16, true, EMIT> : rescore_kernel<kModeF16, false, EMIT>;
        case kModeI8M: return l2 ? rescore_kernel<kModeI8M, true, EMIT> : rescore_kernel<kModeI8M, false, EMIT>;
        case kModeI8R: return rescore_kernel<kModeI8R, false, EMIT>;
        default: return nullptr;
    }
}

namespace {

struct RescorePlan {
    RescoreParams p{};
    int cluster = 1;
    size_t smem = 0;
};

// Validates the arguments shared by both entry points and fills the plan.
int plan_rescore(const void* store, int dtype, float scale, const float* row_scales, int64_t doc_count,
                 int dim, const float* queries, int batch, const int* candidates, int m, int metric,
                 int k, bool emit, RescorePlan* plan) {
    if (dtype == ZCGVS_DTYPE_BINARY) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs rescore: the rescore store must hold float32, float16 or int8 rows");
    }
    if (dtype < ZCGVS_DTYPE_F32 || dtype > ZCGVS_DTYPE_I8_ROW) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs rescore: unknown dtype");
    if (metric < ZCGVS_METRIC_COSINE || metric > ZCGVS_METRIC_L2) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs rescore: unknown metric");
    if (dtype == ZCGVS_DTYPE_I8_ROW && metric == ZCGVS_METRIC_L2) {
        return fail(ZCGVS_ERR_UNSUPPORTED, "zcgvs rescore: L2 is not defined for per-row int8 stores");
    }
    if (store == nullptr || queries == nullptr || candidates == nullptr) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs rescore: null store, query or candidate pointer");
    }
    if (dtype == ZCGVS_DTYPE_I8_ROW && row_scales == nullptr) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs rescore: per-row int8 stores need row_scales");
    }
    if (doc_count > INT32_MAX) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs rescore: doc_count exceeds int32 ids");
    if (m > kRescoreMaxKeys) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs rescore: candidate_count exceeds " + std::to_string(kRescoreMaxKeys));
    }
    if (!emit) {
        if (k <= 0 || k > ZCGVS_MAX_K) {
            return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs rescore: k must be in [1, " + std::to_string(ZCGVS_MAX_K) + "]");
        }
        if (k > m) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs rescore: k exceeds candidate_count");
    }
    const int mode = dtype;  // ScanMode codes equal the ABI dtype codes
    RescoreParams& p = plan->p;
    p.store = static_cast<const uint8_t*>(store);
    p.row_scales = row_scales;
    p.scale = scale;
    p.n = doc_count;
    p.dim = dim;
    p.row_bytes = static_cast<int>(row_bytes_of(dtype, dim));
    p.vec = (p.row_bytes % 16 == 0) && (reinterpret_cast<uintptr_t>(store) % 16 == 0);
    p.nch = p.row_bytes / 16;
    // Staged query: fp32 values covering whole chunks, or int8 bytes for per-row int8.
    const int chunks = (p.row_bytes + 15) / 16;
    const int epc = (mode == kModeF32) ? 4 : (mode == kModeF16) ? 8 : 16;
    p.query_bytes = (mode == kModeI8R) ? chunks * 16 : chunks * epc * 4;
    p.queries = queries;
    p.candidates = candidates;
    p.m = m;
    p.k = emit ? 1 : k;

    // Cluster size: enough CTAs to cover the SMs when the batch is small, at least 32
    // candidates per CTA, and room for every list in rank 0's buffer.
    int cluster = 1;
    if (!emit) {
        const int sms = device_sm_count();
        cluster = std::max(1, std::min(kRescoreMaxCluster, (4 * sms + batch - 1) / std::max(batch, 1)));
        cluster = std::min(cluster, std::max(1, m / 32));
        while (cluster > 1 && static_cast<long long>(cluster) * k > kRescoreMaxKeys) --cluster;
    } else {
        cluster = std::max(1, std::min(kRescoreMaxCluster, (m + 63) / 64));
    }
    p.slice = (m + cluster - 1) / cluster;
    const int want = std::max(p.slice, emit ? 1 : cluster * k);
    p.cap = emit ? 0 : next_pow2(std::max(want, 2));
    plan->cluster = cluster;
    plan->smem = static_cast<size_t>(p.cap) * sizeof(u64) + static_cast<size_t>(p.query_bytes);
    if (plan->smem > static_cast<size_t>(device_max_smem()) - 2048) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs rescore: dimension too large for the shared-memory query stage");
    }
    return ZCGVS_OK;
}

int launch_rescore(RescorePlan& plan, int dtype, int metric, int batch, bool emit, cudaStream_t stream) {
    const RescoreFn fn = emit ? rescore_lookup<true>(dtype, metric == ZCGVS_METRIC_L2)
                              : rescore_lookup<false>(dtype, metric == ZCGVS_METRIC_L2);
    if (fn == nullptr) return fail(ZCGVS_ERR_UNSUPPORTED, "zcgvs rescore: no kernel for this dtype/metric");
    const cudaError_t opt = ensure_smem_optin(reinterpret_cast<const void*>(fn));
    if (opt != cudaSuccess) return fail_cuda(opt, "cudaFuncSetAttribute(rescore shared memory)");
    // grid.y is limited to 65535: long batches run in chunks.
    constexpr int kMaxY = 65535;
    for (int q0 = 0; q0 < batch; q0 += kMaxY) {
        const int nq = std::min(kMaxY, batch - q0);
        RescoreParams p = plan.p;
        p.queries += static_cast<size_t>(q0) * p.dim;
        p.candidates += static_cast<size_t>(q0) * p.m;
        if (emit) {
            p.out_values += static_cast<size_t>(q0) * p.m;
        } else {
            p.out_idx += static_cast<size_t>(q0) * p.k;
            p.out_scores += static_cast<size_t>(q0) * p.k;
        }
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(static_cast<unsigned>(plan.cluster), static_cast<unsigned>(nq));
        cfg.blockDim = dim3(kRescoreThreads);
        cfg.dynamicSmemBytes = plan.smem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = static_cast<unsigned>(plan.cluster);
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaError_t e;
        {
            KernelTimer timer("rescore", stream);
            e = cudaLaunchKernelEx(&cfg, fn, p);
        }
        if (e != cudaSuccess) return fail_cuda(e, "zcgvs rescore launch");
    }
    return ok();
}

}  // namespace
}  // namespace zc

extern "C" {

int zcgvs_rescore_topk(const void* store, int dtype, float scale, const float* row_scales, int64_t doc_count,
                       int dim, const float* queries, int batch, const int* candidates, int candidate_count,
                       int metric, int k, int* out_indices, float* out_scores, void* stream) {
    using namespace zc;
    if (batch <= 0 || dim <= 0 || candidate_count <= 0) return ok();
    if (out_indices == nullptr || out_scores == nullptr) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_rescore_topk: null output pointer");
    }
    RescorePlan plan;
    int status = plan_rescore(store, dtype, scale, row_scales, doc_count, dim, queries, batch, candidates,
                              candidate_count, metric, k, false, &plan);
    if (status != ZCGVS_OK) return status;
    plan.p.out_idx = out_indices;
    plan.p.out_scores = out_scores;
    return launch_rescore(plan, dtype, metric, batch, false, static_cast<cudaStream_t>(stream));
}

int zcgvs_gather_rescore(const void* store, int dtype, float scale, const float* row_scales, int64_t doc_count,
                         int dim, const float* queries, int batch, const int* candidates, int candidate_count,
                         int metric, float* values, void* stream) {
    using namespace zc;
    if (batch <= 0 || dim <= 0 || candidate_count <= 0) return ok();
    if (values == nullptr) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_gather_rescore: null output pointer");
    RescorePlan plan;
    int status = plan_rescore(store, dtype, scale, row_scales, doc_count, dim, queries, batch, candidates,
                              candidate_count, metric, 1, true, &plan);
    if (status != ZCGVS_OK) return status;
    plan.p.out_values = values;
    return launch_rescore(plan, dtype, metric, batch, true, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
