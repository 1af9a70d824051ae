// Score-matrix top-k, converters and the index remap: the remaining launchers of the reference's
// src/cuda/ (topk.cu, convert.cu, rescore.cu:65-79) behind the C ABI, so that a caller that still
// computes a [batch, N] score matrix (or converts host matrices into stores) keeps working.
//
// zcgvs_topk: one thread-block cluster of up to 8 CTAs per score row (grid [C, batch]); each CTA
// offers its slice of the row into an on-chip top-k (rounds of 4 loads per thread in flight,
// flushes by CTA bitonic sort), and rank 0 pulls the other CTAs' k keys through distributed
// shared memory and selects the final k. It needs no scratch: the reference's four scratch
// buffers (src/cuda/topk.cu:132-189) are accepted by the C++ wrapper and left untouched.
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <string>

#include "common.cuh"
#include "host_common.h"
#include "topk_cta.cuh"
#include "zcgvs_sm100.h"

namespace cg = cooperative_groups;

namespace zc {

namespace {

constexpr int kRowThreads = 512;
constexpr int kRowCap = 4096;  // k (<= 1024) + 4 keys per thread per round
constexpr int kRowMaxCluster = 8;
constexpr int kConvertThreads = 256;

__global__ void __launch_bounds__(kRowThreads) topk_rows_kernel(const float* __restrict__ scores, long long n,
                                                                int k, int slice, int cap, int* out_idx,
                                                                float* out_scores) {
    extern __shared__ __align__(16) u64 row_keys[];
    __shared__ int s_count;
    __shared__ u64 s_thr;
    const int q = blockIdx.y;
    const int rank = blockIdx.x;
    const long long s0 = static_cast<long long>(rank) * slice;
    const int len = static_cast<int>(max(0LL, min(static_cast<long long>(slice), n - s0)));
    const float* row = scores + static_cast<size_t>(q) * n + s0;

    TopkSmem t;
    t.buf = row_keys;
    t.count = &s_count;
    t.thr = &s_thr;
    t.cap = cap;
    t.k = k;
    if (threadIdx.x == 0) {
        s_count = 0;
        s_thr = 0ull;
    }
    __syncthreads();
    topk_offer_all<4>(t, 0, len, 0ull,
                      [&](int i) { return make_key(__ldg(row + i), static_cast<uint32_t>(s0 + i)); }, kRowThreads);
    topk_flush_mask(t, 1u, kRowThreads);
    __syncthreads();

    const int C = gridDim.x;
    if (C > 1) {
        // Every list padded to k keys (key 0 = empty) for the merge.
        for (int j = s_count + threadIdx.x; j < k; j += kRowThreads) row_keys[j] = 0ull;
        cg::cluster_group cluster = cg::this_cluster();
        cluster.sync();  // every CTA's list is final
        if (rank == 0) {
            for (int r = 1; r < C; ++r) {
                const u64* remote = cluster.map_shared_rank(row_keys, r);
                for (int j = threadIdx.x; j < k; j += kRowThreads) row_keys[r * k + j] = remote[j];
            }
        }
        cluster.sync();  // the other CTAs may exit after this
        if (rank != 0) return;
        if (threadIdx.x == 0) s_count = C * k;
        __syncthreads();
        topk_flush_mask(t, 1u, kRowThreads);
        __syncthreads();
    }
    topk_write(t, 0, out_idx + static_cast<size_t>(q) * k, out_scores + static_cast<size_t>(q) * k, kRowThreads);
}

__global__ void convert_f16_kernel(const float* __restrict__ src, __half* __restrict__ dst, size_t count) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        dst[i] = __float2half_rn(src[i]);
    }
}

// rint(x * (1 / scale)) clamped to [-127, 127], the reciprocal taken on the host as in the
// reference launcher (src/cuda/convert.cu:25-32, :77-87).
__global__ void convert_i8_kernel(const float* __restrict__ src, int8_t* __restrict__ dst, size_t count, float inv) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const float r = rintf(__fmul_rn(src[i], inv));
        dst[i] = static_cast<int8_t>(fminf(fmaxf(r, -127.0f), 127.0f));
    }
}

// Per-row symmetric int8 (the per-row extension of src/cuda/convert.cu:17-32): one warp per row,
// scale = max|x| / 127 (1 for an all-zero row), then clamp(rint(x * (1 / scale)), +-127), both
// rounded as the host oracle rounds them. The max is order-independent, so any lane split gives
// the same scale. The row is read twice; the second pass hits L1 / L2 (rows of a few KB).
__global__ void __launch_bounds__(kConvertThreads) convert_i8_rows_kernel(const float* __restrict__ src,
                                                                          int8_t* __restrict__ dst,
                                                                          float* __restrict__ row_scales,
                                                                          long long rows, int dim, int vec) {
    const int lane = threadIdx.x & 31;
    const long long warps = static_cast<long long>(gridDim.x) * (kConvertThreads / 32);
    for (long long r = blockIdx.x * static_cast<long long>(kConvertThreads / 32) + (threadIdx.x >> 5); r < rows;
         r += warps) {
        const float* x = src + r * dim;
        int8_t* y = dst + r * dim;
        float peak = 0.0f;
        if (vec) {
            const float4* x4 = reinterpret_cast<const float4*>(x);
            for (int c = lane; c < dim / 4; c += 32) {
                const float4 v = __ldg(x4 + c);
                peak = fmaxf(peak, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
            }
        } else {
            for (int j = lane; j < dim; j += 32) peak = fmaxf(peak, fabsf(__ldg(x + j)));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) peak = fmaxf(peak, __shfl_xor_sync(0xffffffffu, peak, o));
        const float scale = peak > 0.0f ? __fdiv_rn(peak, 127.0f) : 1.0f;
        const float inv = __fdiv_rn(1.0f, scale);
        if (lane == 0) row_scales[r] = scale;
        if (vec) {
            const float4* x4 = reinterpret_cast<const float4*>(x);
            uint32_t* y4 = reinterpret_cast<uint32_t*>(y);
            for (int c = lane; c < dim / 4; c += 32) {
                const float4 v = __ldg(x4 + c);
                const float f[4] = {v.x, v.y, v.z, v.w};
                uint32_t packed = 0u;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float q = fminf(fmaxf(rintf(__fmul_rn(f[e], inv)), -127.0f), 127.0f);
                    packed |= (static_cast<uint32_t>(static_cast<int>(q)) & 0xffu) << (8 * e);
                }
                y4[c] = packed;
            }
        } else {
            for (int j = lane; j < dim; j += 32) {
                const float q = fminf(fmaxf(rintf(__fmul_rn(__ldg(x + j), inv)), -127.0f), 127.0f);
                y[j] = static_cast<int8_t>(q);
            }
        }
    }
}

// Bit b of word w = dimension 32 w + b, set when the value is >= 0 (src/cuda/convert.cu:34-53).
__global__ void pack_binary_kernel(const float* __restrict__ src, uint32_t* __restrict__ dst, long long rows, int dim,
                                   int words) {
    const long long total = rows * words;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = i / words;
        const int w = static_cast<int>(i - r * words);
        const float* x = src + r * dim;
        uint32_t bits = 0u;
        for (int b = 0; b < 32; ++b) {
            const int d = 32 * w + b;
            if (d < dim && x[d] >= 0.0f) bits |= 1u << b;
        }
        dst[i] = bits;
    }
}

// out[q][j] = candidates[q][local[q][j]] for a valid position, else -1 (src/cuda/rescore.cu:65-79).
__global__ void remap_kernel(const int* __restrict__ candidates, const int* __restrict__ local, int m, int k,
                             int* __restrict__ out) {
    const int q = blockIdx.y;
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < k; j += gridDim.x * blockDim.x) {
        const size_t at = static_cast<size_t>(q) * k + j;
        const int l = local[at];
        out[at] = (l >= 0 && l < m) ? candidates[static_cast<size_t>(q) * m + l] : -1;
    }
}

int grid_for(size_t work) {
    const size_t blocks = (work + kConvertThreads - 1) / kConvertThreads;
    return static_cast<int>(std::max<size_t>(1, std::min<size_t>(blocks, 16u * static_cast<unsigned>(device_sm_count()))));
}

int launched(const char* what) {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ok() : fail_cuda(e, what);
}

}  // namespace
}  // namespace zc

extern "C" {

int zcgvs_topk(const float* scores, int64_t doc_count, int k, int batch, int* out_indices, float* out_scores,
               void* stream) {
    using namespace zc;
    if (k <= 0 || doc_count <= 0 || batch <= 0) return ok();
    if (k > ZCGVS_MAX_K) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs top-k: k=" + std::to_string(k) + " exceeds per-tile capacity " +
                                               std::to_string(ZCGVS_MAX_K));
    }
    if (k > doc_count) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs top-k: k=" + std::to_string(k) + " exceeds candidate count " +
                                               std::to_string(doc_count));
    }
    if (doc_count > INT_MAX) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs top-k: more candidates than int32 ids");
    if (scores == nullptr || out_indices == nullptr || out_scores == nullptr) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs top-k: null pointer");
    }
    // CTAs per row: enough to spread one long row over several SMs, at least 4096 scores each.
    const int C = static_cast<int>(std::max<long long>(1, std::min<long long>(kRowMaxCluster, doc_count / 4096)));
    const int slice = static_cast<int>((doc_count + C - 1) / C);
    const int cap = std::max(kRowCap, next_pow2(C * k));
    const size_t smem = static_cast<size_t>(cap) * sizeof(u64);
    const cudaError_t opt = ensure_smem_optin(reinterpret_cast<const void*>(topk_rows_kernel));
    if (opt != cudaSuccess) return fail_cuda(opt, "cudaFuncSetAttribute(topk_rows_kernel)");
    constexpr int kMaxY = 65535;
    for (int q0 = 0; q0 < batch; q0 += kMaxY) {
        const int nq = std::min(kMaxY, batch - q0);
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(static_cast<unsigned>(C), static_cast<unsigned>(nq));
        cfg.blockDim = dim3(kRowThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = static_cast<cudaStream_t>(stream);
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = static_cast<unsigned>(C);
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const cudaError_t e = cudaLaunchKernelEx(&cfg, topk_rows_kernel, scores + static_cast<size_t>(q0) * doc_count,
                                                 static_cast<long long>(doc_count), k, slice, cap,
                                                 out_indices + static_cast<size_t>(q0) * k,
                                                 out_scores + static_cast<size_t>(q0) * k);
        if (e != cudaSuccess) return fail_cuda(e, "topk_rows_kernel launch");
    }
    return ok();
}

int zcgvs_convert_f16(const float* src, void* dst_half, size_t count, void* stream) {
    using namespace zc;
    if (count == 0) return ok();
    if (src == nullptr || dst_half == nullptr) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_convert_f16: null pointer");
    convert_f16_kernel<<<grid_for(count), kConvertThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        src, static_cast<__half*>(dst_half), count);
    return launched("convert_f16_kernel launch");
}

int zcgvs_convert_i8(const float* src, void* dst_int8, size_t count, float scale, void* stream) {
    using namespace zc;
    if (count == 0) return ok();
    if (src == nullptr || dst_int8 == nullptr) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_convert_i8: null pointer");
    const float inv = scale > 0.0f ? 1.0f / scale : 0.0f;
    convert_i8_kernel<<<grid_for(count), kConvertThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        src, static_cast<int8_t*>(dst_int8), count, inv);
    return launched("convert_i8_kernel launch");
}

int zcgvs_convert_i8_rows(const float* src, void* dst_int8, float* row_scales, int64_t rows, int dim, void* stream) {
    using namespace zc;
    if (rows <= 0 || dim <= 0) return ok();
    if (src == nullptr || dst_int8 == nullptr || row_scales == nullptr) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_convert_i8_rows: null pointer");
    }
    const int vec = (dim % 4 == 0 && reinterpret_cast<uintptr_t>(src) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(dst_int8) % 4 == 0) ? 1 : 0;
    const long long blocks = (rows + kConvertThreads / 32 - 1) / (kConvertThreads / 32);
    const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>(blocks, 16LL * device_sm_count())));
    convert_i8_rows_kernel<<<grid, kConvertThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        src, static_cast<int8_t*>(dst_int8), row_scales, rows, dim, vec);
    return launched("convert_i8_rows_kernel launch");
}

int zcgvs_pack_binary(const float* src, void* dst_words, int64_t rows, int dim, void* stream) {
    using namespace zc;
    if (rows <= 0 || dim <= 0) return ok();
    if (src == nullptr || dst_words == nullptr) return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_pack_binary: null pointer");
    const int words = (dim + 31) / 32;
    pack_binary_kernel<<<grid_for(static_cast<size_t>(rows) * words), kConvertThreads, 0,
                         static_cast<cudaStream_t>(stream)>>>(src, static_cast<uint32_t*>(dst_words), rows, dim,
                                                              words);
    return launched("pack_binary_kernel launch");
}

int zcgvs_remap_indices(const int* candidates, const int* local_indices, int candidate_count, int k, int batch,
                        int* out_indices, void* stream) {
    using namespace zc;
    if (k <= 0 || batch <= 0) return ok();
    if (candidates == nullptr || local_indices == nullptr || out_indices == nullptr) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_remap_indices: null pointer");
    }
    const dim3 grid(static_cast<unsigned>((k + 255) / 256), static_cast<unsigned>(batch));
    remap_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(candidates, local_indices, candidate_count, k,
                                                                      out_indices);
    return launched("remap_kernel launch");
}

}  // extern "C"
