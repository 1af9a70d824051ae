// zcgvs_merge_topk: the global top-k of per-shard top-k lists.
//
// A row-sharded search (each GPU scans N / P rows with id_base = its first row) ends with P
// [batch, k_in] candidate lists per query, exchanged with one NCCL all-gather. This kernel merges
// them on the device: one CTA per query turns the P * k_in (id, score) entries into 64-bit keys
// (score desc, id asc; padding ids < 0 are dropped), sorts them in shared memory and writes the
// first k. Because the global top-k is contained in the union of the per-shard top-k lists and
// the order is total, the result equals a single-GPU search over the whole corpus.
//
// The reference has no multi-GPU path; its single-GPU merge step is mergeTopKKernel
// (src/cuda/topk.cu:76-115), which merges tiles of one score row in the same way.
#include <cuda_runtime.h>

#include <algorithm>
#include <string>

#include "common.cuh"
#include "host_common.h"
#include "topk_cta.cuh"
#include "zcgvs_sm100.h"

namespace zc {

namespace {

constexpr int kMergeThreads = 512;
constexpr int kMergeMaxEntries = 16384;  // 128 KB of keys

__global__ void __launch_bounds__(kMergeThreads) merge_lists_kernel(const int* __restrict__ idx,
                                                                    const float* __restrict__ scores, int lists,
                                                                    int batch, int k_in, int k, int cap,
                                                                    int* __restrict__ out_idx,
                                                                    float* __restrict__ out_scores) {
    extern __shared__ __align__(16) u64 keys[];
    __shared__ int s_count;
    __shared__ u64 s_thr;
    const int q = blockIdx.x;
    const int n = lists * k_in;
    for (int i = threadIdx.x; i < cap; i += kMergeThreads) {
        u64 key = 0ull;
        if (i < n) {
            const int p = i / k_in;
            const size_t at = (static_cast<size_t>(p) * batch + q) * k_in + (i - p * k_in);
            const int id = __ldg(idx + at);
            if (id >= 0) key = make_key(__ldg(scores + at), static_cast<uint32_t>(id));
        }
        keys[i] = key;
    }
    TopkSmem t;
    t.buf = keys;
    t.count = &s_count;
    t.thr = &s_thr;
    t.cap = cap;
    t.k = k;
    if (threadIdx.x == 0) s_count = n;
    __syncthreads();
    topk_flush_mask(t, 1u, kMergeThreads);
    __syncthreads();
    topk_write(t, 0, out_idx + static_cast<size_t>(q) * k, out_scores + static_cast<size_t>(q) * k, kMergeThreads);
}

}  // namespace
}  // namespace zc

extern "C" {

int zcgvs_merge_topk(const int* list_indices, const float* list_scores, int lists, int batch, int k_in, int k,
                     int* out_indices, float* out_scores, void* stream) {
    using namespace zc;
    if (lists <= 0 || batch <= 0 || k_in <= 0) return ok();
    if (k <= 0 || k > ZCGVS_MAX_K) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_merge_topk: k must be in [1, " + std::to_string(ZCGVS_MAX_K) + "]");
    }
    if (static_cast<long long>(lists) * k_in > kMergeMaxEntries) {
        return fail(ZCGVS_ERR_INVALID_ARG,
                    "zcgvs_merge_topk: lists * k_in exceeds " + std::to_string(kMergeMaxEntries));
    }
    if (list_indices == nullptr || list_scores == nullptr || out_indices == nullptr || out_scores == nullptr) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_merge_topk: null pointer");
    }
    const int cap = next_pow2(std::max(lists * k_in, 2));
    const cudaError_t opt = ensure_smem_optin(reinterpret_cast<const void*>(merge_lists_kernel));
    if (opt != cudaSuccess) return fail_cuda(opt, "cudaFuncSetAttribute(merge_lists_kernel)");
    {
        KernelTimer timer("merge", static_cast<cudaStream_t>(stream));
        merge_lists_kernel<<<batch, kMergeThreads, static_cast<size_t>(cap) * 8,
                             static_cast<cudaStream_t>(stream)>>>(list_indices, list_scores, lists, batch, k_in, k,
                                                                  cap, out_indices, out_scores);
    }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ok() : fail_cuda(e, "merge_lists_kernel launch");
}

}  // extern "C"
