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

// One CTA per query. Entry i of list p is at p * list_stride + q * k_in + i in both arrays;
// its id becomes id + id_offset[p] (when id_offset is given; padding ids < 0 stay padding).
// Writes the first k keys as (id, score) to out_idx / out_scores (either may be null) and, when
// out_owned is given, the id - own_begin of each selected id in [own_begin, own_end), -1 for
// the others (the candidates this rank's shard holds, as row numbers of the shard).
__global__ void __launch_bounds__(kMergeThreads) merge_lists_kernel(const int* __restrict__ idx,
                                                                    const float* __restrict__ scores,
                                                                    long long list_stride, int lists, int k_in, int k,
                                                                    int cap, const int* __restrict__ id_offset,
                                                                    int* __restrict__ out_idx,
                                                                    float* __restrict__ out_scores, int own_begin,
                                                                    int own_end, int* __restrict__ out_owned) {
    extern __shared__ __align__(16) u64 keys[];
    __shared__ int s_count;
    __shared__ u64 s_thr;
    const int q = blockIdx.x;
    const int n = lists * k_in;
    for (int i = threadIdx.x; i < cap; i += kMergeThreads) {
        u64 key = 0ull;
        if (i < n) {
            const int p = i / k_in;
            const size_t at = static_cast<size_t>(p) * list_stride + static_cast<size_t>(q) * k_in + (i - p * k_in);
            int id = __ldg(idx + at);
            if (id >= 0) {
                if (id_offset != nullptr) id += __ldg(id_offset + p);
                key = make_key(__ldg(scores + at), static_cast<uint32_t>(id));
            }
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
    const size_t row = static_cast<size_t>(q) * k;
    if (out_idx != nullptr && out_scores != nullptr) topk_write(t, 0, out_idx + row, out_scores + row, kMergeThreads);
    if (out_owned != nullptr) {
        const int kept = s_count;
        for (int j = threadIdx.x; j < k; j += kMergeThreads) {
            const int id = j < kept ? key_id(keys[j]) : -1;
            out_owned[row + j] = (id >= own_begin && id < own_end) ? id - own_begin : -1;
        }
    }
}

int launch_merge(const int* idx, const float* scores, long long list_stride, int lists, int batch, int k_in, int k,
                 const int* id_offset, int* out_idx, float* out_scores, int own_begin, int own_end, int* out_owned,
                 cudaStream_t stream) {
    const int cap = next_pow2(std::max(lists * k_in, 2));
    const cudaError_t opt = ensure_smem_optin(reinterpret_cast<const void*>(merge_lists_kernel));
    if (opt != cudaSuccess) return fail_cuda(opt, "cudaFuncSetAttribute(merge_lists_kernel)");
    {
        KernelTimer timer("merge", stream);
        merge_lists_kernel<<<batch, kMergeThreads, static_cast<size_t>(cap) * 8, stream>>>(
            idx, scores, list_stride, lists, k_in, k, cap, id_offset, out_idx, out_scores, own_begin, own_end,
            out_owned);
    }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ok() : fail_cuda(e, "merge_lists_kernel launch");
}

int check_merge(int lists, int k_in, int k, const char* name) {
    if (k <= 0 || k > ZCGVS_MAX_K) {
        return fail(ZCGVS_ERR_INVALID_ARG, std::string(name) + ": k must be in [1, " + std::to_string(ZCGVS_MAX_K) + "]");
    }
    if (static_cast<long long>(lists) * k_in > kMergeMaxEntries) {
        return fail(ZCGVS_ERR_INVALID_ARG, std::string(name) + ": lists * k_in exceeds " + std::to_string(kMergeMaxEntries));
    }
    return ZCGVS_OK;
}

}  // namespace
}  // namespace zc

extern "C" {

int zcgvs_merge_topk(const int* list_indices, const float* list_scores, int lists, int batch, int k_in, int k,
                     int* out_indices, float* out_scores, void* stream) {
    using namespace zc;
    if (lists <= 0 || batch <= 0 || k_in <= 0) return ok();
    const int status = check_merge(lists, k_in, k, "zcgvs_merge_topk");
    if (status != ZCGVS_OK) return status;
    if (list_indices == nullptr || list_scores == nullptr || out_indices == nullptr || out_scores == nullptr) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_merge_topk: null pointer");
    }
    return launch_merge(list_indices, list_scores, static_cast<long long>(batch) * k_in, lists, batch, k_in, k, nullptr,
                        out_indices, out_scores, 0, 0, nullptr, static_cast<cudaStream_t>(stream));
}

int zcgvs_merge_topk_lists(const int* list_indices, const float* list_scores, int64_t list_stride, int lists,
                           int batch, int k_in, const int* list_id_offsets, int k, int* out_indices, float* out_scores,
                           int own_begin, int own_end, int* out_owned, void* stream) {
    using namespace zc;
    if (lists <= 0 || batch <= 0 || k_in <= 0) return ok();
    const int status = check_merge(lists, k_in, k, "zcgvs_merge_topk_lists");
    if (status != ZCGVS_OK) return status;
    if (list_indices == nullptr || list_scores == nullptr) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_merge_topk_lists: null list pointer");
    }
    if ((out_indices == nullptr) != (out_scores == nullptr) || (out_indices == nullptr && out_owned == nullptr)) {
        return fail(ZCGVS_ERR_INVALID_ARG,
                    "zcgvs_merge_topk_lists: give out_indices and out_scores together, out_owned, or both");
    }
    if (list_stride < static_cast<int64_t>(batch) * k_in) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_merge_topk_lists: list_stride is smaller than batch * k_in");
    }
    if (out_owned != nullptr && own_begin > own_end) {
        return fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_merge_topk_lists: own_begin exceeds own_end");
    }
    return launch_merge(list_indices, list_scores, list_stride, lists, batch, k_in, k, list_id_offsets, out_indices,
                        out_scores, own_begin, own_end, out_owned, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
