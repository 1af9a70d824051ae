// zcgvs_scan_topk_noalloc: the fused scan + top-k for callers that cannot allocate device
// memory.
//
// Some hosts of this library own every byte of device memory themselves: a serving process
// that budgets its GPU memory up front and forbids plug-ins from calling cudaMalloc, or a
// latency-critical path where cudaMalloc/cudaFree (which can synchronise the device) are not
// allowed. Such a caller cannot provide the workspace zcgvs_scan_topk asks for. This entry
// point takes the same inputs and outputs but no workspace: its scratch lives in one
// file-scope __device__ array of a fixed size (kNoAllocScratchBytes) that the CUDA module
// reserves on every GPU that loads this library, for as long as the library stays loaded.
//
// Set-up: the first call on a device looks up that device's address of the array with
// cudaGetSymbolAddress (with that device current) and caches it; that first call should
// therefore come before any stream capture. The library's modules load lazily (CUDA's default
// lazy loading), so the array is reserved on a device when that first lookup loads its module,
// not when the library is loaded: a host that wants the reservation made at start-up, before
// it takes the rest of the GPU's memory, calls zcgvs_scan_topk_noalloc_status (or this entry
// point with a zero-sized problem) once per device then.
//
// Sharing: every call on a device uses the same array, which keeps the last call's contents.
// Each call clears the part that must start at zero (status word and merge counters) on its
// own stream before launching. Calls whose kernels overlap on the GPU (other streams, other
// threads) race on the array; callers must serialise them.
//
// Status: the array's first 4 bytes are the status word every kernel of a call writes (a
// bounded wait that ran out, a candidate buffer that overflowed; the ZCGVS_DEVICE_* bits).
// zcgvs_scan_topk_noalloc_status copies it to the host after a call; the next call clears it.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "host_common.h"
#include "zcgvs_sm100.h"

namespace {

// 32 MiB: enough for one query over ~4M rows, or small batches over ~1M rows (the same
// layout zcgvs_scan_topk_workspace_bytes() describes).
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device, looked up once per device.
int scratch_address(void** out) {
    int device = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status != cudaSuccess) return zc::fail_cuda(status, "cudaGetDevice");
    if (device < 0 || device >= kMaxDevices) {
        return zc::fail(ZCGVS_ERR_UNSUPPORTED, "zcgvs: device ordinal beyond the no-alloc table");
    }
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (g_scratch_ptr[device] == nullptr) {
        void* ptr = nullptr;
        status = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (status != cudaSuccess) return zc::fail_cuda(status, "cudaGetSymbolAddress(no-alloc scratch)");
        g_scratch_ptr[device] = ptr;
    }
    *out = g_scratch_ptr[device];
    return ZCGVS_OK;
}

}  // namespace

extern "C" {

int zcgvs_scan_topk_noalloc(const void* corpus, int dtype, float scale, const float* row_scales,
                            int64_t doc_count, int dim, const float* queries, int batch,
                            const uint8_t* mask, int metric, int k, int id_base, int* out_indices,
                            float* out_scores, void* stream) {
    if (doc_count <= 0 || batch <= 0 || dim <= 0) {
        // Nothing to search; the scratch address is still resolved, so a zero-sized call at
        // start-up reserves the array on this device (see the set-up note above).
        void* scratch = nullptr;
        return scratch_address(&scratch);
    }
    const size_t need = zcgvs_scan_topk_workspace_bytes(dtype, doc_count, dim, batch, k);
    if (need > kNoAllocScratchBytes) {
        return zc::fail(ZCGVS_ERR_INVALID_ARG,
                        "zcgvs: this search needs " + std::to_string(need) +
                            " bytes of scratch, more than the " + std::to_string(kNoAllocScratchBytes) +
                            "-byte static area of zcgvs_scan_topk_noalloc; use zcgvs_scan_topk with a "
                            "caller-provided workspace");
    }
    void* scratch = nullptr;
    int status = scratch_address(&scratch);
    if (status != ZCGVS_OK) return status;
    // Status word and one merge counter per query pass (at most `batch` passes) start at zero.
    const size_t zeroed = zc::round_up(16 + 4 * static_cast<size_t>(batch), 256);
    const cudaError_t e = cudaMemsetAsync(scratch, 0, zeroed, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return zc::fail_cuda(e, "zcgvs_scan_topk_noalloc: clearing the scratch header");
    return zcgvs_scan_topk(corpus, dtype, scale, row_scales, doc_count, dim, queries, batch, mask, metric,
                           k, id_base, out_indices, out_scores, scratch, kNoAllocScratchBytes, stream);
}

int zcgvs_scan_topk_noalloc_status(uint32_t* status, void* stream) {
    if (status == nullptr) return zc::fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_scan_topk_noalloc_status: null status pointer");
    void* scratch = nullptr;
    const int rc = scratch_address(&scratch);
    if (rc != ZCGVS_OK) return rc;
    return zcgvs_workspace_status(scratch, kNoAllocScratchBytes, status, stream);
}

}  // extern "C"
