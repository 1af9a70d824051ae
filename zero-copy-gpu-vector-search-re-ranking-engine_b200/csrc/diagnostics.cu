// zcgvs_check_bounded_wait: runs the failure path of the library's bounded waits on the GPU.
//
// Every wait of a kernel here (a corpus tile's copy, an accumulator hand-off, the drain of
// copies in flight) is bounded by kWaitBudgetNs of %globaltimer; when it runs out the kernel
// sets a bit in the workspace status word, stops issuing and returns. This diagnostic makes
// one such wait run out on purpose without any fault: one thread initialises a shared-memory
// mbarrier expecting one arrival that nobody makes, and waits on it with the same helper the
// scan kernels use. Nothing is in flight, so after the budget the thread records
// kStatusTileWaitTimeout and the kernel ends normally; the host then reads the status word as
// a caller would after a real timeout.
#include <cuda_runtime.h>

#include "common.cuh"
#include "host_common.h"
#include "zcgvs_sm100.h"

namespace zc {
namespace {

static_assert(kStatusTileWaitTimeout == ZCGVS_DEVICE_TILE_WAIT_TIMEOUT && kStatusDrainTimeout == ZCGVS_DEVICE_DRAIN_TIMEOUT,
              "device status bits must match the header");

__global__ void unfinished_wait_kernel(uint32_t* status) {
    __shared__ __align__(8) u64 bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1u);
    fence_mbarrier_init();
    // Phase 0 never completes (no arrival): the bounded wait gives up and records the timeout.
    mbar_wait_bounded(&bar, 0u, status, kStatusTileWaitTimeout);
}

}  // namespace
}  // namespace zc

extern "C" {

int zcgvs_check_bounded_wait(void* workspace, size_t bytes, void* stream) {
    if (workspace == nullptr || bytes < sizeof(uint32_t) || (reinterpret_cast<uintptr_t>(workspace) & 3u) != 0) {
        return zc::fail(ZCGVS_ERR_INVALID_ARG, "zcgvs_check_bounded_wait: needs a 4-byte aligned workspace");
    }
    zc::unfinished_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint32_t*>(workspace));
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? zc::ok() : zc::fail_cuda(e, "unfinished_wait_kernel launch");
}

}  // extern "C"
