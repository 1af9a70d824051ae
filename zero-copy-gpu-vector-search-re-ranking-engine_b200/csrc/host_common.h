// Host-side helpers shared by the C-ABI entry points: error reporting, per-device attribute
// caches and the shared-memory opt-in of each kernel.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>

#include "zcgvs_sm100.h"

namespace zc {

// Records `message` as the thread's last error and returns `status`.
int fail(int status, const std::string& message);

// Maps a CUDA error to ZCGVS_ERR_CUDA with a message naming `what`.
int fail_cuda(cudaError_t error, const char* what);

// Clears the thread's last error and returns ZCGVS_OK.
int ok();

// Streaming multiprocessor count of the current device (cached per device).
int device_sm_count();

// Largest dynamic shared memory one CTA may opt into on the current device (cached).
int device_max_smem();

// Opts `kernel` into the largest dynamic shared memory the device allows next to its static
// shared memory, once per device.
cudaError_t ensure_smem_optin(const void* kernel);

// CUDA-event timing of one kernel launch under a tag (a diagnostics switch, off by default):
// when zcgvs_kernel_timing(1) is on, the constructor records an event on `stream` before the
// launch and the destructor one after it; zcgvs_kernel_timing_read sums them per tag.
class KernelTimer {
   public:
    KernelTimer(const char* tag, cudaStream_t stream);
    ~KernelTimer();
    KernelTimer(const KernelTimer&) = delete;
    KernelTimer& operator=(const KernelTimer&) = delete;

   private:
    int slot_ = -1;
    cudaStream_t stream_ = nullptr;
};

inline std::size_t round_up(std::size_t value, std::size_t to) {
    return (value + to - 1) / to * to;
}

inline int next_pow2(int value) {
    int p = 1;
    while (p < value) p <<= 1;
    return p;
}

// Bytes of one stored row (include/zcgvs/core/scalar_type.hpp:27-39; I8_ROW stores int8).
inline long long row_bytes_of(int dtype, int dim) {
    switch (dtype) {
        case ZCGVS_DTYPE_F32: return 4LL * dim;
        case ZCGVS_DTYPE_F16: return 2LL * dim;
        case ZCGVS_DTYPE_I8:
        case ZCGVS_DTYPE_I8_ROW: return dim;
        case ZCGVS_DTYPE_BINARY: return 4LL * ((dim + 31) / 32);
        default: return -1;
    }
}

}  // namespace zc
