// An owned CUDA stream (move-only), the reference's CudaStream
// (include/zcgvs/core/cuda_stream.hpp).
#pragma once

#include <cuda_runtime.h>

#include <utility>

#include "zcgvs/core/cuda_check.hpp"

namespace zcgvs {

class CudaStream {
public:
    CudaStream() { ZCGVS_CUDA_CHECK(cudaStreamCreate(&stream_)); }
    ~CudaStream() { reset(); }

    CudaStream(const CudaStream&) = delete;
    CudaStream& operator=(const CudaStream&) = delete;
    CudaStream(CudaStream&& other) noexcept : stream_(std::exchange(other.stream_, nullptr)) {}
    CudaStream& operator=(CudaStream&& other) noexcept {
        if (this != &other) {
            reset();
            stream_ = std::exchange(other.stream_, nullptr);
        }
        return *this;
    }

    cudaStream_t get() const noexcept { return stream_; }
    void synchronize() const { ZCGVS_CUDA_CHECK(cudaStreamSynchronize(stream_)); }

private:
    void reset() noexcept {
        if (stream_ != nullptr) cudaStreamDestroy(stream_);
        stream_ = nullptr;
    }

    cudaStream_t stream_ = nullptr;
};

}  // namespace zcgvs
