// CUDA error reporting of the C++ interface: the same class and macros as the reference
// (include/zcgvs/core/cuda_check.hpp:10-37), so code written against it compiles unchanged.
#pragma once

#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

namespace zcgvs {

// A failed CUDA runtime call: the error code and where it happened.
class CudaError : public std::runtime_error {
public:
    CudaError(cudaError_t code, const char* expr, const char* file, int line)
        : std::runtime_error(describe(code, expr, file, line)), code_(code) {}

    cudaError_t code() const noexcept { return code_; }

private:
    static std::string describe(cudaError_t code, const char* expr, const char* file, int line) {
        std::string text = "CUDA error ";
        text += cudaGetErrorName(code);
        text += " (";
        text += cudaGetErrorString(code);
        text += ") from `";
        text += expr;
        text += "` at ";
        text += file;
        text += ":" + std::to_string(line);
        return text;
    }

    cudaError_t code_;
};

}  // namespace zcgvs

#define ZCGVS_CUDA_CHECK(expr)                                                   \
    do {                                                                         \
        const cudaError_t zcgvs_status_ = (expr);                                \
        if (zcgvs_status_ != cudaSuccess) {                                      \
            throw ::zcgvs::CudaError(zcgvs_status_, #expr, __FILE__, __LINE__);  \
        }                                                                        \
    } while (0)

#define ZCGVS_CUDA_CHECK_LAST() ZCGVS_CUDA_CHECK(cudaGetLastError())
