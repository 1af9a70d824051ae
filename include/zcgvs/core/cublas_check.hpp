// cuBLAS error reporting with the reference's interface (include/zcgvs/core/cublas_check.hpp):
// CublasError carries the failed status and ZCGVS_CUBLAS_CHECK throws it. Used only by the
// cuBLAS yardstick (zcgvs/cuda/cublas_similarity.hpp), never on the search path.
#pragma once

#include <cublas_v2.h>

#include <stdexcept>
#include <string>

namespace zcgvs {

class CublasError : public std::runtime_error {
public:
    CublasError(cublasStatus_t status, const char* expr, const char* file, int line)
        : std::runtime_error(std::string("cuBLAS error ") + cublasGetStatusName(status) + " (" +
                             cublasGetStatusString(status) + ") from `" + expr + "` at " + file + ":" +
                             std::to_string(line)),
          status_(status) {}

    cublasStatus_t status() const noexcept { return status_; }

private:
    cublasStatus_t status_;
};

}  // namespace zcgvs

#define ZCGVS_CUBLAS_CHECK(expr)                                                        \
    do {                                                                                \
        const cublasStatus_t zcgvs_cublas_status_ = (expr);                             \
        if (zcgvs_cublas_status_ != CUBLAS_STATUS_SUCCESS) {                            \
            throw ::zcgvs::CublasError(zcgvs_cublas_status_, #expr, __FILE__, __LINE__); \
        }                                                                               \
    } while (0)
