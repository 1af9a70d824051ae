// Store converters (the reference's include/zcgvs/cuda/convert.cuh:10-20), implemented over
// zcgvs_convert_f16 / zcgvs_convert_i8 / zcgvs_pack_binary (+ zcgvs_convert_i8_rows).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace zcgvs {
namespace cuda {

void launchConvertF32ToF16(const float* src, void* dst_half, std::size_t count, cudaStream_t stream);
void launchConvertF32ToI8(const float* src, void* dst_int8, std::size_t count, float scale, cudaStream_t stream);
void launchPackBinary(const float* src, void* dst_words, int rows, int dim, cudaStream_t stream);
// Extension: per-row int8 (scale = max|x| / 127 per row into row_scales) for Int8PerRow stores.
void launchConvertF32ToI8Rows(const float* src, void* dst_int8, float* row_scales, std::int64_t rows, int dim,
                              cudaStream_t stream);

}  // namespace cuda
}  // namespace zcgvs
