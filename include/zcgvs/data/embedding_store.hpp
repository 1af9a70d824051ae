// A device-resident corpus (the reference's EmbeddingStore,
// include/zcgvs/data/embedding_store.hpp:17-54): row-major [docCount, rowStride] bytes in the
// storage precision, loaded from a ZCVE file or converted on the device from a host fp32 matrix.
// Int8PerRow stores also hold [docCount] fp32 row scales (ZCVE version 3).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>

#include "zcgvs/core/device_buffer.hpp"
#include "zcgvs/core/scalar_type.hpp"

namespace zcgvs {

class EmbeddingStore {
public:
    EmbeddingStore() = default;

    // ZCVE v1 (fp32 / fp16), v2 (any reference dtype, with scale and stride) or v3 (v2 plus
    // Int8PerRow, whose [N] fp32 row scales follow the matrix) file. The payload streams through
    // two pinned staging chunks straight into device memory.
    static EmbeddingStore loadFromFile(const std::string& path);

    // Converts a host fp32 matrix on the device. `scale` is the int8 per-matrix scale (values
    // <= 0 mean 1; Int8PerRow derives one scale per row); `normalized` only records whether rows
    // are unit length.
    static EmbeddingStore fromHostMatrix(const float* host_float32, std::int64_t doc_count, int dim,
                                         ScalarType dtype, float scale, bool normalized);

    const void* deviceData() const { return device_.data(); }
    std::int64_t docCount() const { return doc_count_; }
    int dim() const { return dim_; }
    bool normalized() const { return normalized_; }
    ScalarType dtype() const { return dtype_; }
    float scale() const { return scale_; }
    // [docCount] fp32 row scales of an Int8PerRow store, nullptr for the other dtypes.
    const float* rowScales() const { return dtype_ == ScalarType::Int8PerRow ? row_scales_.data() : nullptr; }
    std::int64_t capacity() const { return capacity_; }
    std::size_t deviceBytes() const { return device_.bytes(); }
    std::size_t rowStride() const { return rowBytes(dtype_, dim_); }

    // Appends host fp32 rows (converted on `stream`), growing the allocation geometrically.
    void append(const float* host_float32, std::int64_t add_count, cudaStream_t stream);

private:
    void ensureCapacity(std::int64_t required_docs, cudaStream_t stream);
    void convertInto(std::uint8_t* destination, float* row_scales, const float* device_float32, std::int64_t rows,
                     cudaStream_t stream);

    DeviceBuffer<std::uint8_t> device_;
    DeviceBuffer<float> row_scales_;
    std::int64_t doc_count_ = 0;
    std::int64_t capacity_ = 0;
    int dim_ = 0;
    bool normalized_ = false;
    ScalarType dtype_ = ScalarType::Float32;
    float scale_ = 1.0f;
};

}  // namespace zcgvs
