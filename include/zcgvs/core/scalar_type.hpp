// Storage precision of a corpus. The codes equal the reference ScalarType
// (include/zcgvs/core/scalar_type.hpp:12-17), the ZCVE dtype field and the C ABI's zcgvs_dtype,
// so static_cast<int> converts between them. Int8PerRow (code 4) is this library's extension:
// int8 rows with one fp32 scale per row (ZCVE version 3 files, ZCGVS_DTYPE_I8_ROW).
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

namespace zcgvs {

enum class ScalarType : std::int32_t { Float32 = 0, Float16 = 1, Int8 = 2, Binary = 3, Int8PerRow = 4 };

inline bool isQuantized(ScalarType type) {
    return type == ScalarType::Int8 || type == ScalarType::Binary || type == ScalarType::Int8PerRow;
}

// 32-bit words of one sign-bit row.
inline std::size_t binaryWords(int dim) { return static_cast<std::size_t>((dim + 31) / 32); }

// Bytes of one stored row.
inline std::size_t rowBytes(ScalarType type, int dim) {
    const std::size_t d = static_cast<std::size_t>(dim);
    switch (type) {
        case ScalarType::Float16: return 2 * d;
        case ScalarType::Int8:
        case ScalarType::Int8PerRow: return d;
        case ScalarType::Binary: return 4 * binaryWords(dim);
        case ScalarType::Float32:
        default: return 4 * d;
    }
}

inline const char* scalarName(ScalarType type) {
    switch (type) {
        case ScalarType::Float16: return "float16";
        case ScalarType::Int8: return "int8";
        case ScalarType::Binary: return "binary";
        case ScalarType::Int8PerRow: return "int8_row";
        case ScalarType::Float32:
        default: return "float32";
    }
}

// Accepted spellings as in the reference's configs; anything else is float32.
inline ScalarType scalarTypeFromName(const std::string& name) {
    if (name == "float16" || name == "fp16" || name == "half") return ScalarType::Float16;
    if (name == "int8" || name == "i8") return ScalarType::Int8;
    if (name == "binary" || name == "bin" || name == "b1") return ScalarType::Binary;
    if (name == "int8_row" || name == "int8_per_row") return ScalarType::Int8PerRow;
    return ScalarType::Float32;
}

}  // namespace zcgvs
