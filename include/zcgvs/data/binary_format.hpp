// On-disk formats shared with the reference's tools (include/zcgvs/data/binary_format.hpp:12-101;
// written by python/zcgvs_tools/formats.py): the constants of the three files and a small
// little-endian reader. The byte layouts must stay identical so files move between the two
// libraries; only version 3 of the embedding file (per-row int8, dtype 4, a trailing [N] fp32
// row-scale block) is new here.
//
//   ZCVE embeddings : magic, u32 version, u32 flags (bit 0: rows L2-normalised), i64 N, i32 dim,
//                     i32 dtype; version >= 2 adds f32 scale and i32 row stride; then N rows of
//                     row-stride bytes; version 3 (dtype 4 only) then N fp32 row scales.
//   ZCVM metadata   : magic, u32 version, i64 N, then per document u32 length + UTF-8 id and
//                     u32 length + UTF-8 passage text, in corpus order.
//   ZCVL lexical    : magic, u32 version, i64 N, i32 vocabulary V, i64 postings P, f32 k1, f32 b,
//                     f32 average document length, [V + 1] i64 CSR offsets, [P] i32 documents,
//                     [P] f32 BM25 weights.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <istream>
#include <stdexcept>
#include <string>

namespace zcgvs {

constexpr char kEmbeddingMagic[4] = {'Z', 'C', 'V', 'E'};
constexpr char kMetadataMagic[4] = {'Z', 'C', 'V', 'M'};
constexpr char kLexicalMagic[4] = {'Z', 'C', 'V', 'L'};

// Version the writers emit for the reference's dtypes; per-row int8 files are version 3.
constexpr std::uint32_t kEmbeddingVersion = 2;
constexpr std::uint32_t kEmbeddingVersionRowScales = 3;
constexpr std::uint32_t kMetadataVersion = 1;
constexpr std::uint32_t kLexicalVersion = 1;

constexpr std::uint32_t kFlagNormalized = 1u;

constexpr std::int32_t kDtypeFloat32 = 0;
constexpr std::int32_t kDtypeFloat16 = 1;
constexpr std::int32_t kDtypeInt8 = 2;
constexpr std::int32_t kDtypeBinary = 3;
constexpr std::int32_t kDtypeInt8PerRow = 4;  // extension: int8 rows with one fp32 scale each

// Reads the little-endian fields of the formats above from a stream; any short read throws
// std::runtime_error.
class BinaryReader {
public:
    explicit BinaryReader(std::istream& stream) : in_(stream) {}

    template <typename T>
    T readScalar() {
        T value{};
        readBytes(reinterpret_cast<char*>(&value), sizeof(value));
        return value;
    }

    void readBytes(char* destination, std::size_t count) {
        if (count == 0) return;
        in_.read(destination, static_cast<std::streamsize>(count));
        if (in_.gcount() != static_cast<std::streamsize>(count)) {
            throw std::runtime_error("zcgvs binary: the stream ended before the expected field");
        }
    }

    std::string readString(std::size_t length) {
        std::string text(length, '\0');
        readBytes(text.data(), length);
        return text;
    }

    void expectMagic(const char (&expected)[4]) {
        char found[4] = {};
        readBytes(found, sizeof(found));
        if (std::memcmp(found, expected, sizeof(found)) != 0) {
            throw std::runtime_error("zcgvs binary: the file does not start with the expected magic");
        }
    }

private:
    std::istream& in_;
};

}  // namespace zcgvs
